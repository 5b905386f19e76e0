"""Rank program of tests/test_slices_gpu.py::test_peer_leaving_is_detected_two_gpus
(torchrun, one rank per GPU, NCCL with NVLS off).  Both ranks run one sequence-parallel
scan step (forward + backward, slice carries over NCCL) with the host-side liveness check
of SliceGroup; then rank 1 leaves -- between steps, after a device synchronize, so none of
its kernels or collectives is in flight -- and rank 0 starts the next step.  Rank 0 must
learn of it on the host, before launching any collective of that step, and end with a clean
RuntimeError (exit code 3)."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT]

from ssm_mamba_b200.slices import SliceGroup, sliced_scan  # noqa: E402
from ssm_mamba_b200.workloads import scan_inputs  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    store = dist.PrefixStore("seqpar_failure", dist.distributed_c10d._get_default_store())
    group = SliceGroup(dist.group.WORLD, store=store, peer_timeout=datetime.timedelta(seconds=5))
    L = 4096
    inp = scan_inputs(1, 256, L, 16, torch.float32, seed=21, device="cpu", with_z=True)
    lo, hi = rank * L // world, (rank + 1) * L // world
    cut = lambda t: t[..., lo:hi].contiguous().to(dev)  # noqa: E731
    u, delta, B, C, z, dout = (cut(t) for t in (inp.u, inp.delta, inp.B, inp.C, inp.z, inp.dout))
    A, D, bias = (t.to(dev) for t in (inp.A, inp.D, inp.delta_bias))

    def step():
        leaves = [t.clone().requires_grad_() for t in (u, delta, A, B, C, D, z, bias)]
        out, _ = sliced_scan(*leaves, None, True, segments=2, group=group)
        out.backward(dout)

    step()
    torch.cuda.synchronize()
    print(f"rank {rank}: step 1 done", flush=True)
    if rank == 1:
        print("rank 1: leaving between steps", flush=True)
        os._exit(0)
    try:
        step()
        torch.cuda.synchronize()
        print("rank 0: UNEXPECTED: step 2 completed without its peer", flush=True)
        os._exit(1)
    except RuntimeError as e:
        print(f"rank 0: peer loss detected: {e}", flush=True)
        os._exit(3)


if __name__ == "__main__":
    main()
