"""Rank program of tests/test_slices_gpu.py::test_sequence_parallel_two_gpus (launched by
torchrun, one rank per GPU, NCCL): the sequence-parallel scan of a batch-1 sequence split
over the ranks, against the unsliced scan of the whole sequence computed on every rank."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]

from helpers import assert_close, assert_grad_close  # noqa: E402
from ssm_mamba_b200.slices import SliceGroup, sliced_scan  # noqa: E402
from ssm_mamba_b200.workloads import scan_inputs  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L = 4096
    inp = scan_inputs(1, 256, L, 16, torch.float32, seed=21, device="cpu", with_z=True, with_h_init=True)
    dh = torch.randn(1, 256, 16, generator=torch.Generator().manual_seed(5))
    full = [t.to(dev) for t in (inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, inp.z, inp.delta_bias, inp.h_init)]
    dout, dh = inp.dout.to(dev), dh.to(dev)
    # whole sequence on this GPU, no slices
    ref = [t.clone().requires_grad_() for t in full]
    o_ref, h_ref = sliced_scan(*ref, delta_softplus=True, segments=1)
    ((o_ref * dout).sum() + (h_ref * dh).sum()).backward()
    # this rank's slice, 2 segments, carries over NCCL
    lo, hi = rank * L // world, (rank + 1) * L // world
    loc = []
    for i, t in enumerate(full):
        t = t[..., lo:hi].contiguous() if i in (0, 1, 3, 4, 6) else t
        loc.append(t.clone().requires_grad_())
    out, hf = sliced_scan(*loc, delta_softplus=True, segments=2, group=SliceGroup(dist.group.WORLD))
    loss = (out * dout[..., lo:hi]).sum() + ((hf * dh).sum() if rank == world - 1 else 0)
    loss.backward()
    assert_close(out, o_ref[..., lo:hi], 1e-4, 1e-5, "out")
    assert_close(hf, h_ref, 1e-4, 1e-5, "h_final")
    names = ["u", "delta", "A", "B", "C", "D", "z", "delta_bias", "h_init"]
    for i, name in enumerate(names):
        want = ref[i].grad
        if i in (0, 1, 3, 4, 6):
            want = want[..., lo:hi]
        if name == "h_init" and rank != 0:
            want = torch.zeros_like(want)
        assert_grad_close(loc[i].grad, want, name, rtol=1e-3)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("seqpar ok", flush=True)


if __name__ == "__main__":
    main()
