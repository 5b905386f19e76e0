"""Sequence slices on the CPU: the orchestration of ssm_mamba_b200.slices (segment views,
carry bookkeeping, and the exchange between ranks over gloo, world size 2 and 4) run with
the CPU stand-ins of tests/slice_fakes.py, checked against the CPU oracle over the whole,
unsliced sequence.  The CUDA kernels behind the same entry points are covered by
tests/test_slices_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from helpers import np64
import oracle
from slice_fakes import FakeKernels
from ssm_mamba_b200.slices import SliceGroup, plan_segments, segment_view, sliced_scan

TOL = dict(rtol=1e-7, atol=1e-9)


def _inputs(L=256, D=6, N=4, seed=3, with_h=True):
    # float32 draws held in float64: the oracle helpers pass values through float32
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    u, delta, z, dout = rn(1, D, L), rn(1, D, L) * 0.5 - 1.0, rn(1, D, L), rn(1, D, L)
    B, C = rn(1, N, L), rn(1, N, L)
    A = -torch.rand(D, N, generator=g) * 2 - 0.1
    Dv, bias = rn(D), rn(D) * 0.25
    h0 = rn(1, D, N) * 0.5 if with_h else None
    dh = rn(1, D, N)
    x = dict(u=u, delta=delta, A=A, B=B, C=C, D=Dv, z=z, bias=bias, h0=h0, dout=dout, dh=dh)
    return {k: (v.double() if v is not None else None) for k, v in x.items()}


def _oracle(x):
    fw = oracle.scan_fwd(np64(x["u"]), np64(x["delta"]), np64(x["A"]), np64(x["B"]), np64(x["C"]),
                         D=np64(x["D"]), z=np64(x["z"]), delta_bias=np64(x["bias"]), h_init=np64(x["h0"]),
                         delta_softplus=True)
    g = oracle.scan_bwd(np64(x["u"]), np64(x["delta"]), np64(x["A"]), np64(x["B"]), np64(x["C"]),
                        np64(x["dout"]), D=np64(x["D"]), z=np64(x["z"]), delta_bias=np64(x["bias"]),
                        h_init=np64(x["h0"]), delta_softplus=True, dh_last=np64(x["dh"]), fwd=fw)
    return fw, g


def _run_slice(x, lo, hi, segments, group, last):
    keys = ["u", "delta", "A", "B", "C", "D", "z", "bias", "h0"]
    leaves = {}
    for k in keys:
        t = x[k]
        if t is None:
            leaves[k] = None
            continue
        if k in ("u", "delta", "B", "C", "z"):
            t = t[..., lo:hi].contiguous()
        leaves[k] = t.clone().requires_grad_()
    out, hf = sliced_scan(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                          leaves["z"], leaves["bias"], leaves["h0"], True, segments=segments, group=group,
                          kernels=FakeKernels())
    loss = (out * x["dout"][..., lo:hi]).sum()
    if last:
        loss = loss + (hf * x["dh"]).sum()
    loss.backward()
    return out.detach(), hf.detach(), {k: (v.grad if v is not None else None) for k, v in leaves.items()}


def _check(x, fw, g, lo, hi, out, hf, grads, rank0):
    np.testing.assert_allclose(out.numpy(), fw["out"][..., lo:hi], **TOL)
    np.testing.assert_allclose(hf.numpy(), fw["h_last"], **TOL)
    for k, ok in [("u", "du"), ("delta", "ddelta"), ("z", "dz"), ("B", "dB"), ("C", "dC")]:
        np.testing.assert_allclose(grads[k].numpy(), g[ok][..., lo:hi], **TOL, err_msg=k)
    for k, ok in [("A", "dA"), ("D", "dD"), ("bias", "ddelta_bias")]:
        np.testing.assert_allclose(grads[k].numpy(), g[ok], **TOL, err_msg=k)
    if x["h0"] is not None:
        want = g["dh_init"] if rank0 else np.zeros_like(g["dh_init"])
        np.testing.assert_allclose(grads["h0"].numpy(), want, **TOL, err_msg="h0")


def test_plan_segments():
    assert plan_segments(1, 5120, 131072, 16) == 32     # long-sequence config: 32 segments
    assert plan_segments(1, 5120, 16384, 16) == 32      # a 16384-token sequence on one GPU: 512-token segments
    assert plan_segments(1, 5120, 16384, 16, ranks=8) == 16   # the slice of config 5 on each of 8 GPUs
    assert plan_segments(1, 5120, 65536, 16, ranks=2) == 32   # ... on each of 2 GPUs
    assert plan_segments(8, 1536, 2048, 16) == 1        # batch > 1: never
    assert plan_segments(1, 64, 300, 16) == 1           # not a multiple of 256 tokens
    assert plan_segments(1, 64, 2048, 16) == 4          # segments stay >= 512 tokens


def test_segment_view_is_a_view():
    t = torch.arange(2 * 3 * 8, dtype=torch.float32).reshape(1, 6, 8)
    v = segment_view(t, 4)
    assert v.shape == (4, 6, 2) and v.data_ptr() == t.data_ptr()
    assert torch.equal(v[1, 2], t[0, 2, 2:4])
    # a channel-strided input (the first half of an in_proj output) keeps its channel stride
    big = torch.arange(2 * 6 * 8, dtype=torch.float32).reshape(1, 12, 8)
    half = big[:, :6]
    vh = segment_view(half, 2)
    assert vh.stride() == (4, 8, 1) and torch.equal(vh[1, 5], half[0, 5, 4:8])
    with pytest.raises(ValueError):
        segment_view(big.transpose(1, 2), 2)


@pytest.mark.parametrize("segments", [1, 2, 4])
def test_segments_on_one_process_match_the_whole_sequence(segments):
    x = _inputs()
    fw, g = _oracle(x)
    L = x["u"].shape[-1]
    out, hf, grads = _run_slice(x, 0, L, segments, None, last=True)
    _check(x, fw, g, 0, L, out, hf, grads, rank0=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, segments, q):
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        x = _inputs()
        fw, g = _oracle(x)
        L = x["u"].shape[-1]
        lo, hi = rank * L // world, (rank + 1) * L // world
        out, hf, grads = _run_slice(x, lo, hi, segments, SliceGroup(dist.group.WORLD), last=rank == world - 1)
        _check(x, fw, g, lo, hi, out, hf, grads, rank0=rank == 0)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,segments", [(2, 1), (2, 2), (4, 2)])
def test_ranks_over_gloo_match_the_whole_sequence(world, segments):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, segments, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=240)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res == {r: "ok" for r in range(world)}, res


# ---- failures of a peer rank (host-side; no GPU involved) ---------------------------------
def _faulty_rank_main(rank, world, port, mode, q):
    import datetime
    import torch.distributed as dist
    try:
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        if mode == "dies" and rank == 1:
            os._exit(3)                      # a rank that is gone before the exchange
        x = _inputs()
        L = x["u"].shape[-1]
        lo, hi = rank * L // world, (rank + 1) * L // world
        segments = 2 if (mode in ("shape", "shape_store") and rank == 1) else 1
        group = SliceGroup(dist.group.WORLD)
        if mode == "shape_store":            # the agreement through the store, with the liveness check
            group = SliceGroup(dist.group.WORLD, store=dist.PrefixStore("t", store),
                               peer_timeout=datetime.timedelta(seconds=10))
        _run_slice(x, lo, hi, segments, group, last=rank == world - 1)
        q.put((rank, "ok"))
    except Exception as e:  # the clean error this test expects
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("mode", ["shape", "shape_store", "dies"])
def test_peer_failure_gives_a_clean_error(mode):
    """A rank that passes other shapes makes every rank raise the agreement error (by the
    all_gather of check_agreement, or with a store through check_peers); a rank that dies
    before the exchange makes the survivor's collective raise (connection lost or the
    process group's timeout) instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_faulty_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world if mode != "dies" else 1):
            r, msg = q.get(timeout=120)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    if mode != "dies":
        assert set(res) == {0, 1}
        for r in (0, 1):
            assert "ranks disagree" in res[r], res
    else:
        assert procs[1].exitcode == 3
        assert 0 in res and res[0] != "ok", res


def _leaving_rank_main(rank, world, port, q):
    """Two sliced-scan steps with the host-side liveness check; rank 1 leaves after the
    first step (between steps, nothing in flight)."""
    import datetime
    import torch.distributed as dist
    try:
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        group = SliceGroup(dist.group.WORLD, store=store, peer_timeout=datetime.timedelta(seconds=3))
        x = _inputs()
        L = x["u"].shape[-1]
        lo, hi = rank * L // world, (rank + 1) * L // world
        _run_slice(x, lo, hi, 2, group, last=rank == world - 1)
        if rank == 1:
            msg = "left"          # leaves between steps: exits without a word to its peers
        else:
            _run_slice(x, lo, hi, 2, group, last=rank == world - 1)
            msg = "ok"
    except Exception as e:  # the clean error this test expects
        msg = f"{type(e).__name__}: {e}"
    q.put((rank, msg))
    q.close()
    q.join_thread()           # flush the message before the abrupt exit
    os._exit(0)


def test_peer_leaving_between_steps_is_detected_on_the_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, msg = q.get(timeout=120)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[1] == "left", res
    assert res[0].startswith("RuntimeError: sliced scan: rank(s) [1] did not reach exchange 2"), res
