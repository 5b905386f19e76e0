"""Selective scan of long sequences as independent slices.

A sequence can be cut into slices that are scanned at the same time, because the
recurrence h_t = exp(delta_t A) h_{t-1} + delta_t u_t B_t is linear in the state: a slice
q started from the state h_in(q) ends in P_q h_in(q) + h0_end(q), where h0_end(q) is its end
state from a zero start and P_q = exp(A * sum(delta over the slice)).  Two uses:

* segments on one GPU -- a batch-1 sequence with few channels (the long-sequence config:
  batch 1, d_inner 5120) gives the scan kernels one CTA per 32 channels, too few to fill
  148 SMs; viewed as S segments of length L/S (a (S, dim, L/S) view with batch stride
  L/S, no copy) it gives S times more CTAs;
* sequence parallelism -- the ranks of a process group each hold a contiguous slice of the
  sequence (and may segment it further); the per-slice carries cross GPUs with one NCCL
  all_gather per direction.

Forward: chunk_state_fwd (end states and delta sums of every local slice) -> all_gather ->
carry_compose (the state entering every slice, and the final state) -> the ordinary forward
of every slice with that h_init.  Backward: chunk_state_bwd (every slice's gradient into
the state before it) -> all_gather -> carry_compose in reverse (the gradient leaving every
slice) -> the ordinary backward of every slice with that dh_last -> all_reduce of the
parameter gradients dA, dD, ddelta_bias across ranks.

No reference counterpart: the reference scans every sequence serially in 128-token
chunks inside one CTA (csrc/selective_scan/forward_kernel.cu:208-228,
backward_kernel.cu:341-366); the math of each slice is unchanged.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from ._ext import _C

# The scan kernels run 3 CTAs of 128 threads per SM; segmenting stops once the rows give
# this many full waves of them.  Measured on B200, long-sequence config (batch 1, d_inner
# 5120, seqlen 131072, bf16, fwd+bwd): 1 segment 54.0 ms, 2: 43.3, 4: 39.1, 8: 33.7,
# 16: 32.4 (an earlier build); with the current kernels 8: 30.8, 16: 29.6, 32: 28.7,
# 64: 28.7 -- the gain continues to ~8 waves.  Segments of 512 tokens still pay: a 16384-token
# slice (config 5 on each of 8 GPUs) takes 3.84 ms as 16 segments and 3.77 ms as 32.
_CTAS_PER_SM = 3
_TARGET_WAVES = 8


def plan_segments(batch: int, dim: int, seqlen: int, dstate: int, sms: int = 148,
                  min_segment: Optional[int] = None, ranks: int = 1) -> int:
    """Number of segments (a power of two) to split a sequence (or, with ranks > 1, this
    rank's slice of it) into on one GPU: 1 unless batch == 1 and batch * dim rows leave the
    SMs short of warps.  Every segment is a multiple of 128 tokens and at least
    `min_segment` long: 512 on one GPU; 1024 across ranks, where every segment's carry
    crosses the GPUs in the all_gather (measured: config 5 on 4 B200s, 7.90 ms at 16
    segments per rank, 8.01 ms at 32).  SSM_SEGMENTS overrides."""
    if min_segment is None:
        min_segment = 512 if ranks <= 1 else 1024
    env = os.environ.get("SSM_SEGMENTS")
    if env:
        s = int(env)
        return s if s >= 1 and seqlen % (s * 128) == 0 else 1
    if batch != 1:
        return 1
    ns = 4
    while ns < dstate:
        ns *= 2
    lanes = max(ns // 4, 1)  # lanes per channel at 4 states per thread
    rows_needed = sms * _CTAS_PER_SM * (128 // lanes) * _TARGET_WAVES
    s = 1
    while s * dim < rows_needed and seqlen % (2 * s * 128) == 0 and seqlen // (2 * s) >= min_segment:
        s *= 2
    return s


def segment_view(t: Optional[torch.Tensor], s: int) -> Optional[torch.Tensor]:
    """(1, X, L) with unit token stride -> (s, X, L // s) view with batch stride L // s and
    the channel stride of t; s == 1: t."""
    if t is None or s == 1:
        return t
    _, x, L = t.shape
    if t.stride(2) != 1:
        raise ValueError("segment_view needs a unit token stride")
    return t.as_strided((s, x, L // s), (L // s, t.stride(1), 1), t.storage_offset())


class PhaseTimer:
    """Optional CUDA-event markers between the phases of SlicedScanFn (chunk states, carry
    exchange, compose, the per-slice scans, the parameter-gradient all_reduce), for a
    per-phase breakdown of a step.  Install one with set_phase_timer(); with none installed
    (the default) the orchestration records nothing."""

    def __init__(self):
        self.marks = []

    def mark(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append((name, ev))

    def durations_ms(self):
        """{phase: ms} from consecutive marks (call after a synchronize); the duration of a
        mark is the time from it to the next one."""
        out = {}
        for (name, ev), (_, nxt) in zip(self.marks, self.marks[1:]):
            if name.startswith("end"):
                continue
            out[name] = out.get(name, 0.0) + ev.elapsed_time(nxt)
        return out


_PHASES: Optional[PhaseTimer] = None


def set_phase_timer(timer: Optional[PhaseTimer]) -> None:
    global _PHASES
    _PHASES = timer


def _mark(name: str) -> None:
    if _PHASES is not None:
        _PHASES.mark(name)


class SliceGroup:
    """The ranks that share one sequence (rank r holds the r-th contiguous slice), or a
    single process (world 1, no communication).

    With a `store` (any torch.distributed Store the ranks share) and a `peer_timeout`
    (datetime.timedelta), every exchange starts with a host-side liveness check
    (check_peers): a rank that has left makes the others raise RuntimeError before any
    collective or kernel of that exchange is launched, instead of leaving a collective on
    the GPU waiting for the process group's timeout."""

    def __init__(self, group=None, store=None, peer_timeout=None):
        import torch.distributed as dist
        self.group = group
        if group is None:
            self.world, self.rank = 1, 0
        else:
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        self.store = store
        self.peer_timeout = peer_timeout
        self._exchanges = 0

    def check_peers(self, what: str, agree=None) -> None:
        """Host-side liveness check before an exchange (no-op without a store): this rank
        posts that it reached exchange n and waits, at most peer_timeout, until every rank
        has.  Every rank runs the same exchanges in the same order, so n agrees across ranks.
        Each rank then deletes its key of exchange n - 2, which every rank has passed.
        With `agree` = (description, ints), the posted value carries the ints and every rank
        compares all ranks' values, raising the same RuntimeError on a mismatch: the shape
        agreement of check_agreement without a collective or a device synchronization."""
        if self.world == 1 or self.store is None:
            return
        n = self._exchanges
        self._exchanges += 1
        key = lambda i, r: f"ssm_slices/{i}/{r}"  # noqa: E731
        values = "" if agree is None else ",".join(str(int(v)) for v in agree[1])
        self.store.set(key(n, self.rank), f"{what}|{values}")
        keys = [key(n, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.peer_timeout)
        except Exception as e:
            missing = [r for r in range(self.world) if not self.store.check([key(n, r)])]
            raise RuntimeError(f"sliced scan: rank(s) {missing} did not reach exchange {n} ({what}) "
                               f"within {self.peer_timeout}") from e
        if agree is not None:
            rows = [v.decode().split("|", 1)[1] for v in self.store.multi_get(keys)]
            if any(r != rows[0] for r in rows):
                raise RuntimeError(f"sliced scan: ranks disagree on {agree[0]}: "
                                   f"{[[int(x) for x in r.split(',')] for r in rows]}")
        if n >= 2:
            self.store.delete_key(key(n - 2, self.rank))

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """(world, *t.shape): every rank's t, in rank order."""
        if self.world == 1:
            return t.unsqueeze(0)
        import torch.distributed as dist
        t = t.contiguous()
        out = t.new_empty((self.world,) + tuple(t.shape))
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, t, group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), t, group=self.group)
        return out

    def check_agreement(self, what: str, values, device) -> None:
        """Every rank must pass the same `values` (a fixed-length list of ints).  One small
        all_gather; when the ranks disagree, every rank raises the same RuntimeError instead
        of exchanging carries of mismatched shapes."""
        if self.world == 1:
            return
        rows = self.all_gather(torch.tensor(list(values), dtype=torch.int64, device=device)).cpu()
        if not bool((rows == rows[0]).all()):
            raise RuntimeError(f"sliced scan: ranks disagree on {what}: {rows.tolist()}")

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)
        return t


class _Kernels:
    """The native entry points the slice orchestration calls (the torch binding of the C
    ABI: ssm_scan_chunk_state_fwd / _bwd, ssm_scan_carry_compose, ssm_scan_fwd,
    ssm_scan_bwd)."""

    chunk_state_fwd = staticmethod(_C.chunk_state_fwd)
    chunk_state_bwd = staticmethod(_C.chunk_state_bwd)
    carry_compose = staticmethod(_C.carry_compose)
    scan_fwd_out = staticmethod(_C.scan_fwd_out)
    scan_bwd_out = staticmethod(_C.scan_bwd_out)
    ckpt_len = staticmethod(_C.ckpt_len)


KERNELS = _Kernels()


class SlicedScanFn(torch.autograd.Function):
    """Selective scan of this rank's slice of a sequence, cut into `segments` local
    segments (batch must be 1 when segments > 1).  Returns (out, h_final) where h_final is
    the state after the LAST token of the whole sequence (the same on every rank).

    Gradients are those of the sum of every rank's objective: dA, dD and ddelta_bias are
    summed over ranks (every rank gets the total), dh_final is summed over ranks, and the
    gradient of h_init (the state before the first token of rank 0's slice) is returned on
    rank 0 and zero on the other ranks."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, h_init, delta_softplus, segments, group, kernels):
        k = kernels
        S = int(segments)
        Bt, Dm, L = u.shape
        N = A.shape[1]
        if S > 1 and (Bt != 1 or L % S != 0):
            raise ValueError("segmented scan needs batch 1 and seqlen divisible by the segment count")
        _mark("fwd_agree")
        # a peer with other shapes or options would exchange carries of another size: refuse
        # (through the store with the liveness check when there is one, else one all_gather)
        agree = ("batch, dim, dstate, segments, z, D, delta_bias, h_init, softplus, dtype",
                 [Bt, Dm, N, S, z is not None, D is not None, delta_bias is not None,
                  h_init is not None, bool(delta_softplus), u.element_size()])
        if group.store is not None:
            group.check_peers("forward", agree)
        else:
            group.check_agreement(*agree, u.device)
        Bc = Bt if S == 1 else 1            # batch of one slice
        rows = Bt if S == 1 else S          # rows of the segmented views
        sv = lambda t: segment_view(t, S)  # noqa: E731
        u_s, d_s, B_s, C_s, z_s = sv(u), sv(delta), sv(B), sv(C), sv(z)

        # 1. every local slice from a zero start: end state and delta sum
        _mark("fwd_chunk_state")
        h0, dsum = k.chunk_state_fwd(u_s, d_s, A, B_s, delta_bias, bool(delta_softplus))
        per = Bc * Dm * N
        carry_loc = h0.reshape(S, Bc, Dm, N)
        dsum_loc = dsum.reshape(S, Bc, Dm)
        start = h_init.reshape(1, Bc, Dm, N) if h_init is not None else None
        r = group.rank
        if group.world == 1:
            # 2. the state entering every slice, in order
            _mark("fwd_compose")
            carries = k.carry_compose(A, carry_loc, dsum_loc, start, False)        # (S + 1, Bc, Dm, N)
            h_final = carries[S].reshape(Bc, Dm, N)
            dsum_rank = dsum_loc.sum(0, keepdim=True)
        else:
            # 2. in two levels, so that one carry per rank crosses the interconnect: this
            # rank's slices folded into its end state from a zero start and its delta sum,
            # those of all ranks exchanged and folded in rank order (the state entering
            # every rank), then this rank's slices folded again from its entering state
            _mark("fwd_compose")
            local = k.carry_compose(A, carry_loc, dsum_loc, None, False)           # (S + 1, Bc, Dm, N)
            pack = torch.cat([local[S].reshape(per), dsum_loc.sum(0).reshape(Bc * Dm)])
            _mark("fwd_exchange")
            allp = group.all_gather(pack)                                            # (world, per + Bc*Dm)
            _mark("fwd_compose")
            dsum_rank = allp[:, per:].reshape(group.world, Bc, Dm)
            ranks = k.carry_compose(A, allp[:, :per].reshape(group.world, Bc, Dm, N), dsum_rank, start, False)
            h_final = ranks[group.world].reshape(Bc, Dm, N)
            carries = k.carry_compose(A, carry_loc, dsum_loc, ranks[r:r + 1], False)
        h_in = carries[:S].reshape(rows, Dm, N)
        # 3. the ordinary forward of every slice from its own initial state
        need_grad = any(ctx.needs_input_grad[:9])
        _mark("fwd_scan")
        out = torch.empty_like(u)
        y = torch.empty_like(u) if (need_grad and z is not None) else None
        _, _, ckpt, _ = k.scan_fwd_out(u_s, d_s, A, B_s, C_s, D, z_s, delta_bias, h_in, None, True,
                                       bool(delta_softplus), sv(out), sv(y), 1 if need_grad else 0, False)
        if need_grad:
            ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, y, ckpt, h_in, dsum_loc, dsum_rank, h_init)
            ctx.cfg = (bool(delta_softplus), S, group, k, Bc, rows)
        _mark("end_fwd")
        return out, h_final

    @staticmethod
    def backward(ctx, dout, dh_final):
        u, delta, A, B, C, D, z, delta_bias, y, ckpt, h_in, dsum_loc, dsum_rank, h_init = ctx.saved_tensors
        softplus, S, group, k, Bc, rows = ctx.cfg
        Bt, Dm, L = u.shape
        N = A.shape[1]
        sv = lambda t: segment_view(t, S)  # noqa: E731
        dout = dout.contiguous()
        u_s, d_s, B_s, C_s, z_s, dout_s = sv(u), sv(delta), sv(B), sv(C), sv(z), sv(dout)
        _mark("bwd_agree")
        group.check_peers("backward")
        # 1. every local slice's gradient into the state before it, from a zero start
        _mark("bwd_chunk_state")
        g0 = k.chunk_state_bwd(d_s, A, C_s, z_s, delta_bias, softplus, dout_s)     # (rows, Dm, N)
        per = Bc * Dm * N
        if dh_final is None:
            dh_final = torch.zeros(Bc, Dm, N, device=u.device, dtype=g0.dtype)
        g_loc = g0.reshape(S, Bc, Dm, N)
        r = group.rank
        if group.world == 1:
            # 2. the gradient leaving every slice's end
            _mark("bwd_compose")
            dh_last = k.carry_compose(A, g_loc, dsum_loc, dh_final.reshape(1, Bc, Dm, N).to(g0.dtype), True)
        else:
            # 2. in two levels (as the forward): this rank's slices folded, from a zero
            # gradient at its end, into the gradient entering its start (a reverse fold over
            # S + 1 entries whose entry 0 is never read); those of all ranks exchanged with
            # the ranks' final-state gradients and folded in reverse rank order (the gradient
            # leaving every rank's end); then this rank's slices folded again from it
            _mark("bwd_compose")
            ext = torch.cat([g_loc[:1], g_loc])
            dext = torch.cat([dsum_loc[:1], dsum_loc])
            local = k.carry_compose(A, ext, dext, None, True)                       # (S + 1, Bc, Dm, N)
            pack = torch.cat([local[0].reshape(per), dh_final.reshape(per).to(g0.dtype)])
            _mark("bwd_exchange")
            allp = group.all_gather(pack)                                            # (world, 2 per)
            _mark("bwd_compose")
            ranks = k.carry_compose(A, allp[:, :per].reshape(group.world, Bc, Dm, N), dsum_rank,
                                    allp[:, per:].reshape(group.world, Bc, Dm, N), True)
            dh_last = k.carry_compose(A, g_loc, dsum_loc, ranks[r:r + 1], True)      # (S, Bc, Dm, N)
        dh_last = dh_last.reshape(rows, Dm, N)
        # 3. the ordinary backward of every slice
        _mark("bwd_scan")
        du, ddelta = torch.empty_like(u), torch.empty_like(u)
        dB, dC = torch.empty_like(B), torch.empty_like(C)
        dz = torch.empty_like(u) if z is not None else None
        res = k.scan_bwd_out(u_s, d_s, A, B_s, C_s, D, z_s, delta_bias, h_in, None, True, softplus, sv(y),
                             ckpt, dout_s, dh_last, sv(du), sv(ddelta), sv(dB), sv(dC), sv(dz))
        dA, dD, ddb, dh_rows = res[2], res[5], res[6], res[8]
        # 4. parameter gradients are sums over the whole sequence
        _mark("bwd_param_allreduce")
        if group.world > 1:
            parts = [dA.reshape(-1)] + [t for t in (dD, ddb) if t is not None and t.numel()]
            flat = group.all_reduce_(torch.cat(parts))
            dA = flat[:dA.numel()].view_as(dA)
            o = dA.numel()
            if dD is not None and dD.numel():
                dD = flat[o:o + Dm]
                o += Dm
            if ddb is not None and ddb.numel():
                ddb = flat[o:o + Dm]
        dh_init = None
        if h_init is not None:
            dh_init = dh_rows[:Bc].reshape_as(h_init) if r == 0 else torch.zeros_like(h_init)
        _mark("end_bwd")
        return (du, ddelta, dA, dB, dC, dD if D is not None else None, dz,
                ddb if delta_bias is not None else None, dh_init, None, None, None, None)


def sliced_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, h_init=None, delta_softplus=False,
                segments: int = 1, group=None, kernels=None):
    """Selective scan of this rank's contiguous slice of a sequence (the whole sequence
    when `group` is None), cut into `segments` segments; returns (out, h_final).
    Tensors as for selective_scan_fn with B, C of shape (batch, dstate, seqlen)."""
    g = group if isinstance(group, SliceGroup) else SliceGroup(group)
    return SlicedScanFn.apply(u, delta, A, B, C, D, z, delta_bias, h_init, delta_softplus, segments, g,
                              kernels if kernels is not None else KERNELS)


__all__ = ["plan_segments", "segment_view", "SliceGroup", "SlicedScanFn", "sliced_scan", "KERNELS", "PhaseTimer",
           "set_phase_timer"]
