"""GPU parity of the decode kernel (ssm_state_update) against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, np64
from ssm_mamba_b200 import capi
from ssm_mamba_b200.workloads import decode_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,D,N,dtype,gate", [
    (4, 64, 16, torch.float32, False),
    (4, 64, 16, torch.bfloat16, True),
    (3, 50, 17, torch.float32, True),
    (2, 16, 1, torch.float32, False),
    (2, 8, 256, torch.float32, True),
    (64, 5120, 16, torch.bfloat16, True),   # config 3 width
])
def test_state_update_capi(cuda, B, D, N, dtype, gate):
    dec = decode_inputs(B, D, N, 3, dtype, seed=B + N, device=cuda)
    state = dec.state.clone()
    z = dec.z[0] if gate else None
    ref_out, ref_state = oracle.state_update(np64(dec.state), np64(dec.x[0]), np64(dec.dt[0]), np64(dec.A),
                                             np64(dec.B[0]), np64(dec.C[0]), np64(dec.D), np64(z),
                                             np64(dec.dt_bias), True)
    out = torch.empty(B, D, dtype=dtype, device=cuda)
    a = capi.fill_update(state, state, dec.x[0], dec.dt[0], dec.A, dec.B[0], dec.C[0], out, D=dec.D, z=z,
                         dt_bias=dec.dt_bias, dt_softplus=True)
    capi.call_update(a)
    torch.cuda.synchronize()
    tol = (1e-4, 1e-5) if dtype == torch.float32 else (1e-2, 5e-2)
    assert_close(out, ref_out, *tol, name="out")
    assert_close(state, ref_state, 1e-4, 1e-5, name="state (in place)")


def test_selective_state_update_in_place_sequence(cuda):
    """1024-step style loop: in-place updates accumulate exactly like the oracle's steps."""
    from ssm_mamba_b200 import selective_state_update
    dec = decode_inputs(4, 128, 16, 16, torch.bfloat16, seed=3, device=cuda)
    state = dec.state.clone()
    ref_state = np64(dec.state)
    for s in range(16):
        out = selective_state_update(state, dec.x[s], dec.dt[s], dec.A, dec.B[s].unsqueeze(1), dec.C[s].unsqueeze(1),
                                     dec.D, dec.z[s], dec.dt_bias, dt_softplus=True)
        ref_out, ref_state = oracle.state_update(ref_state, np64(dec.x[s]), np64(dec.dt[s]), np64(dec.A),
                                                 np64(dec.B[s]), np64(dec.C[s]), np64(dec.D), np64(dec.z[s]),
                                                 np64(dec.dt_bias), True)
        assert_close(out, ref_out, 1e-2, 5e-2, name=f"out step {s}")
    assert_close(state, ref_state, 1e-4, 1e-5, name="state after 16 steps")


def test_reference_update_api_is_out_of_place(cuda):
    from ssm_mamba_b200 import SelectiveUpdateFn
    dec = decode_inputs(2, 32, 16, 1, torch.float32, seed=1, device=cuda)
    h = dec.state.clone()
    out, new_h = SelectiveUpdateFn.apply(dec.x[0], dec.A, dec.B[0], dec.C[0], dec.D, dec.dt[0], dec.dt_bias, h)
    assert torch.equal(h, dec.state)
    assert new_h.data_ptr() != h.data_ptr()
    ref_out, ref_state = oracle.state_update(np64(dec.state), np64(dec.x[0]), np64(dec.dt[0]), np64(dec.A),
                                             np64(dec.B[0]), np64(dec.C[0]), np64(dec.D), None, np64(dec.dt_bias), True)
    assert_close(out, ref_out, 1e-4, 1e-5, name="out")
    assert_close(new_h, ref_state, 1e-4, 1e-5, name="new_h")


@pytest.mark.parametrize("B,D,N,dtype,gate", [
    (5, 256, 16, torch.bfloat16, True),     # streamed: tiles of 128 channels
    (3, 512, 8, torch.float32, False),      # streamed: tiles of 256 channels
    (2, 128, 32, torch.float32, True),      # streamed: tiles of 64 channels
    (4, 200, 16, torch.bfloat16, True),     # dim not a multiple of the tile: the per-CTA kernel
])
def test_streamed_and_per_cta_decode_kernels_agree(cuda, monkeypatch, B, D, N, dtype, gate):
    """The streamed decode kernel (bulk-copy pipeline, picked for contiguous 16-byte aligned
    layouts) and the per-CTA kernel (SSM_DEC_STREAM=0) give the oracle's step, out of place
    and in place, over 4 consecutive steps."""
    dec = decode_inputs(B, D, N, 4, dtype, seed=D + N, device=cuda)
    results = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("SSM_DEC_STREAM", mode)
        state = dec.state.clone()
        outs = []
        for s in range(4):
            out = torch.empty(B, D, dtype=dtype, device=cuda)
            # even steps in place, odd steps into a fresh state buffer
            nxt = state if s % 2 == 0 else torch.empty_like(state)
            a = capi.fill_update(state, nxt, dec.x[s], dec.dt[s], dec.A, dec.B[s], dec.C[s], out, D=dec.D,
                                 z=dec.z[s] if gate else None, dt_bias=dec.dt_bias, dt_softplus=True)
            capi.call_update(a)
            outs.append(out)
            state = nxt
        torch.cuda.synchronize()
        results[mode] = (torch.stack(outs), state)
    ref_state = np64(dec.state)
    for s in range(4):
        ref_out, ref_state = oracle.state_update(ref_state, np64(dec.x[s]), np64(dec.dt[s]), np64(dec.A),
                                                 np64(dec.B[s]), np64(dec.C[s]), np64(dec.D),
                                                 np64(dec.z[s]) if gate else None, np64(dec.dt_bias), True)
        tol = (1e-4, 1e-5) if dtype == torch.float32 else (1e-2, 5e-2)
        for mode in ("1", "0"):
            assert_close(results[mode][0][s], ref_out, *tol, name=f"mode {mode} step {s} out")
    for mode in ("1", "0"):
        assert_close(results[mode][1], ref_state, 1e-4, 1e-5, name=f"mode {mode} state")
    assert_close(results["1"][1], results["0"][1], 0, 0, name="streamed vs per-CTA state")
