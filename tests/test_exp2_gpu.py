"""The exp2 that the carry passes compute on the FMA pipe for a share of their elements
(exp2_fma2 in ssm_mamba_b200/csrc/common.cuh: rounding split, degree-5 polynomial fitted for
minimax relative error, exponent insertion), evaluated through ssm_exp2_compare next to the
MUFU ex2.approx.ftz the other elements use, against float64 exp2:
  * over the decays' range [-126, 0] (a dense grid plus every multiple of 1/4): relative
    error <= 2^-22, the bound PTX documents for ex2.approx.f32 (the fit: 2^-22.6);
  * the FMA-pipe result is never further from float64 than the MUFU result by more than
    2^-22 relative;
  * exact at x = 0 (identity steps of padded tokens) and at every integer x >= -126;
  * below -126 the result is non-negative and under 2^-125 (ex2.approx.ftz returns 0)."""
import numpy as np
import pytest
import torch

from ssm_mamba_b200 import capi

pytestmark = pytest.mark.gpu


def _eval(x):
    y_fma, y_mufu = torch.empty_like(x), torch.empty_like(x)
    rc = capi.lib().ssm_exp2_compare(capi._t(x), capi._t(y_fma), capi._t(y_mufu), x.numel(), capi._stream())
    assert rc == capi.SSM_OK, capi.lib().ssm_last_error()
    torch.cuda.synchronize()
    return y_fma.cpu().double().numpy(), y_mufu.cpu().double().numpy()


def test_fma_pipe_exp2_error_bound(cuda):
    grid = torch.linspace(-126.0, 0.0, 4_000_001, dtype=torch.float64)
    quarters = torch.arange(-126 * 4, 1, dtype=torch.float64) / 4
    x = torch.cat([grid, quarters]).float().to(cuda)
    fma, mufu = _eval(x)
    ref = np.exp2(x.cpu().double().numpy())
    rel_fma = np.abs(fma - ref) / ref
    rel_mufu = np.abs(mufu - ref) / ref
    bound = 2.0 ** -22
    assert rel_fma.max() <= bound, f"max relative error {rel_fma.max():.3e} > 2^-22"
    assert (rel_fma - rel_mufu).max() <= bound
    xs = x.cpu().numpy()
    ints = xs == np.round(xs)
    assert np.array_equal(fma[ints], ref[ints]), "2^j not exact at integers"
    assert fma[xs == 0].min() == 1.0 and fma[xs == 0].max() == 1.0


def test_fma_pipe_exp2_below_range(cuda):
    x = torch.linspace(-400.0, -126.001, 100_001, device=cuda)
    fma, mufu = _eval(x)
    assert (fma >= 0).all() and (fma < 2.0 ** -125).all()
    assert (mufu <= 2.0 ** -125).all()
