"""The reference's own Python (its Mamba module and CausalLM, unchanged, staged by
oracle/build_ref.py into oracle/_ref/ssm_mamba_ref/) run twice on the same weights and
inputs: once on the reference's own kernels (oracle/_ref/ref_selective_*), once with this
library's drop-in extension modules (ssm_mamba_b200/compat/) standing in for the
`selective_scan` / `selective_update` modules its ops import
(ops/selective_scan_interface.py:2, ops/selective_update_interface.py:2).  This is the
drop-in as a user of the reference would make it.

Checked, in float32 (the reference kernels' only dtype), eval mode (no dropout):
  * Mamba.forward with `lengths` (left padding, the reference default, as
    modules/mamba.py:170-175 calls SelectiveScanFn) and without, and its backward (input
    and every parameter gradient);
  * a 2-layer CausalLM: prefill with use_cache, 16 decoding steps (Mamba.step ->
    SelectiveUpdateFn, modules/mamba.py:231-238) fed the same tokens, logits compared at
    every step, and CausalLM.generate (models/causal_lm.py:98-134) token for token.
Tolerances: outputs and logits rtol 1e-4 / atol 1e-5 (times the largest magnitude for the
logits, which pass through two layers, a norm and the vocabulary projection); gradients
those of tests/helpers.py."""
import importlib
import os
import sys

import pytest
import torch

from helpers import assert_close, assert_grad_close

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _backends():
    import build_ref
    if not (build_ref.available() and build_ref.package_available()):
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    from ssm_mamba_b200.compat import selective_scan as ours_ss, selective_update as ours_su
    return {"reference": (build_ref.load("ref_selective_scan"), build_ref.load("ref_selective_update")),
            "ours": (ours_ss, ours_su)}


def _load_reference_package(scan_mod, update_mod):
    """A fresh import of the staged reference package whose `import selective_scan` /
    `import selective_update` resolve to the given modules."""
    import build_ref
    pkg = build_ref.PKG
    for name in list(sys.modules):
        if name == pkg or name.startswith(pkg + ".") or name in ("selective_scan", "selective_update"):
            del sys.modules[name]
    sys.modules["selective_scan"] = scan_mod
    sys.modules["selective_update"] = update_mod
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        return importlib.import_module(pkg)
    finally:
        del sys.modules["selective_scan"], sys.modules["selective_update"]


@pytest.fixture(scope="module")
def packages(cuda):
    return {k: _load_reference_package(*v) for k, v in _backends().items()}


def _mamba_pair(packages, cuda, **kw):
    mods = {}
    for k, pkg in packages.items():
        torch.manual_seed(0)
        mods[k] = pkg.modules.Mamba(**kw).to(cuda).eval()
    mods["ours"].load_state_dict(mods["reference"].state_dict())
    return mods


@pytest.mark.parametrize("lengths", [None, [200, 150, 77]])
def test_mamba_module_forward_backward(packages, cuda, lengths):
    mods = _mamba_pair(packages, cuda, model_dim=64, state_dim=16)
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(3, 200, 64, device=cuda, generator=g)
    dy = torch.randn(3, 200, 64, device=cuda, generator=g)
    dh = torch.randn(3, 128, 16, device=cuda, generator=g)
    ln = torch.tensor(lengths, device=cuda) if lengths else None
    res = {}
    for k, m in mods.items():
        xi = x.clone().requires_grad_()
        out, last = m(xi, lengths=ln)
        ((out * dy).sum() + (last * dh).sum()).backward()
        res[k] = (out.detach(), last.detach(), xi.grad, {n: p.grad for n, p in m.named_parameters()})
    (o_out, o_last, o_dx, o_g), (r_out, r_last, r_dx, r_g) = res["ours"], res["reference"]
    assert_close(o_out, r_out, 1e-4, 1e-5, "Mamba.forward output")
    assert_close(o_last, r_last, 1e-4, 1e-5, "Mamba.forward last state")
    assert_grad_close(o_dx, r_dx, "d hidden_states")
    assert set(o_g) == set(r_g)
    for n in r_g:
        assert_grad_close(o_g[n], r_g[n], "d " + n)


def test_causal_lm_prefill_steps_and_generate(packages, cuda):
    models = {}
    for k, pkg in packages.items():
        torch.manual_seed(0)
        cfg = pkg.CausalLMConfig(vocab_size=512, model_dim=64, num_layers=2, state_dim=16)
        models[k] = pkg.CausalLM(cfg).to(cuda).eval()
    models["ours"].load_state_dict(models["reference"].state_dict())
    g = torch.Generator(device=cuda).manual_seed(2)
    ids = torch.randint(3, 512, (2, 24), device=cuda, generator=g)
    lengths = torch.tensor([24, 24], device=cuda)

    def close(a, b, what):
        scale = float(b.abs().max())
        assert_close(a, b, 1e-4, 1e-5 * max(scale, 1.0), what)

    with torch.no_grad():
        lo = models["ours"](ids, lengths, use_cache=True)
        lr = models["reference"](ids, lengths, use_cache=True)
        close(lo, lr, "prefill logits")
        tok = lr[:, -1].argmax(-1)
        for step in range(16):
            so = models["ours"].step(tok)
            sr = models["reference"].step(tok)
            close(so, sr, f"step {step} logits")
            tok = sr.argmax(-1)
        go = models["ours"].generate(ids, max_new_tokens=16)
        gr = models["reference"].generate(ids, max_new_tokens=16)
    assert torch.equal(go, gr), f"generated tokens differ:\n{go}\n{gr}"
