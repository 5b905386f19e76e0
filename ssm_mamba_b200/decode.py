"""Token-by-token decoding of a Mamba layer with in-place caches, capturable in a CUDA graph.

The reference decodes one token per Python call (nmquan1503/ssm-mamba,
models/causal_lm.py:118-129 -> modules/mamba.py:188-241, Mamba.step): every step builds
a new conv context with torch.cat and a new SSM state (selective_update.apply returns a
fresh tensor, csrc/selective_update/selective_update.cpp:208-209), so the step cannot be
replayed from a CUDA graph.  Here the two caches are persistent buffers that the step
updates in place (causal_conv1d_update, selective_state_update), every other tensor is an
output of the step, and GraphedStep captures the whole step once and replays it per token.

mamba_layer_step restates Mamba.step with this library's kernels:
    xz = in_proj(h); x, gate = chunk(xz)                              (mamba.py:196-200)
    x = silu(conv step of x over the cached context)                  (:203-213)
    delta, B, C = split(x_proj(x)); delta = dt_proj.weight @ delta     (:215-224)
    y = selective state update (softplus(delta + dt_proj.bias)), y * silu(gate)  (:226-239)
    out = out_proj(y)                                                  (:240)
The projections are plain GEMMs (torch / cuBLAS); the conv step, the state update and the
gate are this library's kernels.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.nn.functional as F

from .ops import causal_conv1d_update, selective_state_update
from .weights import MambaLayerCache, MambaLayerWeights


def mamba_layer_step(w: MambaLayerWeights, cache: MambaLayerCache, hidden: torch.Tensor) -> torch.Tensor:
    """One decoding step of a Mamba layer: hidden (batch, model) -> (batch, model).  Updates
    cache.conv_state and cache.ssm_state in place and allocates only its outputs."""
    xz = F.linear(hidden, w.in_proj_weight, w.in_proj_bias)
    x, gate = xz.chunk(2, dim=-1)
    x = causal_conv1d_update(x, cache.conv_state, w.conv_weight, w.conv_bias)
    params = F.linear(x, w.x_proj_weight)
    delta, Bm, Cm = torch.split(params, [w.rank, w.state, w.state], dim=-1)
    delta = F.linear(delta, w.dt_proj_weight)
    y = selective_state_update(cache.ssm_state, x, delta, w.A, Bm, Cm, w.D, z=gate, dt_bias=w.dt_proj_bias,
                               dt_softplus=True)
    return F.linear(y, w.out_proj_weight, w.out_proj_bias)


class GraphedStep:
    """fn(*inputs) captured once into a CUDA graph.  Calling it copies the new inputs into
    the captured input buffers, replays the graph and returns the captured outputs (the same
    tensors every call: copy them out before the next call if they are kept).  State that fn
    updates in place (the caches) advances with every replay."""

    def __init__(self, fn: Callable, example_inputs: Sequence[torch.Tensor],
                 preserve: Sequence[torch.Tensor] = (), warmup: int = 2):
        """`preserve`: tensors fn updates in place (the caches); they are restored after
        the warm-up and capture runs, so the first replay starts from their current value."""
        self.fn = fn
        self.static_inputs = [t.clone() for t in example_inputs]
        saved = [t.clone() for t in preserve]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_outputs = fn(*self.static_inputs)
        for dst, src in zip(preserve, saved):
            dst.copy_(src)

    def __call__(self, *inputs: torch.Tensor):
        for dst, src in zip(self.static_inputs, inputs):
            if dst.data_ptr() != src.data_ptr():
                dst.copy_(src)
        self.graph.replay()
        return self.static_outputs


__all__ = ["MambaLayerWeights", "MambaLayerCache", "mamba_layer_step", "GraphedStep"]
