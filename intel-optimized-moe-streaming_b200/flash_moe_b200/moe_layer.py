"""The MoE layer entry points of the B200 backend, with the reference's
signatures (``src/flash_moe/moe_layer.py:39-47`` and ``:110-118``).

On this backend a layer is ONE device call for a batch of tokens: routing
with the layer's resident router, the top-k experts, the weighted sum in
top-k order and the sigmoid-gated shared expert all run inside the kernels
(``B200ExpertBackend.forward_layer``).  The ``router`` and ``shared_expert``
arguments are therefore not called; they are checked against the resident
layer instead: the shapes and ``top_k`` must agree, and the router's gate
must be kept in fp32 (``gate_dtype`` float32), because the resident router
is the fp32 ``ffn_gate_inp`` tensor -- the reference's default gate
rounding to fp16 (``src/flash_moe/router.py:43``) would select experts from
different scores.

For a backend without ``forward_layer`` (one that serves single experts
only), use the reference's own ``run_moe_layer`` / ``run_moe_sequence``: they
drive ``B200ExpertBackend.forward`` one expert at a time unchanged.
"""
from __future__ import annotations

from typing import Any

import numpy as np


def _resident_layer(backend, layer: int, router, hidden_size: int, intermediate_size: int):
    """The resident layer's weights after checking the call against them."""
    if not callable(getattr(backend, "forward_layer", None)):
        raise TypeError("this entry point needs a backend with forward_layer (the B200 "
                        "backend); per-expert backends run under the reference's run_moe_layer")
    lw = backend.store.layer(layer).weights
    if (hidden_size, intermediate_size) != (lw.hidden, lw.inter):
        raise ValueError(f"layer {layer} is resident as {lw.hidden}x{lw.inter}, "
                         f"called with {hidden_size}x{intermediate_size}")
    if router is not None:
        wanted = {"top_k": lw.top_k, "num_experts": lw.n_experts, "hidden_size": lw.hidden}
        for attr, value in wanted.items():
            got = getattr(router, attr, value)
            if got != value:
                raise ValueError(f"router {attr} {got} differs from the resident layer's {value}")
        gate_dtype = getattr(router, "gate_dtype", np.dtype(np.float32))
        if np.dtype(gate_dtype) != np.float32:
            raise ValueError(f"router gate kept as {np.dtype(gate_dtype)}: the resident router "
                             "is fp32 (construct ExpertRouter with gate_dtype=np.float32)")
    return lw


def run_moe_layer(layer: int, activation, router, backend: Any, hidden_size: int,
                  intermediate_size: int, shared_expert: Any = None) -> np.ndarray:
    """One token through one MoE layer; returns fp32 [hidden_size]."""
    _resident_layer(backend, layer, router, hidden_size, intermediate_size)
    x = np.asarray(activation, dtype=np.float32).reshape(-1)
    if x.size != hidden_size:
        raise ValueError(f"activation has {x.size} elements, expected {hidden_size}")
    return backend.forward_layer(layer, x)


def run_moe_sequence(layer: int, activations: np.ndarray, router, backend: Any,
                     hidden_size: int, intermediate_size: int,
                     shared_expert: Any = None) -> np.ndarray:
    """Many tokens through one MoE layer; returns fp32 [tokens, hidden_size]."""
    if activations.ndim != 2 or activations.shape[1] != hidden_size:
        raise ValueError(f"MoE activations must have shape (tokens, {hidden_size}), "
                         f"got {activations.shape}")
    _resident_layer(backend, layer, router, hidden_size, intermediate_size)
    return backend.forward_layer(layer, activations)
