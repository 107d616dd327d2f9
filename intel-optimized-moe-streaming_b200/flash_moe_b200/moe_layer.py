"""The MoE layer entry points, with the reference's signatures.

``run_moe_layer`` and ``run_moe_sequence`` take the arguments of their
reference counterparts (``src/flash_moe/moe_layer.py:39-47`` and
``:110-118``).  When the backend offers ``forward_layer`` (the B200 backend
does) the whole layer -- routing with the layer's resident router, the top-k
experts, the weighted sum in top-k order and the sigmoid-gated shared expert
-- runs as one device call per batch of tokens, and the ``router`` and
``shared_expert`` arguments only have to agree with the resident layer.
Otherwise the reference algorithm runs unchanged: route, ``backend.forward``
per selected expert on the backend's executor, ``combined += w * out`` in
top-k order, then ``+ shared_expert.forward``.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Any

import numpy as np

from .key import ExpertKey


def _fused(backend) -> bool:
    return callable(getattr(backend, "forward_layer", None))


def _check_router(backend, layer, router, hidden_size, intermediate_size):
    lw = backend.store.layer(layer).weights
    if hidden_size != lw.hidden or intermediate_size != lw.inter:
        raise ValueError(f"layer {layer} is resident as {lw.hidden}x{lw.inter}, "
                         f"called with {hidden_size}x{intermediate_size}")
    top_k = getattr(router, "top_k", lw.top_k)
    if top_k != lw.top_k:
        raise ValueError(f"router top_k {top_k} differs from the resident layer's {lw.top_k}")


def run_moe_layer(layer: int, activation, router, backend: Any, hidden_size: int,
                  intermediate_size: int, shared_expert: Any = None) -> np.ndarray:
    """One token through one MoE layer; returns fp32 [hidden_size]."""
    if _fused(backend):
        _check_router(backend, layer, router, hidden_size, intermediate_size)
        return backend.forward_layer(layer, np.asarray(activation, dtype=np.float32).reshape(-1))

    expert_ids, weights = router.route(activation)
    keys = [ExpertKey(layer, e) for e in expert_ids]
    prefetch = getattr(backend, "prefetch_weights", None)
    if prefetch is not None:
        prefetch(keys)
    combined = np.zeros(hidden_size, dtype=np.float32)
    executor = getattr(backend, "_moe_executor", None)
    own = executor is None
    if own:
        executor = ThreadPoolExecutor(max_workers=max(1, len(keys)))
    try:
        futures = [executor.submit(backend.forward, k, activation, hidden_size, intermediate_size)
                   for k in keys]
        try:
            for fut, w in zip(futures, weights):
                combined += w * np.asarray(fut.result(), dtype=np.float32)
        finally:
            for fut in futures:
                try:
                    fut.result()
                except Exception:
                    pass
    finally:
        if own:
            executor.shutdown(wait=True)
    if shared_expert is not None:
        shared_out = shared_expert.forward(layer, activation)
        if shared_out is not None:
            combined = combined + shared_out
    return combined


def run_moe_sequence(layer: int, activations: np.ndarray, router, backend: Any,
                     hidden_size: int, intermediate_size: int,
                     shared_expert: Any = None) -> np.ndarray:
    """Many tokens through one MoE layer; returns fp32 [tokens, hidden_size]."""
    if activations.ndim != 2 or activations.shape[1] != hidden_size:
        raise ValueError(f"MoE activations must have shape (tokens, {hidden_size}), "
                         f"got {activations.shape}")
    if _fused(backend):
        _check_router(backend, layer, router, hidden_size, intermediate_size)
        return backend.forward_layer(layer, activations)
    return np.stack([run_moe_layer(layer, a, router, backend, hidden_size, intermediate_size,
                                   shared_expert) for a in activations])
