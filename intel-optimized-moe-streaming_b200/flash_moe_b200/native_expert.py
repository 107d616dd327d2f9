"""The reference's native-kernel Python API over ``libmoe_b200.so``.

The reference binds its CPU DLL with ctypes in ``src/flash_moe/native_expert.py``
(``NativeExpert`` :13-37, ``load_native_expert`` :40-75, ``NativeDelta``
:78-101).  That binding works unchanged against this library, which exports
the same C functions; this module is the package's own form of the same
API, built on ``_lib``:

* ``NativeExpert(path=None, fp16_graph=1).forward(tensors, kinds,
  activation, hidden, intermediate)`` -> fp32 [hidden]: one routed expert
  through ``moe_quant_expert``.  Buffers may be ``bytes``, ``bytearray``,
  ``memoryview`` or uint8 arrays; the reference passes ``fp16_graph=1``.
* ``NativeDelta(library=None).forward(state, q, k, v, beta, gate)``: the
  DeltaNet step ``moe_delta_heads`` on host arrays (state updated in place),
  and ``forward_device`` on CUDA tensors (``moe_b200_delta_heads``).
* ``load_native_expert(mode, library, device, tensor_types)``: the
  ``auto|native|openvino`` selection, with this library's requirement -- a
  CUDA device -- in place of the reference's AVX2/FMA/F16C CPU check.

A nonzero status raises ``RuntimeError("native expert failed with status
N")`` (``"native DeltaNet failed ..."``), the messages the reference's
callers and tests match.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import _lib
from .formats import SUPPORTED_TYPES

EXPERT_TENSORS = ("gate", "up", "down")


def _u8(buf) -> np.ndarray:
    """A flat uint8 view of a packed tensor (no copy for bytes-like input)."""
    if isinstance(buf, (bytes, bytearray, memoryview)):
        return np.frombuffer(buf, dtype=np.uint8)
    return np.ascontiguousarray(buf, dtype=np.uint8).reshape(-1)


def _status(what: str, code: int) -> None:
    if code != 0:
        raise RuntimeError(f"native {what} failed with status {code}")


class NativeExpert:
    """One quantised SwiGLU expert per call on the B200 (``moe_quant_expert``)."""

    def __init__(self, path: str | Path | None = None, fp16_graph: int = 1):
        self.library = _lib.load(path=path)
        self.fp16_graph = int(fp16_graph)
        self.delta = NativeDelta(self.library) if _lib.exports(self.library,
                                                               "moe_delta_heads") else None

    @property
    def function(self):
        return self.library.moe_quant_expert

    def forward(self, tensors, kinds, activation, hidden, intermediate):
        views = {name: _u8(tensors[name]) for name in EXPERT_TENSORS}
        x = np.ascontiguousarray(activation, dtype=np.float32).reshape(-1)
        if x.size != hidden:
            raise ValueError("native expert activation shape mismatch")
        y = np.empty(hidden, dtype=np.float32)
        triples = [v for name in EXPERT_TENSORS
                   for v in (kinds[name], views[name].ctypes.data, views[name].size)]
        _status("expert", self.function(*triples, x.ctypes.data, hidden, intermediate,
                                        y.ctypes.data, self.fp16_graph))
        return y


class NativeDelta:
    """The DeltaNet decode recurrence of every head in one call."""

    def __init__(self, library=None):
        self.library = library if library is not None else _lib.load()

    @staticmethod
    def _shapes(heads: int, key_dim: int, value_dim: int):
        return [(heads, key_dim), (heads, key_dim), (heads, value_dim), (heads,), (heads,)]

    def forward(self, state, q, k, v, beta, gate):
        """Host arrays: ``state`` (heads, value_dim, key_dim) fp32,
        C-contiguous, updated in place; returns the (heads, value_dim)
        output."""
        if state.dtype != np.float32 or not state.flags.c_contiguous:
            raise ValueError("DeltaNet state must be contiguous FP32")
        heads, value_dim, key_dim = state.shape
        ins = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, beta, gate)]
        if [a.shape for a in ins] != self._shapes(heads, key_dim, value_dim):
            raise ValueError("DeltaNet native input shape mismatch")
        out = np.empty((heads, value_dim), dtype=np.float32)
        ptrs = [state.ctypes.data, *(a.ctypes.data for a in ins), out.ctypes.data]
        _status("DeltaNet", self.library.moe_delta_heads(*ptrs, heads, key_dim, value_dim))
        return out

    def forward_device(self, state, q, k, v, beta, gate, out=None, status=None, stream=None):
        """CUDA tensors, asynchronous on ``stream`` (default: torch's current
        stream) through ``moe_b200_delta_heads``: no host synchronisation.
        ``status`` (int32 CUDA tensor of two elements, optional) receives in
        [0] -1 or the first flat row whose output is not finite, in [1] 0 or
        nonzero when a bounded device-side wait gave up."""
        import torch
        if state.dtype != torch.float32 or not state.is_contiguous() or not state.is_cuda:
            raise ValueError("DeltaNet state must be a contiguous FP32 CUDA tensor")
        heads, value_dim, key_dim = state.shape
        ins = [t.contiguous() for t in (q, k, v, beta, gate)]
        for t, shape in zip(ins, self._shapes(heads, key_dim, value_dim)):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or t.device != state.device:
                raise ValueError("DeltaNet device input shape, dtype or device mismatch")
        if status is not None and (status.dtype != torch.int32 or status.numel() < 2
                                   or not status.is_cuda):
            raise ValueError("DeltaNet status must be an int32 CUDA tensor of two elements")
        if out is None:
            out = torch.empty((heads, value_dim), dtype=torch.float32, device=state.device)
        stream = stream if stream is not None else torch.cuda.current_stream(state.device)
        _status("DeltaNet", self.library.moe_b200_delta_heads(
            state.data_ptr(), *(t.data_ptr() for t in ins), out.data_ptr(), heads, key_dim,
            value_dim, status.data_ptr() if status is not None else None, stream.cuda_stream))
        return out


def cuda_device_count() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # torch without CUDA
        return 0


_MODES = ("auto", "native", "openvino")


def _why_not(device, tensor_types) -> str | None:
    """The first reason this library cannot serve the experts, or None."""
    name = str(device).split(":")[0].upper() if device is not None else "CUDA"
    checks = (
        (name in ("CUDA", "GPU"), f"the B200 expert kernels need a CUDA device, not {device}"),
        (cuda_device_count() > 0, "no CUDA device is visible"),
        (bool(tensor_types) and all(kinds.get(t) in SUPPORTED_TYPES
                                    for kinds in tensor_types.values() for t in EXPERT_TENSORS),
         "expert quantization is unsupported"),
    )
    return next((reason for ok, reason in checks if not ok), None)


def load_native_expert(mode, library, device, tensor_types):
    """``NativeExpert`` over `library` (default: the in-tree build) when it
    can serve `tensor_types` on `device`; None for ``openvino`` and for
    ``auto`` when it cannot; ``native`` raises ``RuntimeError(reason)``."""
    if mode not in _MODES:
        raise ValueError("native_decode must be auto, native, or openvino")
    if mode == "openvino":
        return None
    reason = _why_not(device, tensor_types)
    expert = None
    if reason is None:
        try:
            expert = NativeExpert(library)
        except (OSError, AttributeError, RuntimeError) as error:
            reason = f"kernel unavailable ({error})"
    if expert is not None:
        print("[Experts] native quantized B200 decode; DeltaNet "
              + ("native" if expert.delta is not None else "NumPy"))
        return expert
    if mode == "native":
        raise RuntimeError(reason)
    print(f"[Experts] OpenVINO decode: {reason}")
    return None
