"""Drop-in for the reference's ctypes binding of the native expert kernel
(``src/flash_moe/native_expert.py``), backed by ``libmoe_b200.so``.

``NativeExpert(path).forward(tensors, kinds, activation, hidden, inter)``
has the reference's arguments, result and error behaviour: the three packed
byte buffers go to ``moe_quant_expert`` (here the sm_100a kernel), a nonzero
status raises ``RuntimeError("native expert failed with status N")``.  Like
the reference it passes ``fp16_graph=1`` unless told otherwise.

``NativeDelta(library).forward(state, q, k, v, beta, gate)`` is the
reference's DeltaNet binding (``native_expert.py:76-98``) over the sm_100a
``moe_delta_heads``: same shapes, checks, in-place state update and
``RuntimeError("native DeltaNet failed with status N")``.  ``NativeExpert``
exposes it as ``.delta`` like the reference (``native_expert.py:21``).

``load_native_expert(mode, library, device, tensor_types)`` keeps the
reference's ``auto|native|openvino`` policy (``native_expert.py:40-75``): the
gate is a visible CUDA device instead of a CPU with AVX2/FMA/F16C, and
``native`` raises ``RuntimeError`` with the reason when the library cannot
run.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import _lib
from .formats import SUPPORTED_TYPES


class NativeExpert:
    def __init__(self, path: Path | None = None, fp16_graph: int = 1):
        if path is None:
            self.library = _lib.load()
        else:
            self.library = C.CDLL(str(Path(path).resolve()))
            _lib._bind(self.library)
        self.function = self.library.moe_quant_expert
        self.fp16_graph = int(fp16_graph)
        self.delta = NativeDelta(self.library) if hasattr(self.library, "moe_delta_heads") else None

    def forward(self, tensors, kinds, activation, hidden, intermediate):
        arrays = [np.frombuffer(tensors[name], np.uint8) if isinstance(tensors[name], (bytes, bytearray))
                  else np.ascontiguousarray(tensors[name], dtype=np.uint8).reshape(-1)
                  for name in ("gate", "up", "down")]
        args = []
        for name, raw in zip(("gate", "up", "down"), arrays):
            args.extend((kinds[name], raw.ctypes.data, raw.nbytes))
        x = np.ascontiguousarray(activation, dtype=np.float32).reshape(-1)
        if x.size != hidden:
            raise ValueError("native expert activation shape mismatch")
        out = np.empty(hidden, np.float32)
        code = self.function(*args, x.ctypes.data, hidden, intermediate,
                             out.ctypes.data, self.fp16_graph)
        if code:
            raise RuntimeError(f"native expert failed with status {code}")
        return out


class NativeDelta:
    """All-head fp32 DeltaNet state update on the GPU (``moe_delta_heads``)."""

    def __init__(self, library=None):
        self.library = library if library is not None else _lib.load()
        self.function = self.library.moe_delta_heads
        self.function.argtypes = [C.c_void_p] * 7 + [C.c_int] * 3
        self.function.restype = C.c_int

    def forward(self, state, q, k, v, beta, gate):
        """Host arrays, as the reference: ``state`` (heads, value_dim,
        key_dim) fp32 C-contiguous, updated in place; returns the
        (heads, value_dim) output."""
        if state.dtype != np.float32 or not state.flags.c_contiguous:
            raise ValueError("DeltaNet state must be contiguous FP32")
        nv, dv, dk = state.shape
        arrays = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, beta, gate)]
        shapes = [(nv, dk), (nv, dk), (nv, dv), (nv,), (nv,)]
        if any(a.shape != shape for a, shape in zip(arrays, shapes)):
            raise ValueError("DeltaNet native input shape mismatch")
        out = np.empty((nv, dv), np.float32)
        pointers = [state.ctypes.data] + [a.ctypes.data for a in arrays] + [out.ctypes.data]
        code = self.function(*pointers, nv, dk, dv)
        if code:
            raise RuntimeError(f"native DeltaNet failed with status {code}")
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
        nv, dv, dk = state.shape
        ins = [t.contiguous() for t in (q, k, v, beta, gate)]
        shapes = [(nv, dk), (nv, dk), (nv, dv), (nv,), (nv,)]
        for t, shape in zip(ins, shapes):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or t.device != state.device:
                raise ValueError("DeltaNet device input shape, dtype or device mismatch")
        if status is not None and (status.dtype != torch.int32 or status.numel() < 2
                                   or not status.is_cuda):
            raise ValueError("DeltaNet status must be an int32 CUDA tensor of two elements")
        if out is None:
            out = torch.empty((nv, dv), dtype=torch.float32, device=state.device)
        handle = (stream if stream is not None else torch.cuda.current_stream(state.device)).cuda_stream
        code = self.library.moe_b200_delta_heads(
            state.data_ptr(), *(t.data_ptr() for t in ins), out.data_ptr(), nv, dk, dv,
            status.data_ptr() if status is not None else None, handle)
        if code:
            raise RuntimeError(f"native DeltaNet failed with status {code}")
        return out


def cuda_device_count() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # torch without CUDA
        return 0


def load_native_expert(mode, library, device, tensor_types):
    if mode not in ("auto", "native", "openvino"):
        raise ValueError("native_decode must be auto, native, or openvino")
    if mode == "openvino":
        return None
    reason = None
    if cuda_device_count() < 1:
        reason = "native experts require a CUDA device (B200)"
    elif not tensor_types or any(
        kinds.get(name) not in SUPPORTED_TYPES
        for kinds in tensor_types.values() for name in ("gate", "up", "down")
    ):
        reason = "expert quantization is unsupported"
    if reason is None:
        try:
            result = NativeExpert(library)
        except (OSError, AttributeError, RuntimeError) as error:
            reason = f"kernel unavailable ({error})"
        else:
            print("[Experts] native quantized B200 decode")
            print("[DeltaNet] native FP32 decode recurrence (B200)")
            return result
    if mode == "native":
        raise RuntimeError(reason)
    print(f"[Experts] OpenVINO decode: {reason}")
    return None
