"""Drop-in for the reference's ctypes binding of the native expert kernel
(``src/flash_moe/native_expert.py``), backed by ``libmoe_b200.so``.

``NativeExpert(path).forward(tensors, kinds, activation, hidden, inter)``
has the reference's arguments, result and error behaviour: the three packed
byte buffers go to ``moe_quant_expert`` (here the sm_100a kernel), a nonzero
status raises ``RuntimeError("native expert failed with status N")``.  Like
the reference it passes ``fp16_graph=1`` unless told otherwise.

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
        # moe_delta_heads (DeltaNet) is not part of this library; callers
        # fall back to their NumPy recurrence as the reference does when the
        # symbol is absent (native_expert.py:21).
        self.delta = None

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
            return result
    if mode == "native":
        raise RuntimeError(reason)
    print(f"[Experts] OpenVINO decode: {reason}")
    return None
