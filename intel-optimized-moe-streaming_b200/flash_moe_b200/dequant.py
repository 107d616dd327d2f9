"""Drop-ins for the reference's dequantisation entry points, on the GPU.

* ``dequant_to_f16(raw, ggml_type, n_elements, out=None)`` -- the reference
  binding of ``dequant_k`` (``src/run_q4k_f16_openvino.py:62-85``): binary16
  output, an ``out`` buffer of the wrong size/dtype or read-only is ignored
  and a new one allocated.  The reference falls back to ``gguf.quants`` when
  its DLL is missing; this one has no CPU path and raises instead.
* ``dequantize(raw, ggml_type, shape=None)`` -- fp32 output, the contract of
  ``flash_moe.dequant.dequantize`` (``src/flash_moe/dequant.py:109-128``).
* ``dequantize_device(src, ggml_type, n, dtype)`` -- device tensor in,
  device tensor out, asynchronous on the current stream.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .formats import BLOCK


def _as_u8(raw) -> np.ndarray:
    if isinstance(raw, (bytes, bytearray, memoryview)):
        return np.frombuffer(raw, dtype=np.uint8)
    return np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)


def dequant_to_f16(raw, ggml_type: int, n_elements: int, out: np.ndarray | None = None) -> np.ndarray:
    if out is not None and (out.dtype != np.float16 or out.size != n_elements
                            or not out.flags.writeable or not out.flags.c_contiguous):
        out = None
    if out is None:
        out = np.empty(n_elements, dtype=np.float16)
    src = _as_u8(raw)
    lib = _lib.load()
    rc = lib.dequant_k(int(ggml_type), src.ctypes.data, out.ctypes.data, int(n_elements), 1)
    _lib.check(rc, "dequant_k")
    return out


def dequantize(raw, ggml_type: int, shape: tuple[int, ...] | None = None) -> np.ndarray:
    src = _as_u8(raw)
    if src.size == 0:
        raise ValueError("empty buffer passed to dequantize")
    bs, pb = BLOCK.get(int(ggml_type), (0, 0))
    if pb == 0 or src.nbytes % pb:
        raise ValueError(f"{src.nbytes} bytes is not a whole number of type-{ggml_type} blocks")
    n = src.nbytes // pb * bs
    out = np.empty(n, dtype=np.float32)
    rc = _lib.load().dequant_k(int(ggml_type), src.ctypes.data, out.ctypes.data, n, 0)
    _lib.check(rc, "dequant_k")
    return out.reshape(shape) if shape is not None else out


def dequantize_device(src, ggml_type: int, n_elements: int, dtype=None, out=None, stream=None):
    """``src``: device uint8 tensor of packed blocks.  Returns a device tensor
    of fp32 (default) or float16 values."""
    import torch
    dtype = torch.float32 if dtype is None else dtype
    if dtype not in (torch.float32, torch.float16):
        raise ValueError("dtype must be torch.float32 or torch.float16")
    if out is None:
        out = torch.empty(n_elements, dtype=dtype, device=src.device)
    if stream is None:
        stream = torch.cuda.current_stream(src.device)
    rc = _lib.load().moe_b200_dequant(int(ggml_type), src.data_ptr(), out.data_ptr(),
                                      int(n_elements), 1 if dtype == torch.float16 else 0,
                                      stream.cuda_stream)
    _lib.check(rc, "moe_b200_dequant")
    return out
