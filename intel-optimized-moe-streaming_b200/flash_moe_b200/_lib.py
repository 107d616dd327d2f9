"""ctypes binding of ``libmoe_b200.so`` (declared in ``include/moe_b200.h``).

There is no CPU fallback: if the library cannot be loaded, every entry point
raises.  The library is built in-tree (``_build.py``) and loaded from this
package directory, so a GPU run always executes the sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from ._build import LIB, build_library, up_to_date

_lock = threading.Lock()
_lib: C.CDLL | None = None

STATUS = {
    0: "ok", -1: "bad argument", -2: "unsupported type or column count",
    -3: "byte count does not match shape", -4: "non-finite output",
    -5: "host-side failure", -6: "CUDA call failed", -7: "device pointer not 16-byte aligned",
    -8: "workspace too small", -9: "device wait timed out",
    -10: "prefill activation outside the fp16 range",
}

FP16_GRAPH = 1
NO_SHARED = 2
EXACT = 4
SHARED_ONLY = 8
TCGEN05 = 16
EP_BLOB_BYTES = 128  # MOE_B200_EP_BLOB_BYTES
STEP_CHAIN = 1
STEP_BLOCK = 2


class Layer(C.Structure):
    """Mirror of ``struct moe_b200_layer``."""

    _fields_ = [
        ("hidden", C.c_int32), ("intermediate", C.c_int32), ("n_experts", C.c_int32),
        ("top_k", C.c_int32), ("expert_begin", C.c_int32), ("expert_count", C.c_int32),
        ("gate_type", C.c_int32), ("up_type", C.c_int32), ("down_type", C.c_int32),
        ("shared_intermediate", C.c_int32), ("shared_gate_type", C.c_int32),
        ("shared_up_type", C.c_int32), ("shared_down_type", C.c_int32), ("flags", C.c_int32),
        ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
        ("router", C.c_void_p), ("router_bias", C.c_void_p),
        ("shared_gate", C.c_void_p), ("shared_up", C.c_void_p), ("shared_down", C.c_void_p),
        ("shared_gate_inp", C.c_void_p),
    ]


class Step(C.Structure):
    """Mirror of ``struct moe_b200_step``."""

    _fields_ = [
        ("layer", C.c_int32), ("flags", C.c_int32), ("x", C.c_void_p), ("y", C.c_void_p),
        ("topk_ids", C.c_void_p), ("topk_weights", C.c_void_p),
    ]


def exports(lib: C.CDLL, name: str) -> bool:
    """Whether the loaded library exports `name`."""
    try:
        getattr(lib, name)
    except AttributeError:
        return False
    return True


def _bind(lib: C.CDLL) -> None:
    i, i64, vp, f = C.c_int, C.c_int64, C.c_void_p, C.c_float
    sigs = {
        "dequant_k_supported": (i, [i]),
        "dequant_k_block_size": (i, [i]),
        "dequant_k": (i, [i, vp, vp, i64, i]),
        "moe_quant_expert": (i, [i, vp, i64] * 3 + [vp, i, i, vp, i]),
        "moe_b200_decode_workspace": (i, [C.POINTER(Layer), C.c_int32, C.POINTER(C.c_size_t)]),
        "moe_b200_decode_kernels": (i, [C.POINTER(Layer), C.c_int32, C.POINTER(C.c_int)]),
        "moe_b200_decode": (i, [C.POINTER(Layer), vp, C.c_int32, vp, vp, vp, vp, C.c_size_t, vp]),
        "moe_b200_decode_host_workspace": (i, [C.POINTER(Layer), C.c_int32,
                                               C.POINTER(C.c_size_t)]),
        "moe_b200_decode_host": (i, [C.POINTER(Layer), vp, C.c_int32, vp, vp, vp, vp, C.c_size_t,
                                     vp]),
        "moe_b200_prefill": (i, [C.POINTER(Layer), vp, C.c_int32, C.c_int32, vp, vp, vp, vp,
                                 C.c_size_t, vp]),
        "moe_b200_prefill_workspace": (i, [C.POINTER(Layer), C.c_int32, C.POINTER(C.c_size_t)]),
        "moe_b200_decode_steps": (i, [C.POINTER(Layer), vp, vp, C.c_int32, C.c_float, vp,
                                      C.c_size_t, vp]),
        "moe_b200_decode_ep": (i, [C.POINTER(Layer), vp, C.c_int32, C.c_int32, C.c_int32, vp, vp,
                                   vp, vp, C.c_size_t, vp]),
        "moe_b200_ep_create": (i, [C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.POINTER(C.c_void_p), vp]),
        "moe_b200_ep_connect": (i, [vp, vp]),
        "moe_b200_ep_destroy": (i, [vp]),
        "moe_b200_decode_ep_p2p": (i, [C.POINTER(Layer), vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
        "moe_b200_block_prepare": (i, [vp, vp, vp, C.c_int32, C.c_int32, C.c_float, vp]),
        "moe_b200_block_finish": (i, [vp, vp, vp, C.c_int32, C.c_int32, vp]),
        "moe_b200_prefill_supported": (i, [C.POINTER(Layer)]),
        "moe_b200_prefill_kernels": (i, [C.POINTER(Layer), C.c_int32, C.POINTER(C.c_int)]),
        "moe_b200_dequant": (i, [i, vp, vp, i64, i, vp]),
        "moe_delta_heads": (i, [vp] * 7 + [i] * 3),
        "moe_b200_delta_heads": (i, [vp] * 7 + [i] * 3 + [vp, vp]),
        "moe_b200_expert_noalloc": (i, [i, vp, i64] * 3 + [vp, i, i, vp, i, vp]),
        "moe_b200_last_cuda_error": (i, []),
        "moe_b200_workspace_init": (i, [vp, C.c_size_t, vp]),
        "moe_b200_set_trace": (i, [vp, i]),
        "moe_b200_workspace_error": (i, [vp, vp, C.POINTER(C.c_int)]),
        "moe_b200_version": (i, []),
    }
    for name, (res, args) in sigs.items():
        if not exports(lib, name):
            continue
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del f


def library_path() -> Path:
    return LIB


_extra: dict[str, C.CDLL] = {}


def load(build_if_missing: bool = True, path: str | Path | None = None) -> C.CDLL:
    """Load (building first when sources are newer and nvcc is present).

    ``path`` names another build of the library (same exports) instead of
    the in-tree one; it is loaded once per resolved path."""
    global _lib
    if path is not None and Path(path).resolve() != LIB.resolve():
        key = str(Path(path).resolve())
        with _lock:
            if key not in _extra:
                other = C.CDLL(key)
                _bind(other)
                _extra[key] = other
            return _extra[key]
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_missing and not up_to_date():
            try:
                build_library()
            except RuntimeError:
                if not LIB.exists():
                    raise
        if not LIB.exists():
            raise RuntimeError(f"B200 library missing: {LIB} (run __graft_entry__.build())")
        lib = C.CDLL(str(LIB))
        _bind(lib)
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    """Raise like the reference binding does on a nonzero status
    (``src/flash_moe/native_expert.py:35-36``)."""
    if status:
        extra = ""
        if status == -6 and _lib is not None:
            extra = f" (cudaError {_lib.moe_b200_last_cuda_error()})"
        raise RuntimeError(f"{what} failed with status {status}: "
                           f"{STATUS.get(status, 'unknown')}{extra}")
