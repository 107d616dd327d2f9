"""The C ABI library: it loads without a GPU, exports every entry point the
header declares, and rejects malformed calls with the reference's status
codes before touching the device."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "moe_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MOE_B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def test_header_declares_reference_exports():
    names = declared_functions()
    for ref_name in ("dequant_k_supported", "dequant_k_block_size", "dequant_k", "moe_quant_expert"):
        assert ref_name in names


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name


def test_library_exports_nothing_else():
    """Only the declared entry points are visible (no CUDA runtime symbols
    that could interpose with another runtime in the process)."""
    import subprocess
    from flash_moe_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.library_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_functions())


def test_version(lib):
    assert lib.moe_b200_version() >= 100


@pytest.mark.parametrize("t,bs", [(8, 32), (11, 256), (12, 256), (13, 256), (14, 256), (2, 0), (999, 0)])
def test_supported_and_block_size(lib, t, bs):
    assert lib.dequant_k_block_size(t) == bs
    assert lib.dequant_k_supported(t) == (1 if bs else 0)


def test_dequant_k_argument_errors(lib):
    raw = np.zeros(144 * 2, np.uint8)
    out = np.zeros(512, np.float32)
    assert lib.dequant_k(999, raw.ctypes.data, out.ctypes.data, 256, 0) == -1
    assert lib.dequant_k(12, None, out.ctypes.data, 256, 0) == -1
    assert lib.dequant_k(12, raw.ctypes.data, None, 256, 0) == -1
    assert lib.dequant_k(12, raw.ctypes.data, out.ctypes.data, 0, 0) == -1
    assert lib.dequant_k(12, raw.ctypes.data, out.ctypes.data, 257, 0) == -1


def test_moe_quant_expert_argument_errors(lib):
    from cases import small_expert_inputs
    tensors, x = small_expert_inputs((12, 12, 12), 0)
    out = np.zeros(256, np.float32)

    def call(kinds=(12, 12, 12), t=tensors, hidden=256, inter=256, fg=0, xp=x.ctypes.data,
             op=out.ctypes.data):
        args = []
        for name, k in zip(("gate", "up", "down"), kinds):
            args += [k, t[name].ctypes.data if t[name] is not None else None,
                     t[name].nbytes if t[name] is not None else 0]
        return lib.moe_quant_expert(*args, xp, hidden, inter, op, fg)

    assert call(xp=None) == -1
    assert call(op=None) == -1
    assert call(fg=2) == -1
    assert call(hidden=0) == -1
    assert call(hidden=65536 + 256) == -1
    assert call(t=dict(tensors, down=None)) == -1
    assert call(kinds=(999, 12, 12)) == -2
    assert call(kinds=(12, 12, 12), hidden=128) == -2
    assert call(t=dict(tensors, up=tensors["up"][:-1])) == -3


def test_decode_rejects_bad_layer(lib):
    from flash_moe_b200 import _lib
    L = _lib.Layer()
    need = C.c_size_t(0)
    assert lib.moe_b200_decode_workspace(C.byref(L), 1, C.byref(need)) == -1
    assert lib.moe_b200_decode_workspace(None, 1, C.byref(need)) == -1


def test_delta_heads_argument_errors(lib, golden):
    """moe_delta_heads rejects what the reference rejects (-1), before any
    device work; the reference's own statuses are in the golden fixture."""
    g = golden("delta")
    state = np.zeros((2, 8, 8), np.float32)
    vec = np.zeros(8 * 8, np.float32)
    p = [state.ctypes.data] + [vec.ctypes.data] * 6
    bad = {"heads0": (0, 8, 8), "heads257": (257, 8, 8), "dk0": (1, 0, 8),
           "dk1025": (1, 1025, 8), "dv0": (1, 8, 0), "dv1025": (1, 8, 1025)}
    for key, (h, dk, dv) in bad.items():
        assert lib.moe_delta_heads(*p, h, dk, dv) == int(g[f"rc_{key}"]) == -1, key
        assert lib.moe_b200_delta_heads(*p, h, dk, dv, None, None) == -1, key
    for i in range(7):
        q = list(p)
        q[i] = None
        assert lib.moe_delta_heads(*q, 1, 8, 8) == int(g["rc_null"]) == -1
        assert lib.moe_b200_delta_heads(*q, 1, 8, 8, None, None) == -1
    odd = list(p)
    odd[1] = vec.ctypes.data + 2
    assert lib.moe_b200_delta_heads(*odd, 1, 8, 8, None, None) == -7


def test_native_delta_checks_shapes_like_the_reference():
    from flash_moe_b200.native_expert import NativeDelta
    nd = NativeDelta()
    state = np.zeros((2, 4, 8), np.float32)
    q = k = np.zeros((2, 8), np.float32)
    v = np.zeros((2, 4), np.float32)
    b = g = np.zeros(2, np.float32)
    with pytest.raises(ValueError, match="contiguous FP32"):
        nd.forward(state.astype(np.float64), q, k, v, b, g)
    with pytest.raises(ValueError, match="contiguous FP32"):
        nd.forward(np.zeros((2, 8, 4), np.float32).transpose(0, 2, 1), q, k, v, b, g)
    with pytest.raises(ValueError, match="shape mismatch"):
        nd.forward(state, q, k, np.zeros((2, 5), np.float32), b, g)
