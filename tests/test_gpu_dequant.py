"""GPU dequantisation through the C ABI, bit for bit against the oracle.

Covers every format, fp32 and binary16 output, host and device pointers,
ragged block counts (not a multiple of the kernel's 2048-value chunk), a
misaligned source, and the config-1 tensor size."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from flash_moe_b200 import synth
from flash_moe_b200.formats import BLOCK

pytestmark = pytest.mark.gpu
TYPES = [8, 11, 12, 13, 14]


def gpu_dequant_host(lib, t, raw, n, f16):
    out = np.zeros(n, np.uint16 if f16 else np.float32)
    rc = lib.dequant_k(t, raw.ctypes.data, out.ctypes.data, n, 1 if f16 else 0)
    return rc, out


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("nblocks", [1, 3, 8, 9, 64, 65, 1000])
@pytest.mark.parametrize("f16", [False, True])
def test_dequant_host_pointers_bit_exact(lib, oracle, t, nblocks, f16):
    rng = np.random.default_rng(np.random.SeedSequence([1, t, nblocks]))
    raw = synth.quant_blocks(rng, t, nblocks).reshape(-1)
    n = nblocks * BLOCK[t][0]
    rc, got = gpu_dequant_host(lib, t, raw, n, f16)
    assert rc == 0
    orc, want = oracle.dequant(t, raw, want_f16=f16)
    assert orc == 0
    np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("t", TYPES)
def test_dequant_golden_blocks(lib, golden, t):
    g = golden("dequant_blocks")
    raw = g[f"raw_{t}"]
    n = raw.size // BLOCK[t][1] * BLOCK[t][0]
    rc, got = gpu_dequant_host(lib, t, raw, n, False)
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint32), g[f"f32_{t}"].view(np.uint32))
    rc, got16 = gpu_dequant_host(lib, t, raw, n, True)
    assert rc == 0
    np.testing.assert_array_equal(got16, g[f"f16_{t}"])
    assert gpu_dequant_host(lib, t, raw, n + 1, False)[0] == int(g[f"bad_n_status_{t}"])


@pytest.mark.parametrize("t", TYPES)
def test_dequant_device_pointers_and_misaligned_source(lib, oracle, t):
    import torch
    rng = np.random.default_rng(np.random.SeedSequence([2, t]))
    nblocks = 77
    raw = synth.quant_blocks(rng, t, nblocks).reshape(-1)
    n = nblocks * BLOCK[t][0]
    _, want = oracle.dequant(t, raw)
    # offset the packed bytes by one byte inside a device buffer
    dev = torch.zeros(raw.size + 1, dtype=torch.uint8, device="cuda")
    dev[1:] = torch.from_numpy(raw).cuda()
    for off in (0, 1):
        src = dev[1:] if off else torch.from_numpy(raw).cuda()
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        s = torch.cuda.current_stream()
        rc = lib.moe_b200_dequant(t, src.data_ptr(), out.data_ptr(), n, 0, s.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    # the reference-compatible entry point also takes device pointers in place
    out = torch.empty(n, dtype=torch.float16, device="cuda")
    assert lib.dequant_k(t, dev[1:].data_ptr(), out.data_ptr(), n, 1) == 0
    _, want16 = oracle.dequant(t, raw, want_f16=True)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), want16.view(np.uint16))


def test_dequant_config1_tensor(lib, oracle):
    tensors, kinds, _ = synth.make_expert_q4k(seed=1)
    raw = tensors["gate"]
    n = 512 * 2048
    for f16 in (False, True):
        rc, got = gpu_dequant_host(lib, 12, raw, n, f16)
        assert rc == 0
        _, want = oracle.dequant(12, raw, want_f16=f16)
        np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))


def test_dequant_to_f16_drop_in(oracle):
    from flash_moe_b200.dequant import dequant_to_f16, dequantize
    rng = np.random.default_rng(5)
    raw = synth.quant_blocks(rng, 11, 16).reshape(-1)
    n = 16 * 256
    out = np.empty(n, np.float16)
    got = dequant_to_f16(raw.tobytes(), 11, n, out=out)
    assert got is out
    _, want = oracle.dequant(11, raw, want_f16=True)
    np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
    wrong = np.empty(n - 1, np.float16)
    assert dequant_to_f16(raw.tobytes(), 11, n, out=wrong) is not wrong
    _, want32 = oracle.dequant(11, raw)
    np.testing.assert_array_equal(dequantize(raw, 11).view(np.uint32), want32.view(np.uint32))
