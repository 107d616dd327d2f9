"""moe_quant_expert on the GPU through the C ABI, against the oracle.

Mirrors the reference's native test (tools/test_optimized_inference.py:
231-264): eight type triples over Q8_0/Q3_K/Q4_K/Q5_K/Q6_K at 256x256, both
fp16_graph modes, 8 concurrent calls bit-identical, an unsupported type ->
"status -2"; plus the full-size config-1 expert.

Tolerance: max|y - ref| / max|ref| <= 1e-3 in fp32 mode (the contract;
the exact engine lands near 1e-6), 5e-3 in fp16_graph mode (the reference's
own bound for that mode, test_optimized_inference.py:259-260)."""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle as O
from cases import TRIPLES, small_expert_inputs
from flash_moe_b200 import synth
from flash_moe_b200.native_expert import NativeExpert

pytestmark = pytest.mark.gpu

TOL = {0: 1e-3, 1: 5e-3}


@pytest.mark.parametrize("i", range(len(TRIPLES)))
@pytest.mark.parametrize("fg", [0, 1])
def test_expert_triples_match_oracle(oracle, i, fg):
    tensors, x = small_expert_inputs(TRIPLES[i], i)
    kinds = dict(zip(("gate", "up", "down"), TRIPLES[i]))
    native = NativeExpert(fp16_graph=fg)
    with ThreadPoolExecutor(4) as pool:
        results = list(pool.map(lambda _: native.forward(tensors, kinds, x, 256, 256), range(8)))
    rc, want = oracle.expert(tensors, kinds, x, 256, 256, fg)
    assert rc == 0
    err = O.max_relative_error(results[0], want)
    assert err <= TOL[fg], err
    for got in results:
        np.testing.assert_array_equal(got, results[0])
    with pytest.raises(RuntimeError, match="status -2"):
        native.forward(tensors, dict(kinds, gate=999), x, 256, 256)


def test_expert_golden_small(golden):
    g = golden("expert_small")
    for i, kinds in enumerate(TRIPLES):
        tensors, x = small_expert_inputs(kinds, i)
        k = dict(zip(("gate", "up", "down"), kinds))
        for fg in (0, 1):
            y = NativeExpert(fp16_graph=fg).forward(tensors, k, x, 256, 256)
            assert O.max_relative_error(y, g[f"y{fg}_{i}"]) <= TOL[fg]


def test_expert_config1_fp32(oracle, golden):
    g = golden("expert_cfg1")
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    y = NativeExpert(fp16_graph=0).forward(tensors, kinds, x, 2048, 512)
    err = O.max_relative_error(y, g["y0"])
    assert err <= 1e-3, err


def test_expert_config1_fp16_overflow_status(lib, oracle):
    """At config-1 value ranges the binary16 output overflows; the GPU path
    returns -4 like the reference and writes the rows up to the first
    non-finite one."""
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    rc_o, want = oracle.expert(tensors, kinds, x, 2048, 512, 1)
    args = []
    for name in ("gate", "up", "down"):
        args += [kinds[name], tensors[name].ctypes.data, tensors[name].nbytes]
    out = np.full(2048, 7.0, np.float32)
    rc = lib.moe_quant_expert(*args, x.ctypes.data, 2048, 512, out.ctypes.data, 1)
    assert rc == rc_o == -4
    bad = int(np.argmax(~np.isfinite(out)))
    assert not np.isfinite(out[bad])
    assert np.all(out[bad + 1:] == 7.0)


def test_expert_device_pointers(lib, oracle):
    import torch
    tensors, x = small_expert_inputs(TRIPLES[1], 1)
    kinds = dict(zip(("gate", "up", "down"), TRIPLES[1]))
    dev = {k: torch.from_numpy(v).cuda() for k, v in tensors.items()}
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(256, dtype=torch.float32, device="cuda")
    args = []
    for name in ("gate", "up", "down"):
        args += [kinds[name], dev[name].data_ptr(), dev[name].numel()]
    assert lib.moe_quant_expert(*args, xd.data_ptr(), 256, 256, yd.data_ptr(), 0) == 0
    _, want = oracle.expert(tensors, kinds, x, 256, 256, 0)
    assert O.max_relative_error(yd.cpu().numpy(), want) <= 1e-3
