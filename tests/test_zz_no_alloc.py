"""The no-allocation single-expert entry point (moe_b200_expert_noalloc).

It serves callers that cannot allocate device memory -- a process whose
memory is all reserved by its own pool, or a thread that must not enter the
CUDA allocator while other work runs.  Its scratch is a fixed array inside
the library.  This test calls it through the C ABI, twice in a row with
different tokens, and checks each result against the allocating entry point
(moe_quant_expert on the same device buffers) and against the CPU oracle's
moe_quant_expert (the restatement of cpp/moe_quant_dot.cpp:171-214), with
the expert tests' tolerance: the oracle catches an error the two device
paths would share, such as in the plan the no-allocation entry fills in
itself.  It runs last in the suite and also passes on its own in a fresh
process.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import TRIPLES, small_expert_inputs
from flash_moe_b200 import synth

pytestmark = pytest.mark.gpu
TOL = {0: 1e-3, 1: 5e-3}


def _dev(arrays):
    import torch
    return {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in arrays.items()}


def _args(kinds, dev):
    args = []
    for name in ("gate", "up", "down"):
        args += [kinds[name], dev[name].data_ptr(), dev[name].numel()]
    return args


@pytest.mark.parametrize("case", ["triple", "config1"])
@pytest.mark.parametrize("fg", [0, 1])
def test_noalloc_matches_allocating_entry_point(lib, oracle, case, fg):
    import torch
    if case == "triple":
        tensors, x0 = small_expert_inputs(TRIPLES[1], 1)
        kinds = dict(zip(("gate", "up", "down"), TRIPLES[1]))
        hidden = inter = 256
        x1 = (x0[::-1] * 1.5).astype(np.float32).copy()
    else:
        if fg:
            pytest.skip("the config-1 expert overflows binary16 (status -4 in the reference)")
        tensors, kinds, x0 = synth.make_expert_q4k(seed=1)
        hidden, inter = 2048, 512
        x1 = synth.make_tokens(9, 1, hidden)[0]
    dev = _dev(tensors)
    args = _args(kinds, dev)
    stream = torch.cuda.current_stream()
    for x in (x0, x1):  # two calls in a row on the shared scratch
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        want = torch.empty(hidden, dtype=torch.float32, device="cuda")
        got = torch.full((hidden,), float("nan"), dtype=torch.float32, device="cuda")
        assert lib.moe_quant_expert(*args, xd.data_ptr(), hidden, inter, want.data_ptr(), fg) == 0
        rc = lib.moe_b200_expert_noalloc(*args, xd.data_ptr(), hidden, inter, got.data_ptr(), fg,
                                         stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        got_h = got.cpu().numpy()
        err = O.max_relative_error(got_h, want.cpu().numpy())
        assert err <= TOL[fg], err
        rc, ref = oracle.expert(tensors, kinds, x, hidden, inter, fg)
        assert rc == 0
        err = O.max_relative_error(got_h, ref)
        assert err <= TOL[fg], err


def test_noalloc_rejects_oversize_and_host_pointers(lib):
    import torch
    tensors, x = small_expert_inputs(TRIPLES[1], 1)
    kinds = dict(zip(("gate", "up", "down"), TRIPLES[1]))
    dev = _dev(tensors)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(256, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # intermediate above the fixed scratch size: rejected before any launch
    big = 16384 + 256
    assert lib.moe_b200_expert_noalloc(
        kinds["gate"], dev["gate"].data_ptr(), 256 * (big // 256) * 144 // 144,
        kinds["up"], dev["up"].data_ptr(), 1, kinds["down"], dev["down"].data_ptr(), 1,
        xd.data_ptr(), 256, big, out.data_ptr(), 0, s) == -1
    # host buffers are not accepted (every pointer must be device memory)
    host_out = np.empty(256, np.float32)
    assert lib.moe_b200_expert_noalloc(*_args(kinds, dev), xd.data_ptr(), 256, 256,
                                       host_out.ctypes.data, 0, s) == -1
