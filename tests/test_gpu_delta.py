"""moe_delta_heads (the DeltaNet decode step) on the GPU, against the
reference's own outputs (golden fixtures made with its library) and the
oracle.

The host entry point (the reference's ctypes call, NativeDelta.forward) must
give the reference's bits: outputs, the state after every step and, for a
non-finite output, the reference's early stop (status -2, later rows of the
host state untouched, no output from the failing row on).

The device entry point computes exp(gate) with CUDA's double exp instead of
the host libm.  When the two decays agree bit for bit (checked per case) the
device path must be bit-exact as well; otherwise a decayed value can move by
one float ulp, so the bound is max|got - want| / max|want| <= 1e-6.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

import oracle as O
from cases import DELTA_POISON, DELTA_SPECS, delta_case
from flash_moe_b200 import synth
from flash_moe_b200.native_expert import NativeDelta, NativeExpert

pytestmark = pytest.mark.gpu

FINITE = [n for n in DELTA_SPECS if n != "poison"]


@pytest.mark.parametrize("name", FINITE)
def test_host_entry_matches_reference_bits(golden, name):
    g = golden("delta")
    nd = NativeDelta()
    state, steps = delta_case(name)
    ys = [nd.forward(state, *st) for st in steps]
    np.testing.assert_array_equal(np.stack(ys).view(np.uint32), g[f"{name}_y"].view(np.uint32))
    assert synth.digest(state) == str(g[f"{name}_state_sha"])


def test_native_expert_exposes_delta():
    assert isinstance(NativeExpert().delta, NativeDelta)


def test_host_entry_poison_stops_like_the_reference(golden, lib):
    g = golden("delta")
    state, steps = delta_case("poison")
    with pytest.raises(RuntimeError, match="status -2"):
        NativeDelta().forward(state, *steps[0])
    np.testing.assert_array_equal(state.view(np.uint32), g["poison_state"].view(np.uint32))
    # the raw call: outputs before the failing row written, the rest untouched
    state, steps = delta_case("poison")
    heads, dv, dk = state.shape
    out = np.full((heads, dv), np.nan, np.float32)
    arrays = [np.ascontiguousarray(a, np.float32) for a in steps[0]]
    rc = lib.moe_delta_heads(state.ctypes.data, *(a.ctypes.data for a in arrays),
                             out.ctypes.data, heads, dk, dv)
    assert rc == int(g["poison_rc"][0]) == -2
    np.testing.assert_array_equal(out.view(np.uint32), g["poison_y"][0].view(np.uint32))


def test_host_entry_device_state_in_place(golden, lib):
    """state in device memory, the rest on the host: same bits."""
    g = golden("delta")
    state, steps = delta_case("odd")
    dstate = torch.from_numpy(state).cuda()
    heads, dv, dk = state.shape
    ys = []
    for st in steps:
        out = np.empty((heads, dv), np.float32)
        arrays = [np.ascontiguousarray(a, np.float32) for a in st]
        rc = lib.moe_delta_heads(dstate.data_ptr(), *(a.ctypes.data for a in arrays),
                                 out.ctypes.data, heads, dk, dv)
        assert rc == 0
        ys.append(out)
    np.testing.assert_array_equal(np.stack(ys).view(np.uint32), g["odd_y"].view(np.uint32))
    assert synth.digest(dstate.cpu().numpy()) == str(g["odd_state_sha"])


def _device_decay_agrees(steps) -> bool:
    for st in steps:
        gate = st[4].astype(np.float64)
        dev = torch.from_numpy(gate).cuda().exp().cpu().numpy()
        if not np.array_equal(dev.view(np.uint64), np.exp(gate).view(np.uint64)):
            return False
    return True


@pytest.mark.parametrize("name", FINITE)
def test_device_entry_matches_oracle(oracle, name):
    state, steps = delta_case(name)
    dstate = torch.from_numpy(state.copy()).cuda()
    nd = NativeDelta()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    got, want = [], []
    for st in steps:
        dins = [torch.from_numpy(a).cuda() for a in st]
        got.append(nd.forward_device(dstate, *dins, status=status).cpu().numpy())
        assert status.tolist() == [-1, 0]
        rc, y = oracle.delta_heads(state, *st)
        assert rc == 0
        want.append(y)
    got, want = np.stack(got), np.stack(want)
    gstate = dstate.cpu().numpy()
    if _device_decay_agrees(steps):
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        np.testing.assert_array_equal(gstate.view(np.uint32), state.view(np.uint32))
    else:
        assert O.max_relative_error(got, want) <= 1e-6
        assert O.max_relative_error(gstate, state) <= 1e-6


def test_device_entry_reports_first_bad_row():
    state, steps = delta_case("poison")
    heads, dv, dk = state.shape
    dstate = torch.from_numpy(state).cuda()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    out = NativeDelta().forward_device(dstate, *[torch.from_numpy(a).cuda() for a in steps[0]],
                                       status=status)
    h, r = DELTA_POISON
    assert status.tolist() == [h * dv + r, 0]
    assert not np.isfinite(out.cpu().numpy()[h, r])


def test_device_entry_in_a_cuda_graph(oracle):
    """Capturable: a graph of two steps replayed gives two more steps."""
    state, steps = delta_case("model")
    nd = NativeDelta()
    dstate = torch.from_numpy(state.copy()).cuda()
    ins = [[torch.from_numpy(a).cuda() for a in st] for st in steps[:2]]
    outs = [torch.empty(state.shape[:2], device="cuda") for _ in range(2)]
    nd.forward_device(dstate, *ins[0], out=outs[0])   # warm up outside the capture
    torch.cuda.synchronize()
    dstate.copy_(torch.from_numpy(state))
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(2):
                nd.forward_device(dstate, *ins[i], out=outs[i], stream=s)
    dstate.copy_(torch.from_numpy(state))
    graph.replay()
    torch.cuda.synchronize()
    ref_state = state.copy()
    for i in range(2):
        rc, y = oracle.delta_heads(ref_state, *steps[i])
        assert rc == 0
        assert O.max_relative_error(outs[i].cpu().numpy(), y) <= 1e-6
    assert O.max_relative_error(dstate.cpu().numpy(), ref_state) <= 1e-6


def test_device_entry_large_state_properties():
    """Maximum sizes through size-independent properties: with gate = 0
    (decay 1) and beta = 0 the step leaves the state unchanged and the output
    is state . q; with k = 0 the state is only decayed."""
    heads, dk, dv = 256, 1024, 64
    nd = NativeDelta()
    torch.manual_seed(3)
    state = torch.randn(heads, dv, dk, device="cuda") * 0.1
    q = torch.randn(heads, dk, device="cuda") / 32
    k = torch.randn(heads, dk, device="cuda") / 32
    v = torch.randn(heads, dv, device="cuda")
    zero = torch.zeros(heads, device="cuda")
    before = state.clone()
    out = nd.forward_device(state, q, k, v, zero, zero)
    torch.cuda.synchronize()
    assert torch.equal(state, before)
    ref = torch.einsum("hrj,hj->hr", before.double(), q.double()).float()
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-5)
    gate = torch.full((heads,), -0.5, device="cuda")
    nd.forward_device(state, q, torch.zeros_like(k), v, zero + 0.5, gate)
    torch.cuda.synchronize()
    decay = torch.tensor(-0.5, dtype=torch.float64, device="cuda").exp()
    want = (before.double() * decay).float()
    assert torch.equal(state, want)


# Shapes with enough rows (>= 64 per SM) for the TMA-staged streaming kernel:
# key_dim with and without a tail of four, value_dim that puts one and two
# heads in a tile, and a 1024-wide row (16-row tiles; the others use 32).
STREAM_SHAPES = [(80, 100, 128), (160, 64, 64), (256, 132, 40), (148, 1024, 64)]


@pytest.mark.parametrize("heads,dk,dv", STREAM_SHAPES)
def test_streaming_kernel_bits_match_oracle(oracle, lib, heads, dk, dv):
    """Device-resident state through the host entry point (host decay):
    bit-exact against the oracle on two steps, and the non-finite early stop
    reported at the right row."""
    state = synth.make_delta_state(50 + heads, heads, dk, dv)
    dstate = torch.from_numpy(state.copy()).cuda()
    for step in range(2):
        ins = synth.make_delta_step(50 + heads, step, heads, dk, dv)
        out = np.empty((heads, dv), np.float32)
        rc = lib.moe_delta_heads(dstate.data_ptr(), *(a.ctypes.data for a in ins),
                                 out.ctypes.data, heads, dk, dv)
        rc_o, want = oracle.delta_heads(state, *ins)
        assert rc == rc_o == 0
        np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(dstate.cpu().numpy().view(np.uint32), state.view(np.uint32))
    ins = list(synth.make_delta_step(50 + heads, 9, heads, dk, dv))
    ins[2][heads // 2, dv - 1] = np.nan
    out = np.full((heads, dv), np.nan, np.float32)
    rc = lib.moe_delta_heads(dstate.data_ptr(), *(a.ctypes.data for a in ins), out.ctypes.data,
                             heads, dk, dv)
    assert rc == -2
    stop = (heads // 2) * dv + dv - 1
    assert np.isfinite(out.reshape(-1)[:stop]).all() and np.isnan(out.reshape(-1)[stop:]).all()


@pytest.mark.parametrize("heads,dk,dv", STREAM_SHAPES[:1])
def test_streaming_kernel_device_entry(oracle, heads, dk, dv):
    state = synth.make_delta_state(60, heads, dk, dv)
    ins = synth.make_delta_step(60, 0, heads, dk, dv)
    dstate = torch.from_numpy(state.copy()).cuda()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    got = NativeDelta().forward_device(dstate, *[torch.from_numpy(a).cuda() for a in ins],
                                       status=status).cpu().numpy()
    assert status.tolist() == [-1, 0]
    rc, want = oracle.delta_heads(state, *ins)
    assert rc == 0
    if _device_decay_agrees([ins]):
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        np.testing.assert_array_equal(dstate.cpu().numpy().view(np.uint32), state.view(np.uint32))
    else:
        assert O.max_relative_error(got, want) <= 1e-6
