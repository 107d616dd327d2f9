"""Whole-layer decode on the GPU (moe_b200_decode through the C ABI) against
the oracle restatement of the reference's run_moe_layer.

Routing: the device's top-k ids must equal the oracle's, except where the
k-th and (k+1)-th scores are within 1e-5 relative (a near tie that fp32
summation order can flip); then the oracle is re-run with the device's
selection.  Routing weights within 1e-5 relative.  Outputs:
max|y - ref| / max|ref| <= 1e-3."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import FUSED_SPECS, LAYER_SPECS, layer_case, oracle_layer
from flash_moe_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _arena_backend(lw, **kw):
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    arena = ExpertArena()
    arena.add_layer(0, lw)
    return B200ExpertBackend(arena, **kw)


def check_layer(oracle, lw, xs, y, ids, w, fp16_graph=0, tol=TOL):
    want_y, want_ids, want_w = oracle_layer(oracle, lw, xs, fp16_graph)
    sel = None
    if not np.array_equal(np.asarray(ids), want_ids):
        scores = np.stack([O.route(x, lw.gate_he(), lw.top_k, lw.router_bias)[2] for x in xs])
        for t in range(len(xs)):
            s = np.sort(scores[t])[::-1]
            k = lw.top_k
            assert abs(s[k - 1] - s[k]) <= 1e-5 * max(abs(s[k - 1]), 1e-30), \
                f"token {t}: routing differs without a near tie: {ids[t]} vs {want_ids[t]}"
        sel = [(list(map(int, ids[t])), [float(v) for v in w[t]]) for t in range(len(xs))]
        want_y, _, want_w = oracle_layer(oracle, lw, xs, fp16_graph, selections=sel)
    # fp32 scores summed in another order than the host's BLAS (whose kernel,
    # and so order, depends on the CPU): a weight's relative error is the
    # absolute error of the score differences, a few 1e-6 at scores ~1
    np.testing.assert_allclose(np.asarray(w), want_w, rtol=1e-5, atol=1e-7)
    err = O.max_relative_error(y, want_y)
    assert err <= tol, err
    return err


@pytest.mark.parametrize("name", list(LAYER_SPECS))
@pytest.mark.parametrize("exact", [False, True])
def test_decode_layer_matches_oracle(oracle, name, exact):
    lw, xs = layer_case(name)
    be = _arena_backend(lw, exact=exact)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    check_layer(oracle, lw, xs, y, ids, w)


@pytest.mark.parametrize("name", list(FUSED_SPECS))
def test_fused_decode_every_format(oracle, name):
    """One token at a time through the fused kernel (the fast engine),
    every block format and lane grouping, against the oracle."""
    lw, xs = layer_case(name)
    be = _arena_backend(lw)
    for t in range(len(xs)):
        y, (ids, w) = be.forward_layer(0, xs[t:t + 1], return_routing=True)
        check_layer(oracle, lw, xs[t:t + 1], y, ids, w)
    assert be.device_errors() == 0


@pytest.mark.parametrize("name", list(LAYER_SPECS))
def test_decode_layer_matches_reference_golden(golden, name):
    g = golden(f"layer_{name}")
    lw, xs = layer_case(name)
    be = _arena_backend(lw)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    np.testing.assert_array_equal(ids, g["ids"])
    assert O.max_relative_error(y, g["y"]) <= TOL


def test_decode_layer_fp16_graph_matches_stock_reference(golden):
    """Routed experts with the stock NativeExpert rounding (fp16_graph=1)."""
    g = golden("layer_small")
    lw, xs = layer_case("small")
    be = _arena_backend(lw, fp16_graph=True, exact=True)
    y = be.forward_layer(0, xs)
    assert O.max_relative_error(y, g["y_stock"]) <= 5e-3


@pytest.mark.parametrize("tokens", [1, 7, 64])
def test_decode_batched_tokens(oracle, tokens):
    lw = synth.make_layer(seed=11, hidden=512, inter=256, n_experts=32, top_k=8, shared_inter=256)
    xs = synth.make_tokens(11, tokens, lw.hidden)
    be = _arena_backend(lw)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    check_layer(oracle, lw, xs, y, ids, w)


@pytest.mark.parametrize("name", ["small", "f_q3q4q8"])
def test_decode_run_twice_bit_identical(name):
    lw, xs = layer_case(name)
    be = _arena_backend(lw)
    a = [be.forward_layer(0, xs[t:t + 1]) for t in range(len(xs))]
    b = [be.forward_layer(0, xs[t:t + 1]) for t in range(len(xs))]
    np.testing.assert_array_equal(np.stack(a), np.stack(b))
    assert be.device_errors() == 0


def test_run_moe_layer_drop_in_uses_fused_path(oracle):
    from flash_moe_b200.moe_layer import run_moe_layer, run_moe_sequence
    lw, xs = layer_case("small")
    be = _arena_backend(lw)
    router = type("R", (), {"top_k": lw.top_k})()
    y = np.stack([run_moe_layer(0, x, router, be, lw.hidden, lw.inter) for x in xs])
    ys = run_moe_sequence(0, xs, router, be, lw.hidden, lw.inter)
    want, _, _ = oracle_layer(oracle, lw, xs)
    assert O.max_relative_error(y, want) <= TOL
    assert O.max_relative_error(ys, want) <= TOL


def test_backend_per_expert_forward_matches_oracle(oracle):
    from flash_moe_b200.key import ExpertKey
    lw, xs = layer_case("small")
    be = _arena_backend(lw)
    for e in (0, 5, 15):
        got = be.forward(ExpertKey(0, e), xs[0], lw.hidden, lw.inter)
        _, want = oracle.expert(lw.expert(e), lw.kinds, xs[0], lw.hidden, lw.inter, 0)
        assert O.max_relative_error(got, want) <= TOL
    got = be.forward_batch(ExpertKey(0, 3), xs, lw.hidden, lw.inter)
    for t in range(len(xs)):
        _, want = oracle.expert(lw.expert(3), lw.kinds, xs[t], lw.hidden, lw.inter, 0)
        assert O.max_relative_error(got[t], want) <= TOL
    assert be.forward_batch(ExpertKey(0, 3), xs[:0], lw.hidden, lw.inter).shape == (0, lw.hidden)


@pytest.mark.parametrize("tokens", [1, 4, 24])
def test_decode_host_entry_matches_device_entry(tokens):
    """moe_b200_decode_host (host buffers, one synchronous call) gives the
    same bits as moe_b200_decode on device buffers, for pinned tensors and
    pageable numpy arrays alike, routing included."""
    import ctypes as C
    import torch
    lw, xs = layer_case("small")
    xs = np.ascontiguousarray(np.resize(xs, (tokens, lw.hidden)), np.float32)
    be = _arena_backend(lw)
    dev = be.device
    k = lw.top_k
    xd = torch.from_numpy(xs).to(dev)
    yd = torch.empty_like(xd)
    idd = torch.empty((tokens, k), dtype=torch.int32, device=dev)
    wd = torch.empty((tokens, k), dtype=torch.float32, device=dev)
    be.forward_layer_device(0, xd, yd, idd, wd)
    torch.cuda.synchronize()
    want = (yd.cpu().numpy(), idd.cpu().numpy(), wd.cpu().numpy())
    # pinned tensors
    xp = torch.from_numpy(xs).pin_memory()
    yp = torch.empty((tokens, lw.hidden), dtype=torch.float32).pin_memory()
    ip = torch.empty((tokens, k), dtype=torch.int32).pin_memory()
    wp = torch.empty((tokens, k), dtype=torch.float32).pin_memory()
    for _ in range(2):
        be.forward_layer_host(0, xp, yp, ip, wp)
        assert np.array_equal(yp.numpy().view(np.uint32), want[0].view(np.uint32))
        assert np.array_equal(ip.numpy(), want[1])
        assert np.array_equal(wp.numpy().view(np.uint32), want[2].view(np.uint32))
    # pageable numpy, no routing requested
    y = np.empty_like(xs)
    be.forward_layer_host(0, xs, y)
    assert np.array_equal(y.view(np.uint32), want[0].view(np.uint32))
    # argument errors come back as status codes
    dl = be.store.layer(0)
    ws = be._host_workspace(dl, tokens)
    s = dl.with_flags(0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert be.lib.moe_b200_decode_host(C.byref(s), None, tokens, y.ctypes.data, None, None,
                                       ws.data_ptr(), ws.numel(), stream) == -1
    assert be.lib.moe_b200_decode_host(C.byref(s), xs.ctypes.data, tokens, y.ctypes.data, None,
                                       None, ws.data_ptr(), 256, stream) == -8
