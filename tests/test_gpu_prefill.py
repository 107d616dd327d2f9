"""Many-token layer on the tensor cores (moe_b200_prefill through the C ABI)
against the oracle restatement of the reference's run_moe_sequence.

The prefill path feeds the tensor cores fp16 weights (the reference's own
f16 dequantisation) and fp16 activations with fp32 accumulation, so its
outputs are held to the layer tolerance, max|y - ref| / max|ref| <= 1e-3,
against the fp32 oracle.  Routing: the device's top-k ids must equal the
oracle's except at near ties (k-th and (k+1)-th scores within 2e-5
relative: the tensor-core router logits carry ~1e-6 relative error); the
routing weights agree to 1e-5 relative."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O
from cases import layer_case, oracle_layer
from flash_moe_b200 import synth
from flash_moe_b200.formats import Q3_K, Q4_K, Q5_K, Q6_K, Q8_0

pytestmark = pytest.mark.gpu
TOL = 1e-3
TIE = 2e-5

# name -> (synth.make_layer kwargs, tokens)
PREFILL_SPECS = {
    # the configuration formats (Q3_K gate/up, Q4_K down, Q8_0 shared) at H 2048
    "p_q3q4q8": (dict(seed=31, n_experts=32), 96),
    # K-quants of different formats for gate and up, Q8_0 down
    "p_q6q5q8": (dict(seed=32, n_experts=16, top_k=4, gate_type=Q6_K, up_type=Q5_K,
                      down_type=Q8_0, shared_types=(Q4_K, Q4_K, Q5_K)), 80),
    "p_h1024": (dict(seed=33, hidden=1024, inter=256, n_experts=16, top_k=6, gate_type=Q4_K,
                     up_type=Q4_K, down_type=Q8_0, shared_inter=512), 50),
    # router bias with Zipf popularity; an expert with more than 256 pairs
    # (several column tiles); no shared expert
    "p_hot_noshared": (dict(seed=34, n_experts=8, top_k=2, shared_inter=0, zipf_s=1.1), 700),
    "p_bias_q5": (dict(seed=35, hidden=1024, inter=512, n_experts=64, top_k=8, gate_type=Q4_K,
                       up_type=Q4_K, down_type=Q5_K, shared_inter=256,
                       shared_types=(Q8_0, Q8_0, Q4_K), zipf_s=1.1), 64),
}


# Random Q6_K blocks carry int8 scales, four times the magnitude of the
# other formats' six-bit ones; their SwiGLU products outgrow fp16 at x ~ N(0, 1)
# (the call then reports -10), so that case runs at x / 16.
PREFILL_X_SCALE = {"p_q6q5q8": 1.0 / 16}


def _case(name):
    kw, count = PREFILL_SPECS[name]
    lw = synth.make_layer(**kw)
    xs = synth.make_tokens(kw["seed"], count, lw.hidden)
    return lw, xs


def _backend(lw, **kw):
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    arena = ExpertArena()
    arena.add_layer(0, lw)
    return B200ExpertBackend(arena, **kw)


def _prefill(be, xs, dtype=None, flags=None):
    import torch
    dev = be.device
    x = torch.from_numpy(np.ascontiguousarray(xs, np.float32)).to(dev)
    if dtype is not None:
        x = x.to(dtype)
    t, k = x.shape[0], be.store.layer(0).weights.top_k
    y = torch.empty((t, x.shape[1]), dtype=torch.float32, device=dev)
    ids = torch.empty((t, k), dtype=torch.int32, device=dev)
    w = torch.empty((t, k), dtype=torch.float32, device=dev)
    be.prefill_device(0, x, y, ids, w, flags=flags)
    torch.cuda.synchronize(dev)
    assert be.prefill_errors() == 0
    return y.cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()


def check_prefill(oracle, lw, xs, y, ids, w, tol=TOL, tokens=None):
    """Compare rows `tokens` (default all) of a prefill result with the oracle."""
    tokens = np.arange(len(xs)) if tokens is None else np.asarray(tokens)
    xs, y, ids, w = xs[tokens], y[tokens], ids[tokens], w[tokens]
    want_y, want_ids, want_w = oracle_layer(oracle, lw, xs)
    same = np.all(ids == want_ids, axis=1)
    if not same.all():
        for t in np.nonzero(~same)[0]:
            s = np.sort(O.route(xs[t], lw.gate_he(), lw.top_k, lw.router_bias)[2])[::-1]
            k = lw.top_k
            assert abs(s[k - 1] - s[k]) <= TIE * max(abs(s[k - 1]), 1e-30), \
                f"token {t}: routing differs without a near tie: {ids[t]} vs {want_ids[t]}"
        sel = [(list(map(int, ids[t])), [float(v) for v in w[t]]) for t in range(len(xs))]
        want_y, _, _ = oracle_layer(oracle, lw, xs, selections=sel)
    np.testing.assert_allclose(w[same], want_w[same], rtol=1e-5, atol=1e-6)
    err = O.max_relative_error(y, want_y)
    assert err <= tol, err
    return err


@pytest.mark.parametrize("name", list(PREFILL_SPECS))
def test_prefill_matches_oracle(oracle, name):
    lw, xs = _case(name)
    xs = (xs * PREFILL_X_SCALE.get(name, 1.0)).astype(np.float32)
    be = _backend(lw)
    assert be.prefill_supported(0)
    y, ids, w = _prefill(be, xs)
    check_prefill(oracle, lw, xs, y, ids, w)


def test_prefill_bf16_input(oracle):
    """bf16 activations (the prefill configuration's input type): the
    oracle gets the same values widened to fp32."""
    import torch
    lw, xs = _case("p_q3q4q8")
    xb = torch.from_numpy(xs).to(torch.bfloat16)
    xs_exact = xb.to(torch.float32).numpy()
    be = _backend(lw)
    y, ids, w = _prefill(be, xs_exact, dtype=torch.bfloat16)
    check_prefill(oracle, lw, xs_exact, y, ids, w)


def test_prefill_config_size_against_exact_engine_and_oracle(oracle):
    """The prefill configuration: 4096 tokens through the config-2 layer
    (256 experts, top-8).  Every row against the GPU exact engine (fp32
    dequantisation + fma, itself pinned to the oracle), 16 sampled rows
    against the oracle."""
    import torch
    lw = synth.make_layer(seed=2)
    xs = synth.make_tokens(404, 4096, lw.hidden)
    be = _backend(lw)
    y, ids, w = _prefill(be, xs)
    dev = be.device
    xd = torch.from_numpy(xs).to(dev)
    ye = torch.empty_like(xd)
    ide = torch.empty((4096, 8), dtype=torch.int32, device=dev)
    we = torch.empty((4096, 8), dtype=torch.float32, device=dev)
    from flash_moe_b200 import _lib
    be.forward_layer_device(0, xd, ye, ide, we, flags=_lib.EXACT)
    ye, ide = ye.cpu().numpy(), ide.cpu().numpy()
    same = np.all(ids == ide, axis=1)
    assert same.mean() > 0.99
    assert O.max_relative_error(y[same], ye[same]) <= TOL
    rng = np.random.default_rng(7)
    pick = rng.choice(4096, 16, replace=False)
    check_prefill(oracle, lw, xs, y, ids, w, tokens=pick)


def test_prefill_flags_match_decode():
    """NO_SHARED and SHARED_ONLY select the same parts as in decode."""
    import torch
    from flash_moe_b200 import _lib
    lw, xs = _case("p_h1024")
    be = _backend(lw)
    dev = be.device
    xd = torch.from_numpy(xs).to(dev)
    for flags in (_lib.NO_SHARED, 8):
        y, _, _ = _prefill(be, xs, flags=flags)
        ye = torch.empty_like(xd)
        be.forward_layer_device(0, xd, ye, flags=flags | _lib.EXACT)
        assert O.max_relative_error(y, ye.cpu().numpy()) <= TOL


def test_prefill_repeat_is_stable():
    """Two calls: the routed outputs add into y with fp32 reductions whose
    order may differ, so equal to a few ulps, not bit for bit."""
    lw, xs = _case("p_q3q4q8")
    be = _backend(lw)
    a = _prefill(be, xs)
    b = _prefill(be, xs)
    np.testing.assert_array_equal(a[1], b[1])
    np.testing.assert_array_equal(a[2], b[2])
    assert O.max_relative_error(a[0], b[0]) <= 1e-6


def test_prefill_unsupported_layer_returns_status_and_forward_layer_uses_decode(oracle):
    """Q3_K rows of 220 bytes (hidden 512) are outside the tensor-core path:
    moe_b200_prefill answers -2 and forward_layer takes the decode engine."""
    import torch
    from flash_moe_b200 import _lib
    lw, xs = layer_case("small")
    be = _backend(lw, prefill_min_tokens=1)
    assert not be.prefill_supported(0)
    with pytest.raises(RuntimeError, match="status -2"):
        _prefill(be, xs)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    want, _, _ = oracle_layer(oracle, lw, xs)
    assert O.max_relative_error(y, want) <= TOL


def test_forward_layer_uses_prefill_and_falls_back_on_fp16_overflow(oracle):
    """forward_layer runs the prefill kernels from prefill_min_tokens on; a
    token whose SwiGLU activation leaves the fp16 range makes the call
    report -10 and forward_layer recompute with the fp32 engine."""
    lw, xs = _case("p_h1024")
    be = _backend(lw, prefill_min_tokens=16)
    y = be.forward_layer(0, xs)
    want, _, _ = oracle_layer(oracle, lw, xs)
    assert O.max_relative_error(y, want) <= TOL
    big = (xs * 4000.0).astype(np.float32)
    y2 = be.forward_layer(0, big[:20])
    want2, _, _ = oracle_layer(oracle, lw, big[:20])
    assert O.max_relative_error(y2, want2) <= TOL


@pytest.mark.parametrize("tokens", [8, 9, 17, 31])
def test_forward_layer_default_threshold(oracle, tokens):
    """With the default threshold forward_layer keeps the one-launch decode
    kernels up to the token count they take (8 here) and hands every larger
    call to the tensor cores; either way the result meets the oracle."""
    lw = synth.make_layer(seed=36, n_experts=64)
    xs = synth.make_tokens(36 + tokens, tokens, lw.hidden)
    be = _backend(lw)
    one_launch = be.kernels_per_call(0, tokens) == 1
    assert be.uses_tensor_path(0, tokens) == (not one_launch)
    assert one_launch == (tokens <= 8)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    check_prefill(oracle, lw, xs, y, ids, w)


def test_prefill_kernel_count():
    from flash_moe_b200 import _lib
    lw, _ = _case("p_h1024")
    be = _backend(lw)
    s = be.store.layer(0).with_flags(0)
    n = C.c_int(0)
    # prep, router prep, router GEMM, top-k, pairs, gate/up, down; for few
    # tokens the router on the CUDA cores routes the tokens itself
    assert be.lib.moe_b200_prefill_kernels(C.byref(s), 4096, C.byref(n)) == 0
    assert n.value == 7
    assert be.lib.moe_b200_prefill_kernels(C.byref(s), 64, C.byref(n)) == 0
    assert n.value == 5


@pytest.mark.parametrize("tokens", [24, 160])
def test_prefill_more_than_256_experts(oracle, tokens):
    """More than 256 experts: the top-k runs as its own kernel with each
    token's scores staged in shared memory, after the CUDA-core router (few
    tokens) or after the tensor-core router, whose K-chunk partials it adds
    first (many tokens)."""
    lw = synth.make_layer(seed=37, hidden=1024, inter=256, n_experts=320, top_k=8,
                          gate_type=Q4_K, up_type=Q4_K, down_type=Q8_0, shared_inter=256)
    xs = synth.make_tokens(37 + tokens, tokens, lw.hidden)
    be = _backend(lw)
    s = be.store.layer(0).with_flags(0)
    n = C.c_int(0)
    assert be.lib.moe_b200_prefill_kernels(C.byref(s), tokens, C.byref(n)) == 0
    assert n.value == (6 if tokens <= 128 else 7)
    y, ids, w = _prefill(be, xs)
    check_prefill(oracle, lw, xs, y, ids, w)


@pytest.mark.parametrize("name,tokens", [("p_q3q4q8", 40), ("p_bias_q5", 48), ("p_h1024", 17)])
def test_few_tokens_both_expert_gemm_paths(oracle, name, tokens):
    """At most 48 tokens the expert GEMMs run on warp-level MMA (k_bd_gemm);
    MOE_B200_TCGEN05 forces the tcgen05 pipeline.  Both match the oracle, and
    each other to fp32 summation order."""
    from flash_moe_b200 import _lib
    lw, xs = _case(name)
    xs = np.ascontiguousarray(xs[:tokens])
    be = _backend(lw)
    y0, ids0, w0 = _prefill(be, xs)
    y1, ids1, w1 = _prefill(be, xs, flags=be.flags | _lib.TCGEN05)
    assert np.array_equal(ids0, ids1)
    check_prefill(oracle, lw, xs, y0, ids0, w0)
    check_prefill(oracle, lw, xs, y1, ids1, w1)
    assert O.max_relative_error(y0, y1) <= 2e-4


@pytest.mark.parametrize("world", [4, 8])
def test_prefill_expert_parallel_rank_shapes(world):
    """The shapes one expert-parallel rank runs in the multi-GPU benchmark,
    on one GPU: a 1/world expert slice of a 64-expert layer, the tensor-core
    path over 64 gathered tokens without the shared expert, and the shared
    expert alone over the rank's 64/world own tokens; each partial against
    the exact fp32 engine with the same slice and flags."""
    import torch
    from flash_moe_b200 import _lib
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    lw = synth.make_layer(seed=36, n_experts=64, zipf_s=1.1)
    per = lw.n_experts // world
    xs = synth.make_tokens(36, 64, lw.hidden)
    x = torch.from_numpy(xs).cuda()
    for rank in (0, world - 1):
        arena = ExpertArena()
        arena.add_layer(0, lw, expert_begin=rank * per, expert_count=per)
        be = B200ExpertBackend(arena)
        own = x[rank * (64 // world):(rank + 1) * (64 // world)]
        for xin, flags in ((x, _lib.NO_SHARED), (own, _lib.SHARED_ONLY)):
            y = torch.empty_like(xin)
            want = torch.empty_like(xin)
            be.prefill_device(0, xin, y, flags=flags)
            be.forward_layer_device(0, xin, want, flags=_lib.EXACT | flags)
            torch.cuda.synchronize()
            assert be.prefill_errors() == 0
            err = O.max_relative_error(y.cpu().numpy(), want.cpu().numpy())
            assert err <= TOL, (rank, flags, err)
        be.close()
