"""The CPU oracle against the golden fixtures made from the reference.

These pin the checker itself: the oracle must give the bits of
gguf.quants / the reference library / the reference's Python layer on the
seeded inputs the fixtures were generated from (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import DELTA_POISON, DELTA_SPECS, LAYER_SPECS, delta_case, TRIPLES, layer_case, layer_digest, oracle_layer, small_expert_inputs
from flash_moe_b200 import synth

TYPES = [8, 11, 12, 13, 14]


@pytest.mark.parametrize("t", TYPES)
def test_dequant_f32_bits_match_gguf(oracle, golden, t):
    g = golden("dequant_blocks")
    rc, got = oracle.dequant(t, g[f"raw_{t}"])
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint32), g[f"f32_{t}"].view(np.uint32))


@pytest.mark.parametrize("t", TYPES)
def test_dequant_f16_bits_match_reference(oracle, golden, t):
    g = golden("dequant_blocks")
    rc, got = oracle.dequant(t, g[f"raw_{t}"], want_f16=True)
    assert rc == 0
    np.testing.assert_array_equal(got.view(np.uint16), g[f"f16_{t}"])


@pytest.mark.parametrize("t", TYPES)
def test_dequant_rejects_partial_block(oracle, golden, t):
    g = golden("dequant_blocks")
    bs, pb = O.BLOCK[t]
    raw = g[f"raw_{t}"]
    rc, _ = oracle.dequant(t, raw, n=raw.size // pb * bs + 1)
    assert rc == int(g[f"bad_n_status_{t}"]) == -1


def test_dequant_rejects_bad_type_and_sizes(oracle):
    raw = np.zeros(144, np.uint8)
    assert oracle.dequant(999, raw, n=256)[0] == -1
    assert oracle.dequant(12, raw, n=0)[0] == -1
    assert oracle.dequant(12, raw, n=-256)[0] == -1


@pytest.mark.parametrize("i", range(len(TRIPLES)))
@pytest.mark.parametrize("fg", [0, 1])
def test_expert_small_bits_match_reference(oracle, golden, i, fg):
    g = golden("expert_small")
    tensors, x = small_expert_inputs(TRIPLES[i], i)
    assert synth.digest(tensors["gate"], tensors["up"], tensors["down"], x) == str(g[f"digest_{i}"])
    kinds = dict(zip(("gate", "up", "down"), TRIPLES[i]))
    rc, y = oracle.expert(tensors, kinds, x, 256, 256, fg)
    assert rc == int(g[f"rc{fg}_{i}"])
    np.testing.assert_array_equal(y.view(np.uint32), g[f"y{fg}_{i}"].view(np.uint32))


def test_expert_status_codes_match_reference(oracle, golden):
    g = golden("expert_small")
    tensors, x = small_expert_inputs(TRIPLES[0], 0)
    k = dict(zip(("gate", "up", "down"), TRIPLES[0]))
    assert oracle.expert(tensors, dict(k, gate=999), x, 256, 256)[0] == int(g["rc_bad_type"]) == -2
    short = dict(tensors, up=tensors["up"][:-1])
    assert oracle.expert(short, k, x, 256, 256)[0] == int(g["rc_bad_bytes"]) == -3
    assert oracle.expert(tensors, k, x, 256, 256, 2)[0] == int(g["rc_bad_graph"]) == -1
    assert oracle.expert(tensors, k, x, 256, 128)[0] == int(g["rc_bad_cols"])


def test_expert_config1_matches_reference(oracle, golden):
    g = golden("expert_cfg1")
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    assert synth.digest(tensors["gate"], tensors["up"], tensors["down"], x) == str(g["digest"])
    for fg in (0, 1):
        rc, y = oracle.expert(tensors, kinds, x, 2048, 512, fg)
        assert rc == int(g[f"rc{fg}"])
        if rc == 0:
            np.testing.assert_array_equal(y.view(np.uint32), g[f"y{fg}"].view(np.uint32))


@pytest.mark.parametrize("name", list(LAYER_SPECS))
def test_layer_matches_reference_python(oracle, golden, name):
    g = golden(f"layer_{name}")
    lw, xs = layer_case(name)
    assert layer_digest(lw, xs) == str(g["digest"])
    y, ids, w = oracle_layer(oracle, lw, xs)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_allclose(w, g["w"], rtol=0, atol=0)
    assert O.max_relative_error(y, g["y"]) <= 1e-6


def test_layer_stock_fp16_graph_matches_reference(oracle, golden):
    g = golden("layer_small")
    lw, xs = layer_case("small")
    y, _, _ = oracle_layer(oracle, lw, xs, fp16_graph=1)
    assert O.max_relative_error(y, g["y_stock"]) <= 1e-6


@pytest.mark.parametrize("count", [8, 20])
def test_sequence_matches_reference_python(oracle, golden, count):
    """run_moe_sequence: per-token shared expert below 16 tokens, batched
    shared expert for 16..128 (reference moe_layer.py:177-194)."""
    from cases import oracle_shared_weights
    g = golden("layer_small")
    lw, _ = layer_case("small")
    seq = synth.make_tokens(LAYER_SPECS["small"][0]["seed"], count, lw.hidden, stream=1 + count)
    assert synth.digest(seq) == str(g[f"seq{count}_digest"])
    shared = oracle_shared_weights(oracle, lw)

    def expert_fn(e, x):
        return oracle.expert(lw.expert(e), lw.kinds, x, lw.hidden, lw.inter, 0)[1]
    y, _ = O.run_moe_sequence(seq, lw.gate_he(), lw.top_k, expert_fn, shared)
    assert O.max_relative_error(y, g[f"seq{count}"]) <= 1e-6


def test_rmsnorm_matches_reference(golden):
    g = golden("layer_small")
    got = O.rmsnorm_f16(g["norm_in"])
    np.testing.assert_array_equal(got.view(np.uint16), g["norm_out"])


def test_oracle_matches_reference_library_when_built(oracle):
    """Extra pin when the reference library was compiled here: random
    blocks and experts, bit for bit."""
    if not O.REF_LIB.exists():
        pytest.skip("reference library not built (make -C oracle ref)")
    ref = O.ReferenceLibrary()
    rng = np.random.default_rng(99)
    for t in TYPES:
        raw = synth.quant_blocks(rng, t, 40)
        for f16 in (False, True):
            a, b = oracle.dequant(t, raw, want_f16=f16), ref.dequant(t, raw, want_f16=f16)
            assert a[0] == b[0] == 0
            np.testing.assert_array_equal(a[1].view(np.uint8), b[1].view(np.uint8))
    tensors, kinds, x = synth.make_expert_q4k(seed=3, hidden=512, inter=256)
    for fg in (0, 1):
        a, b = oracle.expert(tensors, kinds, x, 512, 256, fg), ref.expert(tensors, kinds, x, 512, 256, fg)
        assert a[0] == b[0]
        np.testing.assert_array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


@pytest.mark.parametrize("name", list(DELTA_SPECS))
def test_delta_step_bits_match_reference(oracle, golden, name):
    """``kq_delta_heads`` reproduces ``moe_delta_heads`` step after step:
    outputs (NaN where the call wrote nothing), statuses and the final state,
    bit for bit."""
    g = golden("delta")
    state, steps = delta_case(name)
    assert synth.digest(state, *[a for st in steps for a in st]) == str(g[f"{name}_digest"])
    ys, rcs = [], []
    for q, k, v, beta, gate in steps:
        rc, y = oracle.delta_heads(state, q, k, v, beta, gate)
        ys.append(y)
        rcs.append(rc)
    assert rcs == g[f"{name}_rc"].tolist()
    np.testing.assert_array_equal(np.stack(ys).view(np.uint32), g[f"{name}_y"].view(np.uint32))
    assert synth.digest(state) == str(g[f"{name}_state_sha"])
    if f"{name}_state" in g:
        np.testing.assert_array_equal(state.view(np.uint32), g[f"{name}_state"].view(np.uint32))


def test_delta_poison_stops_at_the_failing_row(golden):
    """The reference's early stop: rows after the poisoned one keep their
    input state and get no output."""
    g = golden("delta")
    before, _ = delta_case("poison")
    after = g["poison_state"]
    h, r = DELTA_POISON
    y = g["poison_y"][0]
    assert int(g["poison_rc"][0]) == -2
    assert np.isfinite(y.reshape(-1)[:h * y.shape[1] + r]).all()
    assert np.isnan(y.reshape(-1)[h * y.shape[1] + r:]).all()
    flat_b = before.reshape(-1, before.shape[-1])
    flat_a = after.reshape(-1, after.shape[-1])
    stop = h * before.shape[1] + r
    np.testing.assert_array_equal(flat_a[stop + 1:], flat_b[stop + 1:])
    assert not np.array_equal(flat_a[:stop + 1], flat_b[:stop + 1])


def test_delta_status_codes_match_reference(oracle, golden):
    g = golden("delta")
    state, steps = delta_case("many_heads")
    q, k, v, beta, gate = steps[0]
    bad = {"heads0": (0, 8, 8), "heads257": (257, 8, 8), "dk0": (1, 0, 8),
           "dk1025": (1, 1025, 8), "dv0": (1, 8, 0), "dv1025": (1, 8, 1025)}
    for key, (h, dk, dv) in bad.items():
        rc = oracle._delta(state.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data,
                           beta.ctypes.data, gate.ctypes.data, v.ctypes.data, h, dk, dv)
        assert rc == int(g[f"rc_{key}"]) == -1, key
    rc = oracle._delta(None, q.ctypes.data, k.ctypes.data, v.ctypes.data, beta.ctypes.data,
                       gate.ctypes.data, v.ctypes.data, 1, 8, 8)
    assert rc == int(g["rc_null"]) == -1
