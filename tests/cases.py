"""Seeded test cases shared by the golden generator and the tests.

Every case is regenerated from seeds; the golden fixtures store a digest of
the generated inputs so that a drift of the generator is caught.
"""
from __future__ import annotations

import numpy as np

from flash_moe_b200 import synth
from flash_moe_b200.formats import BLOCK, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0

import oracle as O

# type triples of the reference's native test
# (tools/test_optimized_inference.py:237-238)
TRIPLES = [(8, 11, 12), (11, 12, 13), (12, 13, 14), (13, 14, 8), (14, 8, 11),
           (12, 12, 14), (12, 12, 8), (11, 11, 11)]

# name -> (synth.make_layer kwargs, token count)
LAYER_SPECS = {
    "small": (dict(seed=5, hidden=512, inter=256, n_experts=16, top_k=4, shared_inter=256), 4),
    "small_q4": (dict(seed=6, hidden=512, inter=256, n_experts=12, top_k=3, gate_type=Q4_K,
                      up_type=Q4_K, down_type=Q8_0, shared_inter=256,
                      shared_types=(Q6_K, Q6_K, Q6_K)), 3),
    "cfg2": (dict(seed=2), 2),
}

# Layers whose every tensor the fused single-token kernel takes (rows a
# multiple of 16 bytes, 256..2048 columns): every block format, each lane
# grouping (H = 2048, 1024, 512 -> 32, 16, 8 lanes per row), a router bias.
FUSED_SPECS = {
    "f_q3q4q8": (dict(seed=21, n_experts=32), 3),
    "f_q6q5q8": (dict(seed=22, n_experts=16, top_k=4, gate_type=Q6_K, up_type=Q5_K,
                      down_type=Q8_0, shared_types=(Q4_K, Q4_K, Q5_K)), 3),
    "f_h1024": (dict(seed=23, hidden=1024, inter=256, n_experts=16, top_k=6, gate_type=Q4_K,
                     up_type=Q4_K, down_type=Q8_0, shared_inter=512), 3),
    "f_h512_bias": (dict(seed=24, hidden=512, inter=512, n_experts=64, top_k=8, gate_type=Q4_K,
                         up_type=Q8_0, down_type=Q5_K, shared_inter=256,
                         shared_types=(Q8_0, Q4_K, Q8_0), zipf_s=1.1), 3),
    "f_noshared": (dict(seed=25, n_experts=8, top_k=2, shared_inter=0), 2),
}


def small_expert_inputs(kinds, seed_stream: int):
    """The value pattern of the reference's native test
    (``tools/test_optimized_inference.py:239-252``): random bytes with
    d = 0.002 (and dmin = 0.001), a 256x256 expert, x ~ N(0,1)*0.005."""
    rng = np.random.default_rng(np.random.SeedSequence([17, seed_stream]))
    tensors = {}
    for name, kind in zip(("gate", "up", "down"), kinds):
        bs, size = BLOCK[kind]
        raw = rng.integers(0, 256, (256 * (256 // bs), size), np.uint8)
        offset = size - 2 if kind in (11, 14) else 0
        raw[:, offset:offset + 2] = np.frombuffer(np.float16(.002).tobytes(), np.uint8)
        if kind in (12, 13):
            raw[:, 2:4] = np.frombuffer(np.float16(.001).tobytes(), np.uint8)
        tensors[name] = raw.reshape(-1)
    x = (rng.standard_normal(256) * .005).astype(np.float32)
    return tensors, x


def layer_case(name: str):
    kw, count = LAYER_SPECS[name] if name in LAYER_SPECS else FUSED_SPECS[name]
    lw = synth.make_layer(**kw)
    xs = synth.make_tokens(kw["seed"], count, lw.hidden)
    return lw, xs


def layer_digest(lw, xs) -> str:
    extra = [lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_inp] if lw.shared_inter else []
    return synth.digest(lw.gate, lw.up, lw.down, lw.router, *extra, xs)


def oracle_shared_weights(lib, lw):
    """fp32 shared-expert weights as the reference loads them (binary16
    rounding, ``shared_expert.py:157-195``), or None."""
    if not lw.shared_inter:
        return None
    return O.shared_weights_from_packed(lib, lw.shared(), lw.shared_kinds, lw.hidden,
                                        lw.shared_inter, lw.shared_gate_inp)


def oracle_layer(lib, lw, xs, fp16_graph: int = 0, selections=None):
    """The oracle's layer output per token: (y [T,H], ids, weights)."""
    shared = oracle_shared_weights(lib, lw)
    gate_he = lw.gate_he()

    def expert_fn(e, x):
        rc, y = lib.expert(lw.expert(e), lw.kinds, x, lw.hidden, lw.inter, fp16_graph)
        if rc:
            raise RuntimeError(f"native expert failed with status {rc}")
        return y

    ys, ids, ws = [], [], []
    for i, x in enumerate(xs):
        sel = selections[i] if selections is not None else None
        y, e, w = O.run_moe_layer(x, gate_he, lw.top_k, expert_fn, shared, workers=1,
                                  selection=sel, bias=lw.router_bias)
        ys.append(y)
        ids.append(e)
        ws.append(w)
    return np.stack(ys), np.array(ids), np.array(ws)


def check_block(oracle, lw, x, y_dev, ids_dev, w_dev, tol: float = 1e-3, tie: float = 2e-5):
    """One identity-mixer block (h = x + rmsnorm16(x); y = h +
    f16(MoE(rmsnorm16(h)))) against the oracle, fed with the device's own
    input x; a near tie resolved differently by the device is re-routed with
    the device's selection.  Returns the max relative error."""
    h = x + O.rmsnorm_f16(x).astype(np.float32)
    n2 = O.rmsnorm_f16(h).astype(np.float32)
    want_moe, want_ids, _ = oracle_layer(oracle, lw, n2[None])
    if not np.array_equal(ids_dev, want_ids[0]):
        s = np.sort(O.route(n2, lw.gate_he(), lw.top_k, lw.router_bias)[2])[::-1]
        k = lw.top_k
        assert abs(s[k - 1] - s[k]) <= tie * max(abs(s[k - 1]), 1e-30), (ids_dev, want_ids[0])
        sel = [(list(map(int, ids_dev)), [float(v) for v in w_dev])]
        want_moe, _, _ = oracle_layer(oracle, lw, n2[None], selections=sel)
    want = h + want_moe[0].astype(np.float16).astype(np.float32)
    err = O.max_relative_error(y_dev, want)
    assert err <= tol, err
    return err


# DeltaNet step cases: name -> (seed, heads, key_dim, value_dim, steps).
# "model" is the reference model's linear-attention shape (32 value heads of
# 128 x 128); the others cover the lane tail (key_dim % 8, up to 7), key_dim
# < 8, each register-blocking width of the GPU kernel (key_dim / 8 up to 1,
# 2, 4, 8, 16, 32, 64, 128), the size limits of each argument, and a
# poisoned value that stops the step.
DELTA_SPECS = {
    "model": (31, 32, 128, 128, 3),
    "odd": (32, 3, 100, 37, 3),
    "dk7": (33, 5, 7, 9, 2),
    "one": (34, 1, 1, 1, 2),
    "wide": (35, 1, 1024, 64, 1),
    "dk64": (39, 4, 64, 48, 2),
    "dk512": (41, 2, 512, 24, 2),
    "dk263": (40, 2, 263, 40, 2),
    "tall": (36, 2, 16, 1024, 1),
    "many_heads": (37, 256, 8, 8, 2),
    "poison": (38, 3, 24, 10, 1),
}
# (head, row) of the poisoned case whose value is +inf
DELTA_POISON = (1, 4)


def delta_case(name: str):
    """(state, [(q, k, v, beta, gate) per step]) of a DeltaNet case."""
    seed, heads, dk, dv, steps = DELTA_SPECS[name]
    state = synth.make_delta_state(seed, heads, dk, dv)
    inputs = [synth.make_delta_step(seed, s, heads, dk, dv) for s in range(steps)]
    if name == "poison":
        inputs[0][2][DELTA_POISON] = np.inf
    return state, inputs
