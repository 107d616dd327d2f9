"""Fused decode of 2..8 tokens in one launch (k_decode_multi, through
moe_b200_decode and moe_b200_decode_ep) against the oracle restatement of
the reference's run_moe_layer, and the expert-parallel partial outputs of
emulated ranks summed into the layer output."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import FUSED_SPECS, layer_case
from flash_moe_b200 import synth
from test_gpu_layer import TOL, _arena_backend, check_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(FUSED_SPECS))
@pytest.mark.parametrize("tokens", [2, 5, 8])
def test_multi_token_decode_every_format(oracle, name, tokens):
    lw, _ = layer_case(name)
    xs = synth.make_tokens(300 + tokens, tokens, lw.hidden)
    be = _arena_backend(lw)
    assert be.kernels_per_call(0, tokens) == 1
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    check_layer(oracle, lw, xs, y, ids, w)
    assert be.device_errors() == 0


def test_multi_token_config2_ring_refills(oracle):
    """Eight tokens of the config-2 layer: ~64 (token, expert) pairs, more
    routed rows per CTA than the shared-memory ring holds at once (gate/up
    and down slots are refilled)."""
    lw = synth.make_layer(seed=0)
    xs = synth.make_tokens(310, 8, lw.hidden)
    be = _arena_backend(lw)
    y, (ids, w) = be.forward_layer(0, xs, return_routing=True)
    check_layer(oracle, lw, xs, y, ids, w)
    assert be.device_errors() == 0


def test_multi_token_run_twice_bit_identical():
    lw, _ = layer_case("f_q3q4q8")
    xs = synth.make_tokens(311, 8, lw.hidden)
    be = _arena_backend(lw)
    a = be.forward_layer(0, xs)
    b = be.forward_layer(0, xs)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("tokens", [1, 3])
def test_shared_only_plus_routed_only_equals_layer(tokens):
    """SHARED_ONLY and NO_SHARED calls of the fused kernel add up to the
    full layer bit for bit (same routing, same partial sums)."""
    import torch
    from flash_moe_b200 import _lib
    lw, _ = layer_case("f_h1024")
    be = _arena_backend(lw)
    xs = torch.from_numpy(synth.make_tokens(312, tokens, lw.hidden)).to(be.device)
    full, routed, shared = (torch.empty_like(xs) for _ in range(3))
    be.forward_layer_device(0, xs, full)
    be.forward_layer_device(0, xs, routed, flags=be.flags | _lib.NO_SHARED)
    be.forward_layer_device(0, xs, shared, flags=be.flags | _lib.SHARED_ONLY)
    torch.cuda.synchronize()
    assert be.kernels_per_call(0, tokens, be.flags | _lib.SHARED_ONLY) == 1
    assert torch.equal(routed + shared, full)
    assert be.device_errors() == 0


def _ep_partials(lw, xs, world, seed_layer=0):
    """Emulated expert-parallel ranks in one process: rank r holds experts
    [r*E/world, (r+1)*E/world) (its own arena layer) and owns token r."""
    import torch
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.ep import expert_range
    from flash_moe_b200.store import ExpertArena
    arena = ExpertArena()
    for r in range(world):
        b, n = expert_range(lw.n_experts, world, r)
        arena.add_layer(r, lw, expert_begin=b, expert_count=n)
    be = B200ExpertBackend(arena)
    x = torch.from_numpy(xs).to(be.device)
    T, K = xs.shape[0], lw.top_k
    parts, ids, ws = [], [], []
    for r in range(world):
        assert be.ep_fused_supported(r, T)
        y = torch.empty_like(x)
        i = torch.empty((T, K), dtype=torch.int32, device=be.device)
        w = torch.empty((T, K), dtype=torch.float32, device=be.device)
        be.decode_ep_device(r, x, y, r, 1, topk_ids=i, topk_weights=w)
        parts.append(y)
        ids.append(i)
        ws.append(w)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    return ([p.cpu().numpy() for p in parts], [i.cpu().numpy() for i in ids],
            [w.cpu().numpy() for w in ws])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_ep_partials_sum_to_layer(oracle, world):
    lw, _ = layer_case("f_q3q4q8")
    xs = synth.make_tokens(320 + world, world, lw.hidden)
    parts, ids, ws = _ep_partials(lw, xs, world)
    for r in range(1, world):  # the replicated router routes identically on every rank
        np.testing.assert_array_equal(ids[r], ids[0])
        np.testing.assert_array_equal(ws[r], ws[0])
    y = np.sum(np.stack(parts), axis=0)
    check_layer(oracle, lw, xs, y, ids[0], ws[0])


def test_decode_ep_rank_without_selected_experts():
    """A rank none of whose experts any token selects returns zeros for the
    other ranks' tokens and only the gated shared expert for its own."""
    lw = synth.make_layer(seed=33, hidden=1024, inter=256, n_experts=16, top_k=2,
                          gate_type=12, up_type=12, down_type=8, shared_inter=512)
    world = 8
    xs = synth.make_tokens(330, 2, lw.hidden)
    # 8 tokens, six of them copies of the first: at most 4 distinct experts
    xs8 = np.concatenate([xs, np.repeat(xs[:1], world - 2, axis=0)])
    parts, ids, _ = _ep_partials(lw, xs8, world)
    sel = set(np.unique(ids[0]).tolist())
    idle = [r for r in range(world) if not sel & {2 * r, 2 * r + 1}]
    assert idle, sel
    for r in idle:
        others = np.delete(parts[r], r, axis=0)
        assert np.all(others == 0.0)
        assert np.any(parts[r][r] != 0.0)
