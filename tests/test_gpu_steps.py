"""Many decode steps in one launch (moe_b200_decode_steps through the C ABI).

Independent steps must give exactly the outputs of one moe_b200_decode call
per step (same kernel arithmetic).  Chained transformer-block steps (the
40-layer stack configuration: h = x + rmsnorm16(x), y = h +
f16(MoE(rmsnorm16(h)))) are checked layer by layer against the oracle's
stack_block, fed with the device's own input to that layer."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import check_block, oracle_layer
from flash_moe_b200 import synth
from flash_moe_b200.formats import Q4_K, Q8_0

pytestmark = pytest.mark.gpu
TOL = 1e-3

SPEC = dict(hidden=1024, inter=256, n_experts=16, top_k=6, gate_type=Q4_K, up_type=Q4_K,
            down_type=Q8_0, shared_inter=512)


def _arena(n_layers, seed0=70, **extra):
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    arena = ExpertArena()
    lws = []
    for l in range(n_layers):
        lw = synth.make_layer(seed=seed0 + l, **dict(SPEC, **extra))
        arena.add_layer(l, lw)
        lws.append(lw)
    return B200ExpertBackend(arena), lws


def test_independent_steps_equal_single_calls():
    import torch
    from flash_moe_b200 import _lib
    be, lws = _arena(3)
    H, K = lws[0].hidden, lws[0].top_k
    n = 7
    xs = torch.from_numpy(synth.make_tokens(71, n, H)).to(be.device)
    ys = torch.empty((n, H), dtype=torch.float32, device=be.device)
    ids = torch.empty((n, K), dtype=torch.int32, device=be.device)
    ws = torch.empty((n, K), dtype=torch.float32, device=be.device)
    rows = [(i % 3, 0, xs[i], ys[i], ids[i], ws[i]) for i in range(n)]
    be.decode_steps_device(be.layer_table([0, 1, 2]), be.step_table(rows), n, 0)
    torch.cuda.synchronize()
    for i in range(n):
        y1 = torch.empty((1, H), dtype=torch.float32, device=be.device)
        i1 = torch.empty((1, K), dtype=torch.int32, device=be.device)
        be.forward_layer_device(i % 3, xs[i:i + 1], y1, i1)
        torch.cuda.synchronize()
        assert torch.equal(ids[i], i1[0]), i
        assert torch.equal(ys[i], y1[0]), i
    assert be.device_errors() == 0


@pytest.mark.parametrize("n_layers", [1, 4])
def test_block_chain_matches_oracle_layer_by_layer(oracle, n_layers):
    import torch
    from flash_moe_b200 import _lib
    be, lws = _arena(n_layers)
    H, K = lws[0].hidden, lws[0].top_k
    x0 = torch.from_numpy(synth.make_tokens(72, 1, H)).to(be.device)
    ys = torch.empty((n_layers, H), dtype=torch.float32, device=be.device)
    ids = torch.empty((n_layers, K), dtype=torch.int32, device=be.device)
    ws = torch.empty((n_layers, K), dtype=torch.float32, device=be.device)
    rows = []
    for l in range(n_layers):
        fl = _lib.STEP_BLOCK | (_lib.STEP_CHAIN if l else 0)
        rows.append((l, fl, x0[0] if l == 0 else None, ys[l], ids[l], ws[l]))
    be.decode_steps_device(be.layer_table(list(range(n_layers))), be.step_table(rows), n_layers, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    yh, ih, wh = ys.cpu().numpy(), ids.cpu().numpy(), ws.cpu().numpy()
    x = x0[0].cpu().numpy()
    for l in range(n_layers):
        check_block(oracle, lws[l], x, yh[l], ih[l], wh[l])
        x = yh[l]


def test_decode_stack_api_matches_step_tables():
    """backend.decode_stack (ping-pong buffers) equals the same chain with
    one output buffer per layer."""
    import torch
    from flash_moe_b200 import _lib
    be, lws = _arena(3, seed0=90)
    H = lws[0].hidden
    x0 = torch.from_numpy(synth.make_tokens(73, 1, H)).to(be.device)
    y = torch.empty((1, H), dtype=torch.float32, device=be.device)
    be.decode_stack([0, 1, 2], x0, y)
    ys = torch.empty((3, H), dtype=torch.float32, device=be.device)
    rows = [(l, _lib.STEP_BLOCK | (_lib.STEP_CHAIN if l else 0), x0[0] if l == 0 else None, ys[l],
             None, None) for l in range(3)]
    be.decode_steps_device(be.layer_table([0, 1, 2]), be.step_table(rows), 3, 0)
    torch.cuda.synchronize()
    assert torch.equal(y[0], ys[2])
    assert be.device_errors() == 0


def test_block_kernels_match_oracle_norms():
    """moe_b200_block_prepare / finish against the oracle's RMSNorm (fp32
    reduction orders differ: at most one binary16 ulp, on few values)."""
    import torch
    from flash_moe_b200 import _lib
    lib = _lib.load()
    T, H = 9, 1024
    xs = synth.make_tokens(74, T, H) * 3.0
    x = torch.from_numpy(xs).cuda()
    h, n = torch.empty_like(x), torch.empty_like(x)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.moe_b200_block_prepare(x.data_ptr(), h.data_ptr(), n.data_ptr(), T, H, 1e-6, s) == 0
    m = torch.from_numpy(synth.make_tokens(75, T, H)).cuda()
    y = torch.empty_like(x)
    assert lib.moe_b200_block_finish(h.data_ptr(), m.data_ptr(), y.data_ptr(), T, H, s) == 0
    torch.cuda.synchronize()
    want_h = xs + O.rmsnorm_f16(xs).astype(np.float32)
    want_n = O.rmsnorm_f16(want_h).astype(np.float32)
    for got, want in ((h.cpu().numpy(), want_h), (n.cpu().numpy(), want_n)):
        diff = np.abs(got - want)
        ulp = np.abs(want) * 2.0 ** -10 + 2.0 ** -24
        assert np.all(diff <= ulp)
        assert np.mean(diff > 0) < 0.01
    want_y = h.cpu().numpy() + m.cpu().numpy().astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(y.cpu().numpy(), want_y)


def test_stack_batch_layer_by_layer_matches_oracle(oracle):
    """Block kernels around the tensor-core path for 24 tokens, two layers;
    each layer against the oracle block fed with the device's input."""
    import torch
    from flash_moe_b200 import _lib
    be, lws = _arena(2, seed0=95)
    assert be.prefill_supported(0)
    T, H, K = 24, lws[0].hidden, lws[0].top_k
    x = torch.from_numpy(synth.make_tokens(76, T, H)).to(be.device)
    s = torch.cuda.current_stream().cuda_stream
    cur = x
    for l in range(2):
        h, n, m, y = (torch.empty_like(x) for _ in range(4))
        ids = torch.empty((T, K), dtype=torch.int32, device=be.device)
        w = torch.empty((T, K), dtype=torch.float32, device=be.device)
        assert be.lib.moe_b200_block_prepare(cur.data_ptr(), h.data_ptr(), n.data_ptr(), T, H,
                                             1e-6, s) == 0
        be.prefill_device(l, n, m, ids, w)
        assert be.lib.moe_b200_block_finish(h.data_ptr(), m.data_ptr(), y.data_ptr(), T, H, s) == 0
        torch.cuda.synchronize()
        assert be.prefill_errors() == 0
        xh, yh = cur.cpu().numpy(), y.cpu().numpy()
        ih, wh = ids.cpu().numpy(), w.cpu().numpy()
        for t in range(0, T, 5):
            check_block(oracle, lws[l], xh[t], yh[t], ih[t], wh[t])
        cur = y
    # decode_stack_batch runs the same kernels; the prefill combine adds the
    # routed outputs with fp32 reductions in no fixed order, and that
    # last-bit noise can move a binary16-rounded norm value of the next
    # layer by one ulp (5e-4): equal to the layer tolerance
    yb = torch.empty_like(x)
    be.decode_stack_batch([0, 1], x, yb)
    torch.cuda.synchronize()
    assert O.max_relative_error(yb.cpu().numpy(), cur.cpu().numpy()) <= TOL
