"""The one-layer decode configuration itself (256 experts, top-8, Q3_K
gate/up, Q4_K down, Q8_0 shared expert) through the fused single-token
kernel, against the oracle restatement of the reference's run_moe_layer
(src/flash_moe/moe_layer.py:39-107).

This is the layer and the entry point the benchmark times.  With 256
experts, at least as many as the GPU has SMs, the kernel orders its phases
by the tagged exchange words alone, so these tests cover that ordering: one
call per token, many independent steps in one launch rotating over four
distinct layers (the step-parity buffers are reused every other step), and
a chain of transformer blocks, every step's output, routing ids and weights
checked.  Tolerance: max|y - ref| / max|ref| <= 1e-3; ids equal except at
a near tie (k-th and (k+1)-th scores within 1e-5 relative), where the
oracle is re-run with the device's selection; routing weights within 1e-5
relative."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from cases import check_block, oracle_layer
from flash_moe_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-3
SEEDS = (2, 3, 4, 5)


@pytest.fixture(scope="module")
def cfg2():
    """Four distinct config-2 layers resident on the device (1.5 GB)."""
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    arena = ExpertArena()
    lws = []
    for i, seed in enumerate(SEEDS):
        lw = synth.make_layer(seed=seed)
        arena.add_layer(i, lw)
        lws.append(lw)
    be = B200ExpertBackend(arena)
    yield be, lws
    be.close()


def _check_token(oracle, lw, x, y, ids, w):
    """One token's layer output against the oracle (near ties re-routed)."""
    want_y, want_ids, want_w = oracle_layer(oracle, lw, x[None])
    if not np.array_equal(ids, want_ids[0]):
        s = np.sort(O.route(x, lw.gate_he(), lw.top_k, lw.router_bias)[2])[::-1]
        k = lw.top_k
        assert abs(s[k - 1] - s[k]) <= 1e-5 * max(abs(s[k - 1]), 1e-30), (ids, want_ids[0])
        sel = [(list(map(int, ids)), [float(v) for v in w])]
        want_y, _, want_w = oracle_layer(oracle, lw, x[None], selections=sel)
    # the scores are fp32 dots in another summation order than numpy's BLAS;
    # a routing weight's relative error is the absolute error of the score
    # differences, a few 1e-6 at this layer's score magnitudes (~1)
    np.testing.assert_allclose(w, want_w[0], rtol=1e-5, atol=1e-7)
    err = O.max_relative_error(y, want_y[0])
    assert err <= TOL, err
    return err


def test_cfg2_takes_the_fused_kernel(cfg2):
    be, lws = cfg2
    import torch
    assert lws[0].n_experts >= torch.cuda.get_device_properties(0).multi_processor_count
    assert be.kernels_per_call(0, 1) == 1


def test_cfg2_one_call_per_token(oracle, cfg2):
    """Eight tokens, one moe_b200_decode call each, on the same workspace."""
    import torch
    be, lws = cfg2
    lw = lws[0]
    xs = synth.make_tokens(200, 8, lw.hidden)
    for t in range(len(xs)):
        xd = torch.from_numpy(xs[t:t + 1]).to(be.device)
        y = torch.empty_like(xd)
        ids = torch.empty((1, lw.top_k), dtype=torch.int32, device=be.device)
        w = torch.empty((1, lw.top_k), dtype=torch.float32, device=be.device)
        be.forward_layer_device(0, xd, y, ids, w)
        torch.cuda.synchronize()
        _check_token(oracle, lw, xs[t], y[0].cpu().numpy(), ids[0].cpu().numpy(),
                     w[0].cpu().numpy())
    assert be.device_errors() == 0


def test_cfg2_host_buffers(oracle, cfg2):
    """The synchronous host-buffer entry (moe_b200_decode_host), the call the
    reference's ctypes-style caller makes."""
    be, lws = cfg2
    lw = lws[1]
    xs = synth.make_tokens(201, 3, lw.hidden)
    for t in range(len(xs)):
        y, (ids, w) = be.forward_layer(1, xs[t:t + 1], return_routing=True)
        _check_token(oracle, lw, xs[t], y[0], ids[0], w[0])


@pytest.mark.parametrize("n_steps", [12])
def test_cfg2_independent_steps_in_one_launch(oracle, cfg2, n_steps):
    """Twelve independent steps over the four layers in one launch
    (moe_b200_decode_steps): every step against the oracle, and bit-equal to
    a single call of the same token."""
    import torch
    be, lws = cfg2
    H, K = lws[0].hidden, lws[0].top_k
    xs = synth.make_tokens(202, n_steps, H)
    xd = torch.from_numpy(xs).to(be.device)
    ys = torch.empty((n_steps, H), dtype=torch.float32, device=be.device)
    ids = torch.empty((n_steps, K), dtype=torch.int32, device=be.device)
    ws = torch.empty((n_steps, K), dtype=torch.float32, device=be.device)
    rows = [(i % 4, 0, xd[i], ys[i], ids[i], ws[i]) for i in range(n_steps)]
    be.decode_steps_device(be.layer_table([0, 1, 2, 3]), be.step_table(rows), n_steps, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    yh, ih, wh = ys.cpu().numpy(), ids.cpu().numpy(), ws.cpu().numpy()
    for i in range(n_steps):
        _check_token(oracle, lws[i % 4], xs[i], yh[i], ih[i], wh[i])
    for i in (0, n_steps - 1):
        y1 = torch.empty((1, H), dtype=torch.float32, device=be.device)
        i1 = torch.empty((1, K), dtype=torch.int32, device=be.device)
        be.forward_layer_device(i % 4, xd[i:i + 1], y1, i1)
        torch.cuda.synchronize()
        assert torch.equal(ids[i], i1[0]) and torch.equal(ys[i], y1[0]), i


def test_cfg2_block_chain(oracle, cfg2):
    """Eight chained identity-mixer blocks (the 40-layer configuration's
    step) over the four layers in one launch, each block against the oracle
    fed with the device's input to that block."""
    import torch
    from flash_moe_b200 import _lib
    be, lws = cfg2
    n = 8
    H, K = lws[0].hidden, lws[0].top_k
    x0 = torch.from_numpy(synth.make_tokens(203, 1, H)).to(be.device)
    ys = torch.empty((n, H), dtype=torch.float32, device=be.device)
    ids = torch.empty((n, K), dtype=torch.int32, device=be.device)
    ws = torch.empty((n, K), dtype=torch.float32, device=be.device)
    rows = []
    for i in range(n):
        fl = _lib.STEP_BLOCK | (_lib.STEP_CHAIN if i else 0)
        rows.append((i % 4, fl, x0[0] if i == 0 else None, ys[i], ids[i], ws[i]))
    be.decode_steps_device(be.layer_table([0, 1, 2, 3]), be.step_table(rows), n, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    yh, ih, wh = ys.cpu().numpy(), ids.cpu().numpy(), ws.cpu().numpy()
    x = x0[0].cpu().numpy()
    for i in range(n):
        check_block(oracle, lws[i % 4], x, yh[i], ih[i], wh[i])
        x = yh[i]


@pytest.mark.parametrize("extra", [1, 12])
def test_expert_count_just_above_the_sm_count(oracle, extra):
    """E = SMs + 1 and SMs + 12 (every CTA owns at least one router row, some
    two): independent and chained steps in one launch, every step against
    the oracle."""
    import torch
    from flash_moe_b200 import _lib
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    E = sms + extra
    lws = [synth.make_layer(seed=60 + extra + i, n_experts=E, inter=256) for i in range(2)]
    arena = ExpertArena()
    for i, lw in enumerate(lws):
        arena.add_layer(i, lw)
    be = B200ExpertBackend(arena)
    assert be.kernels_per_call(0, 1) == 1
    H, K, n = lws[0].hidden, lws[0].top_k, 6
    xs = synth.make_tokens(210 + extra, n, H)
    xd = torch.from_numpy(xs).to(be.device)
    ys = torch.empty((n, H), dtype=torch.float32, device=be.device)
    ids = torch.empty((n, K), dtype=torch.int32, device=be.device)
    ws = torch.empty((n, K), dtype=torch.float32, device=be.device)
    rows = [(i % 2, 0, xd[i], ys[i], ids[i], ws[i]) for i in range(n)]
    be.decode_steps_device(be.layer_table([0, 1]), be.step_table(rows), n, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    yh, ih, wh = ys.cpu().numpy(), ids.cpu().numpy(), ws.cpu().numpy()
    for i in range(n):
        _check_token(oracle, lws[i % 2], xs[i], yh[i], ih[i], wh[i])
    rows = [(i % 2, _lib.STEP_BLOCK | (_lib.STEP_CHAIN if i else 0), xd[0] if i == 0 else None,
             ys[i], ids[i], ws[i]) for i in range(n)]
    be.decode_steps_device(be.layer_table([0, 1]), be.step_table(rows), n, 0)
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    yh, ih, wh = ys.cpu().numpy(), ids.cpu().numpy(), ws.cpu().numpy()
    x = xs[0]
    for i in range(n):
        check_block(oracle, lws[i % 2], x, yh[i], ih[i], wh[i])
        x = yh[i]
    be.close()
