"""Expert-parallel layer step on CPU ranks (gloo, world size 2).

The exchange protocol of flash_moe_b200.ep (all-gather the ranks' tokens,
each rank adds the experts it holds, reduce-scatter the partial outputs back
to each token's owner, the owner adds the shared expert) runs with the
oracle as the per-rank compute, and must equal the single-process oracle
layer.  A rank that leaves before a collective makes the other rank's
collective fail with an error instead of waiting for ever."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
WORLD = 2
TOKENS_PER_RANK = 2


def _layer():
    from flash_moe_b200 import synth
    from flash_moe_b200.formats import Q4_K, Q8_0
    lw = synth.make_layer(seed=41, hidden=512, inter=256, n_experts=8, top_k=3, gate_type=Q4_K,
                          up_type=Q4_K, down_type=Q8_0, shared_inter=256)
    xs = synth.make_tokens(41, WORLD * TOKENS_PER_RANK, lw.hidden)
    return lw, xs


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, port: int, mode: str, q) -> None:
    try:
        sys.path.insert(0, str(ROOT / "intel-optimized-moe-streaming_b200"))
        sys.path.insert(0, str(ROOT / "oracle"))
        sys.path.insert(0, str(ROOT / "tests"))
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        import oracle as O
        from cases import oracle_shared_weights
        from flash_moe_b200.ep import ep_exchange_step, expert_range

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                                timeout=timedelta(seconds=20))
        lib = O.KQuantOracle()
        lw, xs = _layer()
        begin, count = expert_range(lw.n_experts, WORLD, rank)
        shared = oracle_shared_weights(lib, lw)
        gate_he = lw.gate_he()

        def routed(x_all, y_part):
            for i, xv in enumerate(x_all.numpy()):
                ids, w, _ = O.route(xv, gate_he, lw.top_k, lw.router_bias)
                acc = np.zeros(lw.hidden, np.float32)
                for e, wk in zip(ids, w):
                    if begin <= e < begin + count:
                        rc, out = lib.expert(lw.expert(e), lw.kinds, xv, lw.hidden, lw.inter, 0)
                        assert rc == 0
                        acc += wk * out
                y_part[i] = torch.from_numpy(acc)

        def shared_fn(x, y_sh):
            for i, xv in enumerate(x.numpy()):
                y_sh[i] = torch.from_numpy(O.shared_forward(xv, shared))

        t = TOKENS_PER_RANK
        x = torch.from_numpy(xs[rank * t:(rank + 1) * t].copy())
        H = lw.hidden
        x_all = torch.empty((WORLD * t, H))
        y_part = torch.empty((WORLD * t, H))
        y_routed, y_sh, y = (torch.empty((t, H)) for _ in range(3))
        if mode == "leave" and rank == 1:
            q.put((rank, "left"))
            return  # leaves before the first collective
        ep_exchange_step(x, routed, shared_fn, x_all, y_part, y_routed, y_sh, y)
        q.put((rank, y.numpy()))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the test, never swallowed
        q.put((rank, f"error: {type(exc).__name__}: {exc}\n{traceback.format_exc()[-400:]}"))


def _run(mode: str, timeout: float = 120.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, val = q.get(timeout=timeout)
            results[rank] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def test_ep_step_matches_single_process_oracle(oracle):
    from cases import oracle_layer
    res = _run("normal")
    for r in range(WORLD):
        assert not isinstance(res[r], str), res[r]
    lw, xs = _layer()
    want, _, _ = oracle_layer(oracle, lw, xs)
    got = np.concatenate([res[r] for r in range(WORLD)])
    import oracle as O
    assert O.max_relative_error(got, want) <= 1e-6


def test_ep_rank_leaving_fails_the_other_rank_instead_of_hanging():
    res = _run("leave")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error:"), res[0]
