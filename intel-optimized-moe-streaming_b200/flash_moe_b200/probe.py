"""Timing probes of the B200 kernels, read from their trace slots.

    python -m flash_moe_b200.probe decode [--steps 40] [--copies 16]
        phase timeline (us since the step began, median / max over CTAs) of
        the middle step of one multi-step fused decode launch (config 2).
    python -m flash_moe_b200.probe prefill [--tokens 4096]
        per-role wait and busy shares of the three prefill GEMM kernels
        (router, gate/up, down) on the config-2 layer.
    torchrun --nproc-per-node N -m flash_moe_b200.probe ep [--steps 64]
        phase timeline of one expert-parallel step with the exchange over
        peer memory (k_decode_multi), per rank, us since the rank's first
        CTA began the step (median / max over CTAs), and each rank's step
        time in a CUDA graph of `steps` steps.

Both enable the library's trace buffer (``moe_b200_set_trace``) for one
launch; the numbers come from %globaltimer / clock64 stamps the kernels
write when the buffer is set.  Nothing here runs in the product path.
"""
from __future__ import annotations

import argparse
import ctypes as C

import numpy as np
import torch

from . import _lib, synth
from .backend import B200ExpertBackend
from .ep import DecodeRunner
from .store import ExpertArena

DECODE_STAMPS = ["entry", "x_in", "router_rows", "router", "shared_gu", "routing_barrier",
                 "topk", "gu_warps", "gate_up", "gu_barrier", "down_rows", "down", "exit",
                 "tk_sorted", "tk_rounds", "tk_softmax", "chunk0", "chunk1", "row0",
                 "act_loaded", "act_quantised", "down_item0", "down_item16",
                 "x_quantised", "x_synced", "x_codes"]
EP_STAMPS = ["entry", "x_pushed", "x_in", "router", "routing_barrier", "topk_pairs",
             "shared_gu", "gate_up", "gu_barrier", "act_quantised", "down", "combine_pushed",
             "combine_in", "exit"]
PREFILL_ROLES = ["producer_wait_stage", "raw_producer_wait_slot", "dequant_wait_raw",
                 "dequant_wait_stage", "mma_wait_full", "mma_wait_accumulator",
                 "epilogue_wait", "epilogue_busy"]


def _sms(dev) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


def probe_decode(steps: int = 40, copies: int = 16) -> None:
    dev = torch.device("cuda", 0)
    lw = synth.make_layer(seed=0)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    for c in range(1, copies):
        arena.add_device_layer(c, arena.layer(0).clone())
    be = B200ExpertBackend(arena)
    toks = torch.from_numpy(synth.make_tokens(3, 64, lw.hidden)).to(dev)
    runner = DecodeRunner(be, list(range(copies)), toks)
    tabs = runner.step_tables(steps)
    for _ in range(3):
        runner.run_tables(tabs, steps)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    runner.run_tables(tabs, steps)
    e1.record()
    torch.cuda.synchronize()
    print(f"{steps} steps in one launch: {e0.elapsed_time(e1) * 1e3 / steps:.2f} us/step")
    G = _sms(dev)
    buf = torch.zeros(G * 32, dtype=torch.int64, device=dev)
    be.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
    try:
        runner.run_tables(tabs, steps)
        torch.cuda.synchronize()
    finally:
        be.lib.moe_b200_set_trace(None, 0)
    t = buf.view(G, 32).cpu().numpy()[:, :len(DECODE_STAMPS)].astype(np.float64)
    t0 = t[:, 0][t[:, 0] > 0].min()
    t = np.where(t > 0, (t - t0) / 1e3, np.nan)
    print(f"step {steps // 2}: phase stamps, us since the first CTA began the step (median / max)")
    for i, name in enumerate(DECODE_STAMPS):
        col = t[:, i]
        if np.isfinite(col).any():
            print(f"  {name:16s} {np.nanmedian(col):7.2f} {np.nanmax(col):7.2f}")
    print("device error word:", be.device_errors())


def probe_multi(copies: int = 16, rounds: int = 4) -> None:
    """Time per moe_b200_decode call of 1, 2, 4 and 8 tokens on the config-2
    layer: `copies` resident copies at distinct addresses, a CUDA graph of
    rounds x copies calls (one launch each), CUDA events around its replay."""
    dev = torch.device("cuda", 0)
    lw = synth.make_layer(seed=0)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    for c in range(1, copies):
        arena.add_device_layer(c, arena.layer(0).clone())
    be = B200ExpertBackend(arena)
    toks = torch.from_numpy(synth.make_tokens(3, 64, lw.hidden)).to(dev)
    for T in (1, 2, 4, 8):
        xs = [toks[(i * T) % 64:(i * T) % 64 + T].contiguous() for i in range(copies)]
        ys = [torch.empty_like(x) for x in xs]
        for i in range(copies):
            be.forward_layer_device(i, xs[i], ys[i])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(rounds):
                for i in range(copies):
                    be.forward_layer_device(i, xs[i], ys[i])
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        print(f"{T} token(s): {e0.elapsed_time(e1) * 1e3 / (rounds * copies):.1f} us per call")
        del g
    print("device error word:", be.device_errors())


def probe_prefill(tokens: int = 4096) -> None:
    dev = torch.device("cuda", 0)
    arena = ExpertArena(dev)
    arena.add_layer(0, synth.make_layer(seed=0))
    be = B200ExpertBackend(arena)
    x = torch.from_numpy(synth.make_tokens(404, tokens, 2048)).to(dev).to(torch.bfloat16)
    y = torch.empty((tokens, 2048), dtype=torch.float32, device=dev)
    for _ in range(3):
        be.prefill_device(0, x, y)
    torch.cuda.synchronize()
    G = _sms(dev)
    buf = torch.zeros(G * 32, dtype=torch.int64, device=dev)
    be.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
    try:
        be.prefill_device(0, x, y)
        torch.cuda.synchronize()
    finally:
        be.lib.moe_b200_set_trace(None, 0)
    a = buf.view(G, 32).cpu().numpy().astype(np.float64)
    for mode, name in enumerate(["router", "gate/up", "down"]):
        blk = a[:, mode * 10: mode * 10 + 10]
        cyc = blk[:, 8].mean()
        print(f"{name}: {cyc:.0f} cycles per CTA (max {blk[:, 8].max():.0f}), "
              f"{blk[:, 9].mean():.2f} units per CTA")
        for i, role in enumerate(PREFILL_ROLES):
            print(f"  {role:24s} {blk[:, i].mean() / max(cyc, 1) * 100:6.1f}% of cycles")
    print("device error word:", be.prefill_errors())


def probe_batched(tokens: int = 64, calls: int = 10) -> None:
    """Batched decode on the tensor-core path (the config-3 layer: Zipf(1.1)
    router bias): time per call, the routing's expert counts and the
    per-role wait counters of the expert GEMMs."""
    dev = torch.device("cuda", 0)
    lw = synth.make_layer(seed=0, zipf_s=1.1)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    be = B200ExpertBackend(arena)
    x = torch.from_numpy(synth.make_tokens(3000, tokens, lw.hidden)).to(dev)
    y = torch.empty_like(x)
    ids = torch.empty((tokens, lw.top_k), dtype=torch.int32, device=dev)
    for _ in range(3):
        be.prefill_device(0, x, y, ids)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(calls):
        be.prefill_device(0, x, y, ids)
    e1.record()
    torch.cuda.synchronize()
    cnt = np.bincount(ids.cpu().numpy().ravel(), minlength=lw.n_experts)
    print(f"{tokens} tokens: {e0.elapsed_time(e1) * 1e3 / calls:.1f} us per call, "
          f"{int((cnt > 0).sum())} experts selected, most tokens on one expert {int(cnt.max())}")
    G = _sms(dev)
    buf = torch.zeros(G * 32, dtype=torch.int64, device=dev)
    be.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
    try:
        be.prefill_device(0, x, y, ids)
        torch.cuda.synchronize()
    finally:
        be.lib.moe_b200_set_trace(None, 0)
    a = buf.view(G, 32).cpu().numpy().astype(np.float64)
    for mode, name in [(1, "gate/up"), (2, "down")]:
        blk = a[:, mode * 10: mode * 10 + 10]
        cyc = blk[:, 8].mean()
        print(f"{name}: {cyc:.0f} cycles per CTA (max {blk[:, 8].max():.0f}), "
              f"{blk[:, 9].mean():.2f} units per CTA")
        for i, role in enumerate(PREFILL_ROLES):
            print(f"  {role:24s} {blk[:, i].mean() / max(cyc, 1) * 100:6.1f}% of cycles")
    print("device error word:", be.prefill_errors())


def probe_ep(steps: int = 64, copies: int = 16) -> None:
    import os
    from datetime import timedelta
    import torch.distributed as dist
    from .ep import expert_range
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    lw = synth.make_layer(seed=0)
    b, n = expert_range(lw.n_experts, world, rank)
    arena = ExpertArena(dev)
    first = arena.add_layer(0, lw, expert_begin=b, expert_count=n)
    for c in range(1, copies):
        arena.add_device_layer(c, first.clone())
    be = B200ExpertBackend(arena)
    toks = torch.from_numpy(synth.make_tokens(1000 + rank, 64, lw.hidden)).to(dev)
    runner = DecodeRunner(be, list(range(copies)), toks, world, rank)
    g = runner.capture(steps)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    G = _sms(dev)
    buf = torch.zeros(G * 32, dtype=torch.int64, device=dev)
    dist.barrier()
    be.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
    try:
        runner.step(steps + 7)
        torch.cuda.synchronize()
    finally:
        be.lib.moe_b200_set_trace(None, 0)
    bufs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf)
    held = runner.ids[(steps + 7) % runner.max_steps].cpu().numpy()
    if rank == 0:
        t_all = [bb.view(G, 32).cpu().numpy()[:, :len(EP_STAMPS)].astype(np.float64) for bb in bufs]
        g0 = min(t[:, 0][t[:, 0] > 0].min() for t in t_all)
        for r, t in enumerate(t_all):
            t0 = t[:, 0][t[:, 0] > 0].min()
            lo, hi = expert_range(lw.n_experts, world, r)
            nh = len({int(e) for e in held.reshape(-1) if lo <= e < lo + hi})
            print(f"rank {r}: entry {(t0 - g0) / 1e3:+.2f} us (globaltimer, unsynchronised "
                  f"clocks possible), {nh} held experts selected")
            tt = np.where(t > 0, (t - t0) / 1e3, np.nan)
            print("  " + "  ".join(f"{name} {np.nanmedian(tt[:, i]):.2f}/{np.nanmax(tt[:, i]):.2f}"
                                   for i, name in enumerate(EP_STAMPS)
                                   if np.isfinite(tt[:, i]).any()))
    us_t = torch.tensor([us], device=dev)
    all_us = [torch.empty_like(us_t) for _ in range(world)]
    dist.all_gather(all_us, us_t)
    if rank == 0:
        print("us/step in a graph of", steps, "steps, per rank:",
              " ".join(f"{float(v.item()):.2f}" for v in all_us))
    print(f"rank {rank} device error word: {be.device_errors()}", flush=True)
    del g
    runner.close()
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(prog="python -m flash_moe_b200.probe")
    sub = ap.add_subparsers(dest="what", required=True)
    d = sub.add_parser("decode")
    d.add_argument("--steps", type=int, default=40)
    d.add_argument("--copies", type=int, default=16)
    p = sub.add_parser("prefill")
    p.add_argument("--tokens", type=int, default=4096)
    b = sub.add_parser("batched")
    b.add_argument("--tokens", type=int, default=64)
    b.add_argument("--calls", type=int, default=10)
    m = sub.add_parser("multi")
    m.add_argument("--copies", type=int, default=16)
    q = sub.add_parser("ep")
    q.add_argument("--steps", type=int, default=64)
    args = ap.parse_args()
    _lib.load()
    if args.what == "decode":
        probe_decode(args.steps, args.copies)
    elif args.what == "multi":
        probe_multi(args.copies)
    elif args.what == "ep":
        probe_ep(args.steps)
    elif args.what == "batched":
        probe_batched(args.tokens, args.calls)
    else:
        probe_prefill(args.tokens)


if __name__ == "__main__":
    main()
