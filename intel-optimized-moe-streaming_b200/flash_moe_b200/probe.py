"""Timing probes of the B200 kernels, read from their trace slots.

    python -m flash_moe_b200.probe decode [--steps 40] [--copies 16]
        phase timeline (us since the step began, median / max over CTAs) of
        the middle step of one multi-step fused decode launch (config 2).
    python -m flash_moe_b200.probe prefill [--tokens 4096]
        per-role wait and busy shares of the three prefill GEMM kernels
        (router, gate/up, down) on the config-2 layer.

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
                 "act_loaded", "act_quantised", "down_item0", "down_item16"]
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


def main() -> None:
    ap = argparse.ArgumentParser(prog="python -m flash_moe_b200.probe")
    sub = ap.add_subparsers(dest="what", required=True)
    d = sub.add_parser("decode")
    d.add_argument("--steps", type=int, default=40)
    d.add_argument("--copies", type=int, default=16)
    p = sub.add_parser("prefill")
    p.add_argument("--tokens", type=int, default=4096)
    args = ap.parse_args()
    _lib.load()
    if args.what == "decode":
        probe_decode(args.steps, args.copies)
    else:
        probe_prefill(args.tokens)


if __name__ == "__main__":
    main()
