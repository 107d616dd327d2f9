"""Benchmark: MoE-layer decode on B200.

Workload (N = 1): the one-layer decode configuration -- 256 experts, top-8,
Q3_K gate/up and Q4_K down (1,490,944 B per expert), a Q8_0 shared expert
(3,342,336 B), an fp32 router [256 x 2048] and shared gate vector; one fp32
token per step.  Algorithmic bytes per token = 8 x 1,490,944 + 3,342,336 +
2,097,152 + 8,192 = 17,375,232 B (packed weights actually read + router +
gate vector).  To keep the timing out of L2 (126 MB), steps rotate over
`--copies` resident copies of the layer at distinct HBM addresses (16 copies:
278 MB touched per rotation > 2x L2) and over distinct tokens.

Multi-GPU (torchrun, N > 1): expert parallel.  Each rank holds 256/N
experts of every layer copy plus the router and shared expert; each rank
decodes its own token per step (weak scaling): route locally, all-gather the
tokens and routing, compute the held experts' contributions for every
rank's token, reduce-scatter the partial outputs back to each token's owner.

`--impl reference` times the reference's own CPU implementation of the same
step on the host cores: the reference's AVX2 moe_quant_expert (compiled from
its sources into oracle/_ref) for the 8 routed experts on a thread pool, and
the numpy router / combine / shared expert of its Python layer.

At N = 1 the line also carries "prefill" (config 4: 4096 bf16 tokens on the
tensor cores, TFLOP/s against the measured bf16 peak), "batched_decode"
(config 3: 64 tokens with a Zipf(1.1) router bias), "stack" (config 5:
40 identity-mixer blocks, batch 1 in one launch and batch 32) and "delta"
(the DeltaNet decode step, moe_delta_heads, at the model's 32 x 128 x 128
state, with the reference's own CPU kernel timed beside it).

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "intel-optimized-moe-streaming_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "MoE-layer decode µs/token & quant-weight HBM GB/s (% of 8 TB/s) at 1/2/4/8 GPU"
UNIT = "GB/s"
EXPERT_BYTES = 1_490_944
SHARED_BYTES = 3_342_336
ROUTER_BYTES = 2_097_152
GATE_VEC_BYTES = 8_192


def step_bytes(n_experts_read: int, shared: bool = True) -> int:
    return n_experts_read * EXPERT_BYTES + (SHARED_BYTES if shared else 0) + ROUTER_BYTES + GATE_VEC_BYTES


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------- CPU arms

def cpu_reference_step_fn(lw, threads: int):
    """One token through the layer with the reference's CPU implementation:
    the reference AVX2 kernel per routed expert (oracle/_ref) on a thread
    pool, numpy router/combine/shared expert.  Falls back to the scalar
    oracle port when the reference library was not built."""
    from concurrent.futures import ThreadPoolExecutor
    import oracle as O
    try:
        lib, kind = O.ReferenceLibrary(), "reference"
    except FileNotFoundError:
        lib, kind = O.KQuantOracle(), "port"
    shared = O.shared_weights_from_packed(lib, lw.shared(), lw.shared_kinds, lw.hidden,
                                          lw.shared_inter, lw.shared_gate_inp)
    gate_he = lw.gate_he()
    pool = ThreadPoolExecutor(max_workers=threads)
    experts = [lw.expert(e) for e in range(lw.n_experts)]

    def expert_fn(e, x):
        rc, y = lib.expert(experts[e], lw.kinds, x, lw.hidden, lw.inter, 0)
        if rc:
            raise RuntimeError(f"native expert failed with status {rc}")
        return y

    def step(x):
        ids, w, _ = O.route(x, gate_he, lw.top_k)
        outs = list(pool.map(lambda e: expert_fn(e, x), ids))
        comb = np.zeros(lw.hidden, np.float32)
        for o, wk in zip(outs, w):
            comb += wk * o
        return comb + O.shared_forward(x, shared)
    return step, kind, pool


def time_cpu(lw, tokens, threads, min_seconds=10.0, max_tokens=2000):
    step, kind, pool = cpu_reference_step_fn(lw, threads)
    step(tokens[0])
    n, t0 = 0, time.perf_counter()
    while True:
        step(tokens[n % len(tokens)])
        n += 1
        el = time.perf_counter() - t0
        if (el >= min_seconds and n >= 8) or n >= max_tokens:
            break
    pool.shutdown()
    return el / n, n, kind


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from flash_moe_b200 import synth
    lw = synth.make_layer(seed=0)
    tokens = synth.make_tokens(0, 64, lw.hidden)
    threads = os.cpu_count() or 1
    step, kind, pool = cpu_reference_step_fn(lw, threads)
    for i in range(args.warmup):
        step(tokens[i % 64])
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(tokens[i % 64])
    el = time.perf_counter() - t0
    pool.shutdown()
    per = el / args.steps
    gbs = step_bytes(8) / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 4), "us_per_token": round(per * 1e6, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, config-2 shapes and distributions)",
        "config": {"workload": "config 2: one MoE layer decode, 1 token/step, 256 experts top-8, "
                               "Q3_K/Q3_K/Q4_K experts + Q8_0 shared expert", "tokens_per_step": 1},
        "cpu_baseline": {"value": round(gbs, 4), "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{args.steps} tokens, {cpu_model()}"},
        "e2e": {"value": round(gbs, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- GPU arm

PREFILL_FLOPS_PER_TOKEN = 8 * 3 * 2 * 2048 * 512 + 3 * 2 * 2048 * 512 + 2 * 2048 * 256


def _time_calls(fn, n: int, warmup: int = 3) -> float:
    """Mean device milliseconds of fn() over n calls (CUDA events)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def bench_prefill(backend, layer: int, dev, peaks: dict, peak_kind: str) -> dict:
    """Config 4: 4096 bf16 tokens through the config-2 layer on the tensor
    cores (moe_b200_prefill).  The packed weights (382 MB) exceed L2, so each
    call streams them from HBM."""
    import torch
    from flash_moe_b200 import synth
    T = 4096
    lw = backend.store.layer(layer).weights
    x = torch.from_numpy(synth.make_tokens(404, T, lw.hidden)).to(dev).to(torch.bfloat16)
    y = torch.empty((T, lw.hidden), dtype=torch.float32, device=dev)
    ms = _time_calls(lambda: backend.prefill_device(layer, x, y), 10)
    err = backend.prefill_errors()
    flops = PREFILL_FLOPS_PER_TOKEN * T
    tf = flops / (ms / 1e3) / 1e12
    peak = peaks.get("bf16_tflops", 1590.0)
    return {"config": "config 4: 4096 bf16 tokens, config-2 layer (256 experts top-8, Q3_K/Q4_K + "
                      "Q8_0 shared), fp16 operands on tcgen05 with fp32 accumulation",
            "us_per_layer": round(ms * 1e3, 1), "tokens_per_s": round(T / (ms / 1e3)),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                         "flops_per_layer": flops,
                         "peak_source": f"{peak_kind} bf16_tflops (dense fp16 runs at the same rate)"},
            "kernels_per_call": backend.prefill_kernels(layer, T), "device_error": err}


def bench_batched(dev, peaks: dict, peak_kind: str) -> dict:
    """Config 3: 64 concurrent tokens on the config-2 layer with a Zipf(1.1)
    router bias, one GPU: the fp32 decode engine and the tensor-core path."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    lw = synth.make_layer(seed=0, zipf_s=1.1)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    be = B200ExpertBackend(arena)
    T = 64
    x = torch.from_numpy(synth.make_tokens(3000, T, lw.hidden)).to(dev)
    y = torch.empty_like(x)
    ids = torch.empty((T, lw.top_k), dtype=torch.int32, device=dev)
    ms_dec = _time_calls(lambda: be.forward_layer_device(0, x, y, ids), 20)
    uniq = int(np.unique(ids.cpu().numpy()).size)
    ms_pf = _time_calls(lambda: be.prefill_device(0, x, y, ids), 20)
    err = be.prefill_errors()
    algo = uniq * EXPERT_BYTES + SHARED_BYTES + ROUTER_BYTES + T * 2 * lw.hidden * 4
    best = min(ms_dec, ms_pf)
    gbs = algo / (best / 1e3) / 1e9
    out = {"config": "config 3: 64 tokens/step, Zipf(s=1.1) router bias, 1 GPU",
           "unique_experts": uniq, "algorithmic_bytes_per_step": algo,
           "us_per_step_decode_engine": round(ms_dec * 1e3, 1),
           "us_per_step_tensor_core_path": round(ms_pf * 1e3, 1),
           "tokens_per_s": round(T / (best / 1e3)),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                        "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                        "peak_source": f"{peak_kind} hbm_gbs"},
           "device_error": err}
    be.close()
    return out


def bench_delta(dev, peaks: dict, peak_kind: str, cpu: bool = True) -> dict:
    """The DeltaNet decode step (moe_delta_heads) at the reference model's
    linear-attention shape: 32 value heads of 128 x 128 fp32 state (2 MiB per
    layer).  Calls rotate over 96 layer states (192 MiB > L2), one call per
    layer as a decode step makes them; timed as stream launches, as one CUDA
    graph of 96 calls, and through the host entry point with host arrays
    (the reference's ctypes call, state copied in and out each call).  A
    256-head x 512 x 512 state (256 MiB per call) shows the streaming rate.
    Algorithmic bytes per call: the state read and written, q, k, v, output,
    beta and gate once."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.native_expert import NativeDelta
    nd = NativeDelta()

    def algo(h, dk, dv):
        return 8 * h * dv * dk + 4 * (2 * h * dk + 2 * h * dv + 2 * h)

    heads, dk, dv, layers = 32, 128, 128, 96
    states = torch.from_numpy(synth.make_delta_state(7, heads, dk, dv)).to(dev).repeat(layers, 1, 1, 1)
    ins = [torch.from_numpy(a).to(dev) for a in synth.make_delta_step(7, 0, heads, dk, dv)]
    ins[4].clamp_(min=-0.01)   # decay near 1 keeps the repeated steps' state bounded
    outs = torch.empty((layers, heads, dv), device=dev)
    counter = [0]

    def one():
        i = counter[0] % layers
        counter[0] += 1
        nd.forward_device(states[i], *ins, out=outs[i])
    ms = _time_calls(one, 4 * layers, warmup=layers)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(layers):
                nd.forward_device(states[i], *ins, out=outs[i], stream=s)
    ms_graph = _time_calls(graph.replay, 20) / layers
    del graph
    # host entry: numpy state and inputs, the reference caller's form
    hstate = synth.make_delta_state(7, heads, dk, dv)
    hins = synth.make_delta_step(7, 0, heads, dk, dv)
    for _ in range(5):
        nd.forward(hstate, *hins)
    n_host = 200
    t0 = time.perf_counter()
    for _ in range(n_host):
        nd.forward(hstate, *hins)
    us_host = (time.perf_counter() - t0) / n_host * 1e6
    # a large state streamed from HBM
    H2, D2 = 256, 512
    big = torch.empty((H2, D2, D2), device=dev).normal_(0, 0.1)
    bins = [torch.from_numpy(a).to(dev) for a in synth.make_delta_step(8, 0, H2, D2, D2)]
    bout = torch.empty((H2, D2), device=dev)
    ms_big = _time_calls(lambda: nd.forward_device(big, *bins, out=bout), 10)
    del big
    peak = peaks["hbm_gbs"]
    a_small, a_big = algo(heads, dk, dv), algo(H2, D2, D2)
    gbs = a_small / (ms_graph / 1e3) / 1e9
    gbs_big = a_big / (ms_big / 1e3) / 1e9
    out = {"config": "DeltaNet step, 32 heads x 128 x 128 fp32 state (2 MiB), 96 layer states "
                     "rotated (192 MiB > L2); large: 256 heads x 512 x 512 (256 MiB)",
           "algorithmic_bytes_per_call": a_small,
           "us_per_call_stream": round(ms * 1e3, 2),
           "us_per_call_graph": round(ms_graph * 1e3, 2),
           "us_per_call_host_entry": round(us_host, 1),
           "us_per_call_large": round(ms_big * 1e3, 1),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                        "large_achieved": round(gbs_big, 1),
                        "large_frac": round(gbs_big / peak, 4)}}
    if cpu:
        import oracle as O
        try:
            lib, kind = O.ReferenceLibrary(), "reference"
        except FileNotFoundError:
            lib, kind = O.KQuantOracle(), "port"
        cstate = synth.make_delta_state(7, heads, dk, dv)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 2.0:
            lib.delta_heads(cstate, *hins)
            n += 1
        us_cpu = (time.perf_counter() - t0) / n * 1e6
        out["cpu_baseline"] = {"us_per_call": round(us_cpu, 1), "cores": 1, "kind": kind,
                               "sample": f"{n} calls on one 32 x 128 x 128 state (~2 s), {cpu_model()}"}
    return out


def bench_stack(backend, base_layer: int, dev, peaks: dict, peak_kind: str) -> dict:
    """Config 5: 40 identity-mixer blocks (RMSNorm f16 + residual around each
    MoE layer), 40 distinct resident layers (15.3 GB of packed weights), batch
    1 (one launch of 40 chained block steps) and batch 32 (block kernels
    around the tensor-core path per layer)."""
    import torch
    from flash_moe_b200 import synth
    arena = backend.store
    base = arena.layer(base_layer)
    ids = []
    for l in range(40):
        lid = 1000 + l
        arena.add_device_layer(lid, base.reshuffled(5000 + l) if l else base)
        ids.append(lid)
    H = base.weights.hidden
    x1 = torch.from_numpy(synth.make_tokens(7000, 1, H)).to(dev)
    y1 = torch.empty_like(x1)
    lt = backend.layer_table(ids)
    tmp = torch.empty((2, H), dtype=torch.float32, device=dev)
    rows = [(i, 2 | (1 if i else 0), x1[0] if i == 0 else None,
             y1[0] if i == 39 else tmp[i % 2], None, None) for i in range(40)]
    st = backend.step_table(rows)
    ms1 = _time_calls(lambda: backend.decode_steps_device(lt, st, 40, ids[0]), 10)
    x32 = torch.from_numpy(synth.make_tokens(7001, 32, H)).to(dev)
    y32 = torch.empty_like(x32)
    ms32 = _time_calls(lambda: backend.decode_stack_batch(ids, x32, y32), 3, warmup=1)
    err = backend.device_errors() or backend.prefill_errors()
    per_tok_bytes = 40 * step_bytes(8)
    gbs = per_tok_bytes / (ms1 / 1e3) / 1e9
    for lid in ids:
        arena.drop_layer(lid)
    return {"config": "config 5: 40 blocks (identity mixer + RMSNorm f16 eps 1e-6 + residual), "
                      "40 distinct resident layers (layer 0 seeded, 1..39 seeded row permutations "
                      "with their own routers), 1 GPU",
            "batch1_us_per_token": round(ms1 * 1e3, 1),
            "batch1_us_per_layer": round(ms1 * 1e3 / 40, 2),
            "batch1_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                                "algorithmic_bytes_per_token": per_tok_bytes,
                                "peak_source": f"{peak_kind} hbm_gbs"},
            "batch1_launches": 1,
            "batch32_ms_per_step": round(ms32, 3),
            "batch32_tokens_per_s": round(32 / (ms32 / 1e3)),
            "device_error": err}


def run_prefill_only(args) -> None:
    """The config-4 prefill measurement alone (one GPU), for profiling."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    dev = torch.device("cuda", 0)
    arena = ExpertArena(dev)
    arena.add_layer(0, synth.make_layer(seed=0))
    backend = B200ExpertBackend(arena)
    peaks, peak_kind = measured_peaks()
    print(json.dumps({"prefill": bench_prefill(backend, 0, dev, peaks, peak_kind)}), flush=True)


def check_last_step(runner, steps: int) -> float:
    """Max relative error of the last timed step's output (runner.y) against
    the exact fp32 engine (every weight dequantised bit-exactly, fp32 FMA;
    pinned to the oracle by the tests) on the same token and layer; under
    torchrun the exact engine runs expert-parallel with NCCL collectives
    (all-gather, held experts, reduce-scatter, own shared expert).  Max over
    ranks."""
    import torch
    from flash_moe_b200 import _lib
    from flash_moe_b200 import ep as EP
    i = steps - 1
    layer = runner.layers[i % len(runner.layers)]
    x = runner.tokens[i % runner.tokens.shape[0]].view(1, -1)
    got = runner.y.clone()
    want = torch.empty_like(got)
    be = runner.be
    if runner.world == 1:
        be.forward_layer_device(layer, x, want, flags=_lib.EXACT)
    else:
        H = x.shape[1]
        xa = torch.empty((runner.world, H), dtype=torch.float32, device=x.device)
        yp, yr, ys = torch.empty_like(xa), torch.empty_like(got), torch.empty_like(got)
        EP.ep_exchange_step(
            x, lambda a, p: be.forward_layer_device(layer, a, p, flags=_lib.EXACT | _lib.NO_SHARED),
            lambda a, p: be.forward_layer_device(layer, a, p, flags=_lib.EXACT | _lib.SHARED_ONLY),
            xa, yp, yr, ys, want)
    torch.cuda.synchronize()
    err = ((got - want).abs().max() / want.abs().max().clamp_min(1e-30)).view(1)
    if runner.world > 1:
        import torch.distributed as dist
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
    return float(err.item())


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    from flash_moe_b200 import ep as EP

    lw = synth.make_layer(seed=0)
    E = lw.n_experts
    per = E // world
    begin = rank * per
    arena = ExpertArena(dev)
    first = arena.add_layer(0, lw, expert_begin=begin, expert_count=per)
    # further copies at distinct addresses: clone the device buffers
    for c in range(1, args.copies):
        arena.add_device_layer(c, first.clone())
    backend = B200ExpertBackend(arena, exact=args.engine == "exact")
    H = lw.hidden
    ntok = 64
    tokens = torch.from_numpy(synth.make_tokens(1000 + rank, ntok, H)).to(dev)

    runner = EP.DecodeRunner(backend, list(range(args.copies)), tokens, world, rank)
    stream = torch.cuda.current_stream(dev)

    # warm-up (also compiles nothing; the library is prebuilt)
    for i in range(args.warmup):
        runner.step(i)
    torch.cuda.synchronize()

    graph = None
    tables = None
    if world == 1 and not args.single_launch:
        # all K steps in one launch of the fused kernel (moe_b200_decode_steps)
        tables = runner.step_tables(args.steps)
        runner.run_tables(tables, args.steps)
        torch.cuda.synchronize()
    elif not args.no_graph:
        graph = runner.capture(args.steps)

    def timed_steps():
        if tables is not None:
            runner.run_tables(tables, args.steps)
        elif graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                runner.step(i)

    peaks, peak_kind = measured_peaks()
    with ClockSampler(local) as clk:
        # soak ~0.5 s so the clock sampler sees the GPU under this load; every
        # rank runs the same number of rounds (rank 0's count), since each
        # round holds collectives when world > 1
        n_soak = 0
        if args.soak > 0:
            t0 = time.perf_counter()
            timed_steps()
            torch.cuda.synchronize()
            n_soak = int(args.soak / max(time.perf_counter() - t0, 1e-6))
        if world > 1:
            n_t = torch.tensor([n_soak], device=dev)
            dist.broadcast(n_t, 0)
            n_soak = int(n_t.item())
        for _ in range(n_soak):
            timed_steps()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        timed_steps()
        ev1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = ev0.elapsed_time(ev1)
    ms_t = torch.tensor([ms], device=dev)
    bytes_local = runner.algorithmic_bytes(args.steps)
    bytes_t = torch.tensor([float(bytes_local)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        dist.all_reduce(bytes_t, op=dist.ReduceOp.SUM)
    ms_max = float(ms_t.item())
    total_bytes = float(bytes_t.item())
    per_step_ms = ms_max / args.steps
    gbs = total_bytes / (ms_max / 1e3) / 1e9

    launch_mode = ("one launch of all steps" if tables is not None
                   else "CUDA graph of per-step launches" if graph is not None else "per-step launches")
    # roofline of the decode kernel chain on this rank (one launch sequence
    # per step), from the same timed region
    ach = bytes_local / (ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": EP.profiled_traffic(ROOT),
            "peak_source": f"{peak_kind} hbm_gbs",
            "kernel": ("k_decode_fused (all steps in one launch)" if launch_mode.startswith("one")
                       else runner.kernel_name)}

    max_err = check_last_step(runner, args.steps)

    # end to end through the public API: pinned host token in, host result out
    e2e = runner.e2e(args.steps, args.warmup)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        per_tok, n, kind = time_cpu(lw, synth.make_tokens(1000, 64, H), os.cpu_count() or 1,
                                    min_seconds=args.cpu_seconds)
        cpu = {"value": round(step_bytes(8) / per_tok / 1e9, 4), "unit": UNIT,
               "cores": os.cpu_count() or 1, "kind": kind,
               "sample": f"{n} tokens of the same layer ({per_tok * 1e6:.0f} us/token), {cpu_model()}"}
    launches = 1 if tables is not None else runner.launches_per_step * args.steps
    graph = None
    tables = None
    extra = {}
    if rank == 0 and world == 1 and not args.no_extra:
        extra["prefill"] = bench_prefill(backend, 0, dev, peaks, peak_kind)
        extra["batched_decode"] = bench_batched(dev, peaks, peak_kind)
        extra["stack"] = bench_stack(backend, 0, dev, peaks, peak_kind)
        extra["delta"] = bench_delta(dev, peaks, peak_kind, cpu=not args.no_cpu)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 6),
            "us_per_token": round(per_step_ms * 1e3 / 1, 3),
            "hbm_frac_of_8tbs": round(gbs / (8000.0 * world), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config-2 shapes and distributions)",
            "config": {"workload": "config 2: one MoE layer decode, 1 token/step/GPU, 256 experts "
                                   "top-8, Q3_K/Q3_K/Q4_K experts + Q8_0 shared expert",
                       "tokens_per_step_per_gpu": 1, "layer_copies": args.copies,
                       "l2": f"rotating {args.copies} layer copies at distinct addresses "
                             f"({args.copies * step_bytes(8) / 1e6:.0f} MB touched per rotation > 2x L2)",
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "engine": args.engine, "launch": launch_mode,
                       "algorithmic_bytes_per_token": step_bytes(8)},
            "roofline": roof,
            "e2e": e2e,
            "gpu_launches": launches,
            "max_rel_err": float(f"{max_err:.3e}"),
            "max_rel_err_vs": "exact fp32 engine, last timed step (max over ranks)",
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        line.update(extra)
        print(json.dumps(line), flush=True)
    runner.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--copies", type=int, default=16)
    ap.add_argument("--engine", choices=["fast", "exact"], default="fast")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--single-launch", action="store_true",
                    help="one kernel launch per step (CUDA graph) instead of one for all steps")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--soak", type=float, default=0.5)
    ap.add_argument("--only", choices=["prefill", "delta"], default=None,
                    help="run only the config-4 prefill measurement (for profiling)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the prefill and batched-decode measurements (N = 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.only == "prefill":
        run_prefill_only(args)
    elif args.only == "delta":
        import torch
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        peaks, peak_kind = measured_peaks()
        print(json.dumps({"delta": bench_delta(dev, peaks, peak_kind, cpu=not args.no_cpu)}),
              flush=True)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
