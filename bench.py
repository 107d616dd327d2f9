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

# BLAS thread policy of the reference's entry point (chat.py:50-56): one
# BLAS thread per process unless FLASH_MOE_BLAS_THREADS says otherwise, set
# before NumPy loads, so the CPU arms run the same way with and without
# torchrun (which sets OMP_NUM_THREADS=1)
_BLAS_THREADS = os.environ.get("FLASH_MOE_BLAS_THREADS", "1")
for _v in ("OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS", "BLIS_NUM_THREADS"):
    os.environ[_v] = _BLAS_THREADS

import numpy as np  # noqa: E402

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
#
# The reference's CPU implementation of the path, timed on this host: its own
# AVX2 kernels (cpp/moe_quant_dot.cpp, dequant_k.cpp, compiled from its
# sources into oracle/_ref; the scalar oracle port if that build is absent)
# driven by the numpy restatement of its Python layer (router, combine,
# shared expert, run_moe_sequence: oracle/oracle.py, pinned bit for bit to the
# reference's own Python by tests/golden).  The reference's Python itself
# cannot travel to the GPU box.

REF_WORKERS = 4  # the reference's expert pool (src/flash_moe/backend_ov.py:107,160)


def _cpu_lib():
    import oracle as O
    try:
        return O.ReferenceLibrary(), "reference"
    except FileNotFoundError:
        return O.KQuantOracle(), "port"


class CpuLayer:
    """One MoE layer run on the host the way the reference's decode runs it:
    route, the top-k native experts on a pool of `workers` threads
    (moe_quant_expert, fp16_graph=0), the fp32 combine in top-k order, the
    shared expert with binary16-rounded weights (numpy, BLAS threads as set
    above)."""

    def __init__(self, lw):
        import oracle as O
        self.O, self.lw = O, lw
        self.lib, self.kind = _cpu_lib()
        self.shared = (O.shared_weights_from_packed(self.lib, lw.shared(), lw.shared_kinds, lw.hidden,
                                                    lw.shared_inter, lw.shared_gate_inp)
                       if lw.shared_inter else None)
        self.gate_he = lw.gate_he()
        self.experts = [lw.expert(e) for e in range(lw.n_experts)]

    def expert(self, e, x):
        rc, y = self.lib.expert(self.experts[e], self.lw.kinds, x, self.lw.hidden, self.lw.inter, 0)
        if rc:
            raise RuntimeError(f"native expert failed with status {rc}")
        return y

    def token(self, x, pool):
        ids, w, _ = self.O.route(x, self.gate_he, self.lw.top_k, self.lw.router_bias)
        outs = list(pool.map(lambda e: self.expert(e, x), ids))
        comb = np.zeros(self.lw.hidden, np.float32)
        for o, wk in zip(outs, w):
            comb += wk * o
        return comb + self.O.shared_forward(x, self.shared) if self.shared is not None else comb

    def experts_f32(self, e):
        """(gate, up, down) fp32 of expert e through the reference's dequant_k."""
        lw = self.lw
        t = self.experts[e]
        out = []
        for name, rows, cols in (("gate", lw.inter, lw.hidden), ("up", lw.inter, lw.hidden),
                                 ("down", lw.hidden, lw.inter)):
            rc, w = self.lib.dequant(lw.kinds[name], t[name], rows * cols)
            assert rc == 0
            out.append(w.reshape(rows, cols))
        return out


def time_tokens(fn, tokens, min_seconds: float, max_tokens: int = 4000):
    """Mean seconds per call of fn(token) over at least `min_seconds`."""
    fn(tokens[0])
    n, t0 = 0, time.perf_counter()
    while True:
        fn(tokens[n % len(tokens)])
        n += 1
        el = time.perf_counter() - t0
        if (el >= min_seconds and n >= 4) or n >= max_tokens:
            return el / n, n


def cpu_layer_baseline(lw, tokens, seconds: float) -> dict:
    """Config 2 on the host: us per token with the reference's 4 expert
    workers and with one worker per host thread; `value` is the faster."""
    from concurrent.futures import ThreadPoolExecutor
    cl = CpuLayer(lw)
    threads = os.cpu_count() or 1
    res = {}
    for workers in sorted({REF_WORKERS, threads}):
        with ThreadPoolExecutor(max_workers=workers) as pool:
            per, n = time_tokens(lambda x: cl.token(x, pool), tokens, seconds / 2)
        res[workers] = (per, n)
    best = min(res, key=lambda k: res[k][0])
    per, n = res[best]
    return {"value": round(step_bytes(8) / per / 1e9, 4), "unit": UNIT, "cores": best,
            "kind": cl.kind, "us_per_token": round(per * 1e6, 1),
            "us_per_token_by_workers": {str(k): round(v[0] * 1e6, 1) for k, v in res.items()},
            "blas_threads": int(_BLAS_THREADS),
            "sample": f"{n} tokens of the config-2 layer with {best} expert workers "
                      f"(reference default {REF_WORKERS}); {cpu_model()}, {threads} host threads"}


def cpu_expert_baseline(seconds: float) -> dict:
    """Config 1 on the host: one Q4_K expert per call, single thread, the
    reference's moe_quant_expert (fp16_graph=0, the parity mode; the stock
    product passes 1, timed beside it)."""
    from flash_moe_b200 import synth
    lib, kind = _cpu_lib()
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    out = {}
    for fg in (0, 1):
        def call(xv):
            lib.expert(tensors, kinds, xv, 2048, 512, fg)
        per, n = time_tokens(call, [x], seconds / 2)
        out[fg] = (per, n)
    per, n = out[0]
    return {"us_per_call": round(per * 1e6, 1), "us_per_call_fp16_graph": round(out[1][0] * 1e6, 1),
            "gbs": round(1_769_472 / per / 1e9, 4), "cores": 1, "kind": kind,
            "sample": f"{n} calls, one thread, {cpu_model()}"}


def cpu_sequence_baseline(lw, xs, sample_experts: int | None = None) -> dict:
    """Many tokens through one layer on the host: the reference's
    run_moe_sequence (src/flash_moe/moe_layer.py:110-195) with forward_batch =
    the reference's dequant_k to fp32 + NumPy BLAS matmuls on all host cores
    (its OpenVINO prefill graph is not available here), the shared expert
    batched.  With `sample_experts`, only that many of the touched experts
    run and the expert time is scaled to all of them."""
    from threadpoolctl import threadpool_limits
    cl = CpuLayer(lw)
    O = cl.O
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ids = []
    for x in xs:
        ids.append(O.route(x, cl.gate_he, lw.top_k, lw.router_bias)[0])
    ids = np.array(ids)
    t_route = time.perf_counter() - t0
    uniq = np.unique(ids)
    run = uniq if sample_experts is None else uniq[:sample_experts]
    with threadpool_limits(limits=threads, user_api="blas"):
        t0 = time.perf_counter()
        for e in run:
            rows = np.nonzero((ids == e).any(axis=1))[0]
            g, u, d = cl.experts_f32(int(e))
            xe = xs[rows]
            gx, ux = xe @ g.T, xe @ u.T
            _ = ((gx * O.sigmoid(gx)) * ux) @ d.T
        t_exp = (time.perf_counter() - t0) * len(uniq) / max(len(run), 1)
        t0 = time.perf_counter()
        if cl.shared is not None:
            _ = O.shared_forward_batch(xs, cl.shared)
        t_sh = time.perf_counter() - t0
    total = t_route + t_exp + t_sh
    return {"s_per_step": round(total, 4), "tokens_per_s": round(len(xs) / total, 1),
            "cores": threads, "kind": cl.kind, "unique_experts": int(len(uniq)),
            "sample": f"{len(xs)} tokens; {len(run)} of {len(uniq)} touched experts run and "
                      f"scaled; forward_batch = reference dequant_k f32 + NumPy BLAS "
                      f"({threads} threads); {cpu_model()}"}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_stack_baseline(lw, H: int) -> dict:
    """Config 5 on the host: batch 1 through 40 identity-mixer blocks (RMSNorm
    f16 + residual around each layer, the reference's decode per layer; the
    same layer's weights for every block: the CPU time does not depend on
    which), 3 tokens; batch 32 through one block with run_moe_sequence's
    forward_batch path (dequant_k f32 + BLAS), times 40."""
    from concurrent.futures import ThreadPoolExecutor
    from flash_moe_b200 import synth
    cl = CpuLayer(lw)
    O = cl.O
    threads = os.cpu_count() or 1
    xs = synth.make_tokens(7000, 3, H)
    with ThreadPoolExecutor(max_workers=threads) as pool:
        t0 = time.perf_counter()
        for x in xs:
            for _ in range(40):
                h = x + O.rmsnorm_f16(x).astype(np.float32)
                m = cl.token(O.rmsnorm_f16(h).astype(np.float32), pool)
                x = h + m.astype(np.float16).astype(np.float32)
        per1 = (time.perf_counter() - t0) / len(xs)
    b32 = cpu_sequence_baseline(lw, synth.make_tokens(7001, 32, H))
    return {"batch1_ms_per_token": round(per1 * 1e3, 2),
            "batch1_gbs": round(40 * step_bytes(8) / per1 / 1e9, 4),
            "batch32_ms_per_step": round(40 * b32["s_per_step"] * 1e3, 1), "cores": threads,
            "kind": cl.kind,
            "sample": f"batch 1: {len(xs)} tokens x 40 blocks, {threads} expert workers; batch 32: "
                      f"one block's run_moe_sequence x 40 ({b32['sample']})"}


def run_reference_arm(args) -> None:
    """The reference's CPU implementation of config 2 on the host cores
    (rank 0 only under torchrun): `--steps` tokens after `--warmup`, with the
    reference's 4 expert workers and with one per host thread; the line
    reports the faster, both per-token times beside it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor
    from flash_moe_b200 import synth
    lw = synth.make_layer(seed=0)
    tokens = synth.make_tokens(0, 64, lw.hidden)
    cl = CpuLayer(lw)
    threads = os.cpu_count() or 1
    res = {}
    for workers in sorted({REF_WORKERS, threads}):
        with ThreadPoolExecutor(max_workers=workers) as pool:
            for i in range(args.warmup):
                cl.token(tokens[i % 64], pool)
            t0 = time.perf_counter()
            for i in range(args.steps):
                cl.token(tokens[i % 64], pool)
            res[workers] = (time.perf_counter() - t0) / args.steps
    best = min(res, key=res.get)
    per = res[best]
    gbs = step_bytes(8) / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 4), "us_per_token": round(per * 1e6, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (reference AVX2 kernels, fp16_graph=0; numpy layer)",
        "data": "synthetic (seeded, config-2 shapes and distributions)",
        "config": {"workload": "config 2: one MoE layer decode, 1 token/step, 256 experts top-8, "
                               "Q3_K/Q3_K/Q4_K experts + Q8_0 shared expert", "tokens_per_step": 1},
        "cpu_baseline": {"value": round(gbs, 4), "unit": UNIT, "cores": best, "kind": cl.kind,
                         "us_per_token_by_workers": {str(k): round(v * 1e6, 1) for k, v in res.items()},
                         "blas_threads": int(_BLAS_THREADS),
                         "sample": f"{args.steps} tokens, {best} expert workers (reference default "
                                   f"{REF_WORKERS}), {cpu_model()}, {threads} host threads"},
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


def bench_expert(dev, peaks: dict, peak_kind: str, cpu_seconds: float | None) -> dict:
    """Config 1: one Q4_K SwiGLU expert (hidden 2048, intermediate 512) for
    one token through moe_quant_expert, the reference's C entry point: with
    host buffers (the reference's unchanged ctypes caller: the 1,769,472
    packed bytes cross PCIe every call) and with device buffers (weights
    resident; calls rotate over 160 expert copies, 283 MB > 2x L2).  Each
    call is synchronous, timed by the host clock over many calls."""
    import torch
    from flash_moe_b200 import _lib, synth
    lib = _lib.load()
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    out = np.empty(2048, np.float32)
    hbufs = {k: np.ascontiguousarray(v) for k, v in tensors.items()}

    def host_call():
        st = lib.moe_quant_expert(kinds["gate"], hbufs["gate"].ctypes.data, hbufs["gate"].size,
                                  kinds["up"], hbufs["up"].ctypes.data, hbufs["up"].size,
                                  kinds["down"], hbufs["down"].ctypes.data, hbufs["down"].size,
                                  x.ctypes.data, 2048, 512, out.ctypes.data, 0)
        assert st == 0, st
    copies = 160
    dev_t = {k: torch.from_numpy(v).to(dev).repeat(copies, 1) for k, v in
             ((k, v.reshape(1, -1)) for k, v in hbufs.items())}
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty(2048, dtype=torch.float32, device=dev)
    ctr = [0]

    def dev_call():
        i = ctr[0] % copies
        ctr[0] += 1
        g, u, d = dev_t["gate"][i], dev_t["up"][i], dev_t["down"][i]
        st = lib.moe_quant_expert(kinds["gate"], g.data_ptr(), g.numel(), kinds["up"], u.data_ptr(),
                                  u.numel(), kinds["down"], d.data_ptr(), d.numel(), xd.data_ptr(),
                                  2048, 512, yd.data_ptr(), 0)
        assert st == 0, st

    res = {}
    for name, fn, n in (("host_buffers", host_call, 400), ("device_buffers", dev_call, 2000)):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        res[name] = (time.perf_counter() - t0) / n
    peak = peaks["hbm_gbs"]
    gbs = 1_769_472 / res["device_buffers"] / 1e9
    obj = {"config": "config 1: one Q4_K expert (2048 x 512), 1 token per call, moe_quant_expert "
                     "(fp16_graph=0), synchronous",
           "us_per_call_host_buffers": round(res["host_buffers"] * 1e6, 1),
           "us_per_call_device_buffers": round(res["device_buffers"] * 1e6, 1),
           "reference_published_ms": "0.607-0.750 (README.md:98-99, the reference's CPU kernel)",
           "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                        "note": "device buffers; a synchronous call per expert is launch-bound"}}
    if cpu_seconds:
        obj["cpu_baseline"] = cpu_expert_baseline(cpu_seconds)
    del dev_t
    return obj


def bench_fp16_graph(backend, layer: int, dev) -> dict:
    """The reference product's stock mode, fp16_graph=1 (binary16 rounding of
    x, the weights, the gate/up products and the SwiGLU activation,
    cpp/moe_quant_dot.cpp:36,160,192-209; src/flash_moe/native_expert.py:33-34):
    the fused engines compute in fp32 activations, so a layer call with
    FP16_GRAPH runs the exact route-plus-expert engine.  Its cost at 1 and 64
    tokens on the config-2 layer, beside the fused engines' fp32-mode time."""
    import torch
    from flash_moe_b200 import _lib, synth
    lw = backend.store.layer(layer).weights
    out = {}
    for T in (1, 64):
        x = torch.from_numpy(synth.make_tokens(5100, T, lw.hidden)).to(dev)
        y = torch.empty_like(x)
        ms16 = _time_calls(lambda: backend.forward_layer_device(
            layer, x, y, flags=backend.flags | _lib.FP16_GRAPH), 10)
        ms32 = _time_calls(lambda: backend.forward_layer_device(layer, x, y), 10)
        out[f"tokens_{T}"] = {"us_fp16_graph_exact_engine": round(ms16 * 1e3, 1),
                              "us_default_call": round(ms32 * 1e3, 1),
                              "kernels_default": backend.kernels_per_call(layer, T),
                              "kernels_fp16_graph": backend.kernels_per_call(
                                  layer, T, backend.flags | _lib.FP16_GRAPH)}
    out["config"] = ("config-2 layer, moe_b200_decode with MOE_B200_FP16_GRAPH (the exact engine) "
                     "against the default call (1 token: the fused kernel, 1 launch; 64 tokens: "
                     "the fp32 exact engine), one call per step")
    return out


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


def with_cpu(obj: dict, fn, enabled: bool) -> dict:
    if enabled:
        obj["cpu_baseline"] = fn()
    return obj


def bench_batched(dev, peaks: dict, peak_kind: str, lw=None) -> dict:
    """Config 3: 64 concurrent tokens on the config-2 layer with a Zipf(1.1)
    router bias, one GPU: the fp32 decode engine and the tensor-core path."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    lw = lw if lw is not None else synth.make_layer(seed=0, zipf_s=1.1)
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


# ------------------------------------------------------- multi-GPU objects

def _time_ranks(fn, n: int, warmup: int = 3) -> float:
    """Device milliseconds per fn() call, CUDA events on each rank after a
    barrier, the maximum over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / n], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _rel_err_ranks(got, want) -> float:
    import torch
    import torch.distributed as dist
    e = ((got - want).abs().max() / want.abs().max().clamp_min(1e-30)).view(1)
    dist.all_reduce(e, op=dist.ReduceOp.MAX)
    return float(e.item())


def bench_allreduce(backend, layers, dev, world: int, rank: int, steps: int, peaks: dict,
                    peak_kind: str) -> dict:
    """The batch-1 alternative to the all-to-all: the token is replicated on
    every rank; each rank decodes it through the experts it holds (the fused
    single-token kernel over its expert range, the shared expert on rank 0
    only) and one 8 KB all-reduce sums the partial outputs.  `steps` steps
    over the resident layer copies in one CUDA graph (the fused launch and the
    NCCL all-reduce per step); device time max over ranks."""
    import torch
    import torch.distributed as dist
    from flash_moe_b200 import _lib, synth
    lw = backend.store.layer(layers[0]).weights
    H = lw.hidden
    xs = torch.from_numpy(synth.make_tokens(2000, 64, H)).to(dev)  # same tokens on every rank
    ys = torch.empty((steps, H), dtype=torch.float32, device=dev)
    ids = torch.full((steps, lw.top_k), -1, dtype=torch.int32, device=dev)
    flags = backend.flags | (_lib.NO_SHARED if rank else 0)

    def step(i):
        backend.forward_layer_device(layers[i % len(layers)], xs[i % 64].view(1, -1), ys[i:i + 1],
                                     topk_ids=ids[i:i + 1], flags=flags)
        dist.all_reduce(ys[i])
    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    g, mode = None, "CUDA graph of the steps"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                step(i)
        run = g.replay
    except RuntimeError:  # capture refused: the same steps as stream launches
        g, mode = None, "stream launches"
        torch.cuda.synchronize()
        dist.barrier()

        def run():
            for i in range(steps):
                step(i)
    ms = _time_ranks(run, 3, warmup=2) / steps
    # the last step against the exact fp32 engine, decomposed the same way
    i = steps - 1
    want = torch.empty((1, H), dtype=torch.float32, device=dev)
    backend.forward_layer_device(layers[i % len(layers)], xs[i % 64].view(1, -1), want,
                                 flags=_lib.EXACT | (_lib.NO_SHARED if rank else 0))
    dist.all_reduce(want)
    err = _rel_err_ranks(ys[i:i + 1], want)
    del g
    uniq = [len(np.unique(r)) for r in ids.cpu().numpy()]
    byts = sum(uniq) * lw.expert_bytes + steps * (lw.shared_bytes + lw.router.nbytes + H * 4)
    gbs = byts / steps / (ms / 1e3) / 1e9
    return {"config": f"config 2, batch 1 replicated on {world} GPUs: each rank its {lw.n_experts // world} "
                      "experts of the top-8 (fused single-token kernel), rank 0 the shared expert, "
                      f"one NCCL all-reduce of 8 KB per layer; {mode}",
            "us_per_token": round(ms * 1e3, 2), "gbs_union": round(gbs, 1),
            "frac_of_one_gpu_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "peak_source": f"{peak_kind} hbm_gbs", "max_rel_err": float(f"{err:.3e}")}


def bench_stack_ep(backend, base_layer: int, dev, world: int, rank: int, peaks: dict,
                   peak_kind: str) -> dict:
    """Config 5 sharded over the ranks: 40 distinct identity-mixer blocks,
    each rank holding 256/N experts of every layer.  Batch 1: the token
    replicated on every rank; per block the RMSNorm kernels, the fused
    single-token kernel over the rank's experts (the shared expert on rank 0)
    and one 8 KB NCCL all-reduce; the 40 blocks in one CUDA graph.  Batch 32:
    the 32 tokens split over the ranks; per block the norms, the expert-
    parallel exchange around the tensor-core path, the residual.  Device
    time max over ranks."""
    import torch
    import torch.distributed as dist
    from flash_moe_b200 import _lib, synth
    from flash_moe_b200.ep import ep_exchange_step
    arena = backend.store
    base = arena.layer(base_layer)
    ids = []
    for l in range(40):
        lid = 1000 + l
        arena.add_device_layer(lid, base.reshuffled(5000 + l) if l else base)
        ids.append(lid)
    H = base.weights.hidden
    lib = backend.lib
    x1 = torch.from_numpy(synth.make_tokens(7000, 1, H)).to(dev)
    h, n, m = (torch.empty_like(x1) for _ in range(3))
    outs = [torch.empty_like(x1) for _ in range(2)]
    flags = backend.flags | (_lib.NO_SHARED if rank else 0)

    def chain1(layer_flags):
        # the stream current at the call: inside a graph capture, the
        # capturing stream, so that the norm kernels join the graph
        stream = torch.cuda.current_stream(dev).cuda_stream
        src = x1
        for i, lid in enumerate(ids):
            _lib.check(lib.moe_b200_block_prepare(src.data_ptr(), h.data_ptr(), n.data_ptr(), 1, H,
                                                  1e-6, stream), "moe_b200_block_prepare")
            backend.forward_layer_device(lid, n, m, flags=layer_flags)
            dist.all_reduce(m)
            dst = outs[i % 2]
            _lib.check(lib.moe_b200_block_finish(h.data_ptr(), m.data_ptr(), dst.data_ptr(), 1, H,
                                                 stream), "moe_b200_block_finish")
            src = dst
        return src
    chain1(flags)
    torch.cuda.synchronize()
    mode = "CUDA graph of the 40 blocks"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            last = chain1(flags)
        run1 = g.replay
    except RuntimeError:
        g, mode = None, "stream launches"
        torch.cuda.synchronize()
        dist.barrier()
        run1 = lambda: chain1(flags)  # noqa: E731
        last = outs[1]
    ms1 = _time_ranks(run1, 5, warmup=2)
    # the last block against the exact engine on the same input (a 40-block
    # chain is compared block by block: one near-tied routing that flips in
    # an early block changes everything after it)
    x39, y_fast = outs[0].clone(), last.clone()
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.moe_b200_block_prepare(x39.data_ptr(), h.data_ptr(), n.data_ptr(), 1, H, 1e-6,
                                          stream), "moe_b200_block_prepare")
    backend.forward_layer_device(ids[-1], n, m, flags=_lib.EXACT | (_lib.NO_SHARED if rank else 0))
    dist.all_reduce(m)
    y_exact = torch.empty_like(x1)
    _lib.check(lib.moe_b200_block_finish(h.data_ptr(), m.data_ptr(), y_exact.data_ptr(), 1, H, stream),
               "moe_b200_block_finish")
    err1 = _rel_err_ranks(y_fast, y_exact)
    del g
    # batch 32, tokens split over the ranks
    T = 32
    per = T // world
    xs = torch.from_numpy(synth.make_tokens(7001, T, H)[rank * per:(rank + 1) * per]).to(dev)
    hb, nb, mb, yb = (torch.empty_like(xs) for _ in range(4))
    x_all = torch.empty((T, H), dtype=torch.float32, device=dev)
    y_part = torch.empty_like(x_all)
    y_r, y_s = torch.empty_like(xs), torch.empty_like(xs)

    def chain32():
        src = xs
        for lid in ids:
            _lib.check(lib.moe_b200_block_prepare(src.data_ptr(), hb.data_ptr(), nb.data_ptr(), per,
                                                  H, 1e-6, stream), "moe_b200_block_prepare")
            ep_exchange_step(
                nb, lambda xa, yp, lid=lid: backend.prefill_device(lid, xa, yp, flags=_lib.NO_SHARED),
                lambda xx, ys, lid=lid: backend.prefill_device(lid, xx, ys, flags=_lib.SHARED_ONLY),
                x_all, y_part, y_r, y_s, mb)
            _lib.check(lib.moe_b200_block_finish(hb.data_ptr(), mb.data_ptr(), yb.data_ptr(), per, H,
                                                 stream), "moe_b200_block_finish")
            src = yb
    ms32 = _time_ranks(chain32, 2, warmup=1)
    for lid in ids:
        arena.drop_layer(lid)
    per_tok = 40 * step_bytes(8)
    gbs = per_tok / (ms1 / 1e3) / 1e9
    return {"config": f"config 5 sharded over {world} GPUs: 40 blocks, {base.weights.n_experts // world} "
                      "experts per layer per GPU; batch 1 replicated (fused kernel on the own "
                      f"experts + 8 KB NCCL all-reduce per block, {mode}); batch 32 split "
                      f"({per} per GPU), expert-parallel tensor-core path per block",
            "batch1_us_per_token": round(ms1 * 1e3, 1), "batch1_us_per_layer": round(ms1 * 1e3 / 40, 2),
            "batch1_gbs_union": round(gbs, 1),
            "batch1_last_block_max_rel_err_vs_exact": float(f"{err1:.3e}"),
            "batch32_ms_per_step": round(ms32, 3), "batch32_tokens_per_s": round(T / (ms32 / 1e3)),
            "peak_source": f"{peak_kind} hbm_gbs"}


def bench_sequence_ep(backend, layer: int, dev, world: int, rank: int, tokens: int, name: str,
                      peaks: dict, peak_kind: str, use_prefill: bool, bound: str = "tensor") -> dict:
    """A many-token layer expert-parallel: the `tokens` tokens split evenly
    over the ranks; per call an all-gather of the tokens (NCCL), the rank's
    experts over all of them (tensor-core path, or the decode engine), a
    reduce-scatter of the partial outputs, and the shared expert of the
    rank's own tokens.  Device time max over ranks; the output against the
    one-call exact fp32 reference on the same rank's tokens."""
    import torch
    from flash_moe_b200 import _lib, synth
    from flash_moe_b200.ep import ep_exchange_step
    lw = backend.store.layer(layer).weights
    H = lw.hidden
    per = tokens // world
    x_all_host = synth.make_tokens(404 if use_prefill else 3000, tokens, H)
    xo = torch.from_numpy(x_all_host[rank * per:(rank + 1) * per]).to(dev)
    x_all = torch.empty((tokens, H), dtype=torch.float32, device=dev)
    y_part = torch.empty_like(x_all)
    y_r, y_s, y = (torch.empty((per, H), dtype=torch.float32, device=dev) for _ in range(3))
    ids = torch.empty((tokens, lw.top_k), dtype=torch.int32, device=dev)
    if use_prefill:
        routed = lambda xa, yp: backend.prefill_device(layer, xa, yp, ids, flags=_lib.NO_SHARED)  # noqa: E731
        shared = lambda xx, ys: backend.prefill_device(layer, xx, ys, flags=_lib.SHARED_ONLY)  # noqa: E731
    else:
        routed = lambda xa, yp: backend.forward_layer_device(layer, xa, yp, ids,  # noqa: E731
                                                             flags=backend.flags | _lib.NO_SHARED)
        shared = lambda xx, ys: backend.forward_layer_device(layer, xx, ys,  # noqa: E731
                                                             flags=backend.flags | _lib.SHARED_ONLY)

    def call():
        ep_exchange_step(xo, routed, shared, x_all, y_part, y_r, y_s, y)
    ms = _time_ranks(call, 5)
    # reference: the exact engine through the same decomposition
    want = torch.empty_like(y)
    ep_exchange_step(
        xo, lambda xa, yp: backend.forward_layer_device(layer, xa, yp, flags=_lib.EXACT | _lib.NO_SHARED),
        lambda xx, ys: backend.forward_layer_device(layer, xx, ys, flags=_lib.EXACT | _lib.SHARED_ONLY),
        x_all, y_part, y_r, y_s, want)
    call()
    err = _rel_err_ranks(y, want)
    uniq = int(np.unique(ids.cpu().numpy()).size)
    out = {"config": f"{name}: {tokens} tokens split over {world} GPUs ({per} per rank), "
                     f"{lw.n_experts // world} experts per rank; all-gather, "
                     f"{'tensor-core prefill path' if use_prefill else 'decode engine'} on the "
                     "held experts, reduce-scatter, own shared expert",
           "us_per_step": round(ms * 1e3, 1), "tokens_per_s": round(tokens / (ms / 1e3)),
           "unique_experts_touched": uniq, "max_rel_err_vs_exact": float(f"{err:.3e}")}
    if bound == "tensor":
        tf = PREFILL_FLOPS_PER_TOKEN * tokens / (ms / 1e3) / 1e12
        out["tflops"] = round(tf, 1)
        out["frac_of_world_tensor_peak"] = round(tf / (peaks.get("bf16_tflops", 1590.0) * world), 4)
    else:
        algo = uniq * lw.expert_bytes + lw.shared_bytes + lw.router.nbytes + tokens * 2 * H * 4
        gbs = algo / (ms / 1e3) / 1e9
        out["gbs_union"] = round(gbs, 1)
        out["frac_of_world_hbm"] = round(gbs / (peaks["hbm_gbs"] * world), 4)
    out["peak_source"] = f"{peak_kind} peaks x {world} GPUs"
    return out


def run_e2e_breakdown(args) -> None:
    """Where the time of one synchronous host-buffer decode call goes (config
    2, one token, one GPU): host wall-clock per call, mean over many calls,
    of (a) a ctypes call of a trivial export (the binding's fixed cost),
    (b) the public host-buffer call (moe_b200_decode_host: pinned staging,
    one graph launch, completion wait, copy out), (c) a device-buffer call
    followed by a stream synchronisation, and the device time of (d) one
    single-step launch (CUDA events, back to back)."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lw = synth.make_layer(seed=0)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    be = B200ExpertBackend(arena)
    H = lw.hidden
    xs = synth.make_tokens(11, 1, H)
    hx = torch.from_numpy(xs).pin_memory()
    hy = torch.empty((1, H), dtype=torch.float32).pin_memory()
    xd = hx.to(dev)
    yd = torch.empty_like(xd)
    stream = torch.cuda.current_stream(dev)
    n = 2000

    def wall(fn):
        for _ in range(50):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        return (time.perf_counter() - t0) / n * 1e6
    lib = be.lib
    out = {"ctypes_call_us": round(wall(lambda: lib.moe_b200_version()), 2)}
    out["host_buffer_call_us"] = round(wall(lambda: be.decode_host_ptrs(
        0, hx.data_ptr(), 1, hy.data_ptr(), stream_handle=stream.cuda_stream)), 2)

    def dev_sync():
        be.forward_layer_device(0, xd, yd)
        stream.synchronize()
    out["device_call_plus_sync_us"] = round(wall(dev_sync), 2)
    out["device_call_us_back_to_back"] = round(_time_calls(lambda: be.forward_layer_device(0, xd, yd), n) * 1e3, 2)
    out["config"] = "config-2 layer, 1 token per call, one GPU, host wall clock (perf_counter) per call"
    print(json.dumps({"e2e_breakdown": out}), flush=True)


PREFILL_ROLES = ["producer_waits_stage", "raw_producer_waits_slot", "dequant_waits_raw",
                 "dequant_waits_stage", "mma_waits_full", "mma_waits_accumulator",
                 "epilogue_waits", "epilogue_busy"]


def prefill_role_counters(backend, layer: int, x, y) -> dict:
    """Per-role wait counters of the expert GEMMs of one prefill call: the
    kernels' trace slots (clock64 cycles each role spent waiting, per CTA),
    as shares of the CTA's cycles, mean over CTAs.  A diagnostic."""
    import ctypes as C
    import torch
    G = torch.cuda.get_device_properties(x.device).multi_processor_count
    buf = torch.zeros(G * 32, dtype=torch.int64, device=x.device)
    backend.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
    try:
        backend.prefill_device(layer, x, y)
        torch.cuda.synchronize()
    finally:
        backend.lib.moe_b200_set_trace(None, 0)
    a = buf.view(G, 32).cpu().numpy().astype(np.float64)
    out = {}
    for mode, name in enumerate(["router", "gate_up", "down"]):
        blk = a[:, mode * 10: mode * 10 + 10]
        cyc = blk[:, 8].mean()
        if cyc <= 0:
            continue
        out[name] = {"cycles_per_cta": round(cyc), "units_per_cta": round(blk[:, 9].mean(), 2)}
        out[name].update({r: round(blk[:, i].mean() / cyc * 100, 1) for i, r in enumerate(PREFILL_ROLES)})
    return out


def run_prefill_only(args) -> None:
    """The config-4 prefill and the config-3 tensor-core call alone (one
    GPU), with the GEMMs' per-role wait counters, for profiling."""
    import torch
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    dev = torch.device("cuda", 0)
    arena = ExpertArena(dev)
    arena.add_layer(0, synth.make_layer(seed=0))
    lwz = synth.make_layer(seed=0, zipf_s=1.1)
    arena.add_layer(1, lwz)
    backend = B200ExpertBackend(arena)
    peaks, peak_kind = measured_peaks()
    out = {"prefill": bench_prefill(backend, 0, dev, peaks, peak_kind)}
    x = torch.from_numpy(synth.make_tokens(404, 4096, 2048)).to(dev).to(torch.bfloat16)
    y = torch.empty((4096, 2048), dtype=torch.float32, device=dev)
    out["prefill"]["role_counters_pct"] = prefill_role_counters(backend, 0, x, y)
    x64 = torch.from_numpy(synth.make_tokens(3000, 64, 2048)).to(dev)
    y64 = torch.empty_like(x64)
    ms = _time_calls(lambda: backend.prefill_device(1, x64, y64), 20)
    out["batched_tensor_path"] = {"us_per_call_64_tokens": round(ms * 1e3, 1),
                                  "role_counters_pct": prefill_role_counters(backend, 1, x64, y64)}
    print(json.dumps(out), flush=True)


def run_kernel_times(args) -> None:
    """Per-kernel device time of one tensor-core layer call at 32, 64 (the
    config-3 layer with its Zipf bias) and 4096 tokens (config 4), from the
    CUDA activity records torch.profiler collects (no replay, no
    serialisation), mean over 10 calls, beside the call's own CUDA-event
    time.  The kernels are profiled with programmatic dependent launch off
    (MOE_B200_NO_PDL): with it, a kernel's span would include its wait for
    the previous kernel.  A diagnostic: nothing of it is a bench value."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    from flash_moe_b200 import synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    arena = ExpertArena(dev)
    arena.add_layer(0, synth.make_layer(seed=0))
    arena.add_layer(1, synth.make_layer(seed=0, zipf_s=1.1))
    be = B200ExpertBackend(arena)
    cases = (("tokens_32", 1, synth.make_tokens(3001, 32, 2048), torch.float32),
             ("tokens_64", 1, synth.make_tokens(3000, 64, 2048), torch.float32),
             ("tokens_4096", 0, synth.make_tokens(404, 4096, 2048), torch.bfloat16))
    out = {}
    n = 10
    for name, layer, xs, dt in cases:
        x = torch.from_numpy(xs).to(dev).to(dt)
        y = torch.empty((x.shape[0], 2048), dtype=torch.float32, device=dev)
        ms = _time_calls(lambda: be.prefill_device(layer, x, y), 20)
        os.environ["MOE_B200_NO_PDL"] = "1"
        ms_plain = _time_calls(lambda: be.prefill_device(layer, x, y), 20)
        try:
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(n):
                    be.prefill_device(layer, x, y)
                torch.cuda.synchronize()
        finally:
            del os.environ["MOE_B200_NO_PDL"]
        per = {}
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                t = getattr(ev, "device_time", None)
                t = ev.cuda_time if t is None else t
                key = ev.name.split("(")[0].replace("moeb200::", "").replace("void ", "")
                per[key] = per.get(key, 0.0) + t / n
        assert be.prefill_errors() == 0
        out[name] = {"us_per_call": round(ms * 1e3, 1),
                     "us_per_call_plain_launches": round(ms_plain * 1e3, 1),
                     "kernel_us_per_call": {k: round(v, 1) for k, v in per.items()},
                     "kernel_sum_us": round(sum(per.values()), 1)}
    print(json.dumps({"kernel_times": out}), flush=True)


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


DECODE_STAMPS = ["entry", "x_ready", "router_rows", "scores_out", "topk", "shared_gu",
                 "chunk0", "gate_up", "act_gathered", "act_quantised", "down_rows", "down",
                 "step_end"]


def run_trace(args) -> None:
    """Phase timeline of the fused single-token kernel (config-2 layer): the
    middle step of one multi-step launch, independent steps over `--copies`
    layer copies and a chained 40-block stack, from the kernel's trace
    stamps (%globaltimer, 32 ns ticks); us since the first CTA began the
    step, median / max over the CTAs.  A diagnostic: nothing of it is a
    bench value."""
    import ctypes as C
    import torch
    from flash_moe_b200 import _lib, synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    from flash_moe_b200.ep import DecodeRunner
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lw = synth.make_layer(seed=0)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw)
    for c in range(1, args.copies):
        arena.add_device_layer(c, arena.layer(0).clone())
    be = B200ExpertBackend(arena)
    G = torch.cuda.get_device_properties(dev).multi_processor_count
    H = lw.hidden
    toks = torch.from_numpy(synth.make_tokens(3, 64, H)).to(dev)
    runner = DecodeRunner(be, list(range(args.copies)), toks)
    steps = max(args.steps, 8)
    ind = runner.step_tables(steps)
    x1 = toks[:1]
    tmp = torch.empty((2, H), dtype=torch.float32, device=dev)
    y1 = torch.empty_like(x1)
    rows = [(i % args.copies, _lib.STEP_BLOCK | (_lib.STEP_CHAIN if i else 0),
             x1[0] if i == 0 else None, y1[0] if i == steps - 1 else tmp[i % 2], None, None)
            for i in range(steps)]
    chain = (be.layer_table(list(range(args.copies))), be.step_table(rows))
    out = {}
    for name, tabs in (("independent", ind), ("chained_blocks", chain)):
        fn = lambda: be.decode_steps_device(tabs[0], tabs[1], steps, 0)  # noqa: E731
        ms = _time_calls(fn, 3)
        buf = torch.zeros(G * 32, dtype=torch.int64, device=dev)
        be.lib.moe_b200_set_trace(C.c_void_p(buf.data_ptr()), G)
        try:
            fn()
            torch.cuda.synchronize()
        finally:
            be.lib.moe_b200_set_trace(None, 0)
        t = buf.view(G, 32).cpu().numpy()[:, :len(DECODE_STAMPS)].astype(np.float64)
        t0 = t[:, 0][t[:, 0] > 0].min()
        t = np.where(t > 0, (t - t0) / 1e3, np.nan)
        stamps = {nm: [round(float(np.nanmedian(t[:, i])), 2), round(float(np.nanmax(t[:, i])), 2)]
                  for i, nm in enumerate(DECODE_STAMPS) if np.isfinite(t[:, i]).any()}
        out[name] = {"us_per_step": round(ms * 1e3 / steps, 2), "stamps_median_max_us": stamps}
    out["device_error"] = be.device_errors()
    print(json.dumps({"trace": out}), flush=True)


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
    rank_sum_bytes = float(bytes_t.item())
    # the job's bytes: the distinct experts all ranks' tokens select per step,
    # router and shared expert once (the replicated copies each rank reads
    # are not counted again)
    total_bytes = float(runner.union_bytes(args.steps))
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
        cpu = cpu_layer_baseline(lw, synth.make_tokens(1000, 64, H), args.cpu_seconds)
    launches = 1 if tables is not None else runner.launches_per_step * args.steps
    graph = None
    tables = None
    extra = {}
    if world > 1 and not args.no_extra:
        # every rank takes part; rank 0 prints
        extra["allreduce"] = bench_allreduce(backend, list(range(args.copies)), dev, world, rank,
                                             min(args.steps, 64), peaks, peak_kind)
        extra["prefill"] = bench_sequence_ep(backend, 0, dev, world, rank, 4096,
                                             "config 4 prefill", peaks, peak_kind, True)
        lwz = synth.make_layer(seed=0, zipf_s=1.1)
        arena.add_layer(5000, lwz, expert_begin=begin, expert_count=per)
        extra["batched_decode"] = bench_sequence_ep(backend, 5000, dev, world, rank, 64,
                                                    "config 3 batched decode (Zipf 1.1)", peaks,
                                                    peak_kind, True, bound="hbm")
        arena.drop_layer(5000)
        extra["stack"] = bench_stack_ep(backend, 0, dev, world, rank, peaks, peak_kind)
    if rank == 0 and world == 1 and not args.no_extra:
        cpu_on = not args.no_cpu
        extra["expert"] = bench_expert(dev, peaks, peak_kind, args.cpu_seconds if cpu_on else None)
        extra["fp16_graph"] = bench_fp16_graph(backend, 0, dev)
        extra["prefill"] = with_cpu(
            bench_prefill(backend, 0, dev, peaks, peak_kind),
            lambda: cpu_sequence_baseline(lw, synth.make_tokens(404, 4096, H), sample_experts=24),
            cpu_on)
        lwz = synth.make_layer(seed=0, zipf_s=1.1)
        extra["batched_decode"] = with_cpu(
            bench_batched(dev, peaks, peak_kind, lwz),
            lambda: cpu_sequence_baseline(lwz, synth.make_tokens(3000, 64, H)), cpu_on)
        extra["stack"] = with_cpu(bench_stack(backend, 0, dev, peaks, peak_kind),
                                  lambda: cpu_stack_baseline(lw, H), cpu_on)
        extra["delta"] = bench_delta(dev, peaks, peak_kind, cpu=not args.no_cpu)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 6),
            "us_per_token": round(per_step_ms * 1e3 / 1, 3),
            "hbm_frac_of_8tbs": round(gbs / (8000.0 * world), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "s16 x packed GGUF codes (activations quantised to 16-bit fixed point per "
                     "256-value block as two int8 planes, dp4a int32 sums; fp32 router, block "
                     "scales, SwiGLU and combine)",
            "data": "synthetic (seeded, config-2 shapes and distributions)",
            "config": {"workload": "config 2: one MoE layer decode, 1 token/step/GPU, 256 experts "
                                   "top-8, Q3_K/Q3_K/Q4_K experts + Q8_0 shared expert",
                       "tokens_per_step_per_gpu": 1, "layer_copies": args.copies,
                       "l2": f"rotating {args.copies} layer copies at distinct addresses "
                             f"({args.copies * step_bytes(8) / 1e6:.0f} MB touched per rotation > 2x L2)",
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "engine": args.engine, "launch": launch_mode,
                       "algorithmic_bytes_per_token": step_bytes(8),
                       "bytes_counted": "union per step: distinct experts of all ranks' tokens + "
                                        "router + shared expert + gate vector once",
                       "union_bytes_per_step": round(total_bytes / args.steps),
                       "rank_sum_bytes_per_step": round(rank_sum_bytes / args.steps)},
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
    ap.add_argument("--only", choices=["prefill", "delta", "trace", "e2e", "kernels"], default=None,
                    help="run only one measurement: the config-4 prefill or the DeltaNet step "
                         "(for profiling), the decode kernel's phase timeline, the host-call "
                         "breakdown, or per-kernel device times of the tensor-core calls")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the prefill and batched-decode measurements (N = 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.only == "prefill":
        run_prefill_only(args)
    elif args.only == "trace":
        run_trace(args)
    elif args.only == "e2e":
        run_e2e_breakdown(args)
    elif args.only == "kernels":
        run_kernel_times(args)
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
