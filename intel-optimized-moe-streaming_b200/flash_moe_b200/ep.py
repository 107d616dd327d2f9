"""Decode stepping on one GPU or expert-parallel over several.

Expert parallelism (EP): rank r of N holds routed experts
[r*E/N, (r+1)*E/N) of every layer plus full copies of the router and the
shared expert.  One decode step for the T tokens each rank owns is ONE
launch of the fused multi-token kernel per rank (``moe_b200_decode_ep_p2p``)
that also does the exchange, over NVLink peer memory:

  1. dispatch: the kernel pushes the rank's tokens into every rank's
     exchange buffer and waits (bounded) for all ranks' tokens;
  2. it routes all N*T tokens with the replicated router and applies the
     experts this rank holds (experts held elsewhere contribute zero), plus
     the sigmoid-gated shared expert of its own tokens;
  3. combine: each CTA pushes its output rows of every token's partial sum
     to the token's owner, waits for the same rows from every rank and adds
     them in rank order.

Where the buffers cannot be mapped between the ranks, the same step runs
with collectives around the kernel: all-gather the tokens,
``moe_b200_decode_ep`` (held experts + own shared expert), reduce-scatter
the partial outputs.  For more than 8 gathered tokens, or shapes the fused
kernel does not take, the kernel is ``moe_b200_decode`` with NO_SHARED and
the owner adds ``moe_b200_decode`` with SHARED_ONLY after the
reduce-scatter.  With N = 1 a step is a single device call and nothing is
exchanged.
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import torch

from . import _lib

def expert_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of the routed experts rank `rank` of `world` holds."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return rank * per, per


def ep_exchange_step(x, routed_fn, shared_fn, x_all, y_part, y_routed, y_sh, y,
                     group=None) -> None:
    """One expert-parallel layer step of this rank's tokens ``x`` [t, H].

    ``routed_fn(x_all, y_part)`` writes, for all ``world * t`` gathered
    tokens, the weighted sum of the outputs of the experts this rank holds;
    ``shared_fn(x, y_sh)`` writes the gated shared expert of the own tokens,
    or is None when ``routed_fn`` already added it to the own tokens' rows
    (the reduce-scatter then writes ``y`` directly).  The collectives are
    the same on every rank and in the same order (all-gather, then
    reduce-scatter), whatever the device or backend."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(x_all, x, group=group)
    routed_fn(x_all, y_part)
    if shared_fn is None:
        dist.reduce_scatter_tensor(y, y_part, group=group)
        return
    dist.reduce_scatter_tensor(y_routed, y_part, group=group)
    shared_fn(x, y_sh)
    torch.add(y_routed, y_sh, out=y)


def profiled_traffic(root: Path, name: str = "decode_layer") -> float | None:
    """DRAM bytes per launch of the decode kernel from the committed ncu
    summary (``profiles/<name>*.txt`` line ``traffic_bytes_per_launch: N``)."""
    for p in sorted((root / "profiles").glob(f"{name}*.txt")):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
        if m:
            return float(m.group(1))
    return None


class PeerExchange:
    """This rank's exchange context for expert-parallel steps with the
    dispatch and combine over NVLink peer memory (``moe_b200_ep_create`` /
    ``_connect``).  Built collectively by every rank of `group`; when any
    rank cannot create or map the buffers, every rank gets None from
    ``create`` and the caller keeps the collective-based step."""

    def __init__(self, lib, handle, world: int, rank: int, tokens_per_rank: int):
        self.lib, self.handle = lib, handle
        self.world, self.rank, self.tokens_per_rank = world, rank, tokens_per_rank

    @classmethod
    def create(cls, lib, world: int, rank: int, tokens_per_rank: int, hidden: int, group=None):
        import ctypes as C
        import torch.distributed as dist
        ctx = C.c_void_p()
        blob = (C.c_uint8 * _lib.EP_BLOB_BYTES)()
        st = lib.moe_b200_ep_create(world, rank, tokens_per_rank, hidden, C.byref(ctx), blob)
        got = [None] * world
        dist.all_gather_object(got, (st, bytes(blob)), group=group)
        if any(s != 0 for s, _ in got):
            if st == 0:
                lib.moe_b200_ep_destroy(ctx)
            return None
        blobs = (C.c_uint8 * (_lib.EP_BLOB_BYTES * world)).from_buffer_copy(
            b"".join(b for _, b in got))
        st = lib.moe_b200_ep_connect(ctx, blobs)
        oks = [None] * world
        dist.all_gather_object(oks, st, group=group)
        if any(s != 0 for s in oks):
            lib.moe_b200_ep_destroy(ctx)
            return None
        return cls(lib, ctx, world, rank, tokens_per_rank)

    def close(self, group=None) -> None:
        """Free the buffers once no rank can still write into them: after
        every rank's last step (synchronise, then a barrier)."""
        import torch.distributed as dist
        if self.handle is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.lib.moe_b200_ep_destroy(self.handle)
        self.handle = None


class DecodeRunner:
    """Runs decode steps over a rotation of resident layers.

    Step i decodes token ``i % len(tokens)`` of this rank through layer
    ``layers[i % len(layers)]``."""


    def __init__(self, backend, layers, tokens: torch.Tensor, world: int = 1, rank: int = 0,
                 max_steps: int = 4096, peer_exchange: bool = True):
        self.be = backend
        self.layers = list(layers)
        self.tokens = tokens                      # [n, H] fp32 on device
        self.world, self.rank = world, rank
        dl = backend.store.layer(self.layers[0])
        self.lw = dl.weights
        self.dev = tokens.device
        H, K = self.lw.hidden, self.lw.top_k
        self.y = torch.empty((1, H), dtype=torch.float32, device=self.dev)
        self.max_steps = max_steps
        self.ids = torch.full((max_steps, world, K), -1, dtype=torch.int32, device=self.dev)
        if world > 1:
            self.x_all = torch.empty((world, H), dtype=torch.float32, device=self.dev)
            self.y_part = torch.empty((world, H), dtype=torch.float32, device=self.dev)
            self.y_routed = torch.empty((1, H), dtype=torch.float32, device=self.dev)
            self.y_sh = torch.empty((1, H), dtype=torch.float32, device=self.dev)
        self.fused_ep = world > 1 and backend.ep_fused_supported(self.layers[0], world)
        self.xchg = None
        if self.fused_ep and peer_exchange:
            self.xchg = PeerExchange.create(backend.lib, world, rank, 1, H)
        if world == 1:
            self.launches_per_step = backend.kernels_per_call(self.layers[0], 1)
        elif self.fused_ep:
            self.launches_per_step = 1
        else:
            self.launches_per_step = (
                backend.kernels_per_call(self.layers[0], world, backend.flags | _lib.NO_SHARED)
                + backend.kernels_per_call(self.layers[0], 1, backend.flags | _lib.SHARED_ONLY))
        self.kernel_name = ("k_decode_multi (peer-memory dispatch and combine, 1 launch per step)"
                            if self.xchg is not None
                            else "k_decode_multi (1 launch per step)" if self.fused_ep
                            else "k_decode_fused (1 launch per step)" if self.launches_per_step == 1
                            else f"moe_b200_decode ({self.launches_per_step} kernels per step)")
        self.recorded = 0
        self._graph = None

    # ------------------------------------------------------------------ step

    def _flags(self, extra=0):
        return self.be.flags | extra

    def step(self, i: int, x: torch.Tensor | None = None, y: torch.Tensor | None = None) -> None:
        layer = self.layers[i % len(self.layers)]
        x = self.tokens[i % self.tokens.shape[0]].view(1, -1) if x is None else x
        y = self.y if y is None else y
        slot = i % self.max_steps
        self.recorded = max(self.recorded, slot + 1)
        if self.world == 1:
            self.be.forward_layer_device(layer, x, y, topk_ids=self.ids[slot])
            return
        if self.xchg is not None:
            self.be.decode_ep_p2p_device(layer, self.xchg, x, y, topk_ids=self.ids[slot])
            return
        if self.fused_ep:
            ep_exchange_step(
                x,
                lambda xa, yp: self.be.decode_ep_device(layer, xa, yp, self.rank, 1,
                                                        topk_ids=self.ids[slot]),
                None, self.x_all, self.y_part, None, None, y)
            return
        ep_exchange_step(
            x,
            lambda xa, yp: self.be.forward_layer_device(layer, xa, yp, topk_ids=self.ids[slot],
                                                        flags=self._flags(_lib.NO_SHARED)),
            lambda xo, ys: self.be.forward_layer_device(layer, xo, ys,
                                                        flags=self._flags(_lib.SHARED_ONLY)),
            self.x_all, self.y_part, self.y_routed, self.y_sh, y)

    def step_tables(self, steps: int):
        """(layer table, step table) running `steps` consecutive steps in one
        launch (single GPU): step i decodes token i % n through layer i % L."""
        if self.world > 1:
            raise ValueError("multi-step launches run on one GPU")
        n = self.tokens.shape[0]
        rows = []
        for i in range(steps):
            slot = i % self.max_steps
            rows.append((i % len(self.layers), 0, self.tokens[i % n], self.y.view(-1),
                         self.ids[slot], None))
        self.recorded = max(self.recorded, min(steps, self.max_steps))
        return self.be.layer_table(self.layers), self.be.step_table(rows)

    def run_tables(self, tables, steps: int) -> None:
        self.be.decode_steps_device(tables[0], tables[1], steps, self.layers[0])

    def capture(self, steps: int):
        """CUDA graph of `steps` consecutive steps (single GPU, or
        expert-parallel steps over peer memory, which hold no collective)."""
        if self.world > 1 and self.xchg is None:
            return None
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for i in range(3):
                self.step(i)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                self.step(i)
        torch.cuda.synchronize()
        self._graph = g
        return g

    # ------------------------------------------------------------ accounting

    def union_bytes(self, steps: int) -> int:
        """Bytes the job's steps must read on any number of GPUs: per step
        the distinct experts all ranks' tokens select, and the router, the
        shared expert and the gate vector once (what one device decoding the
        same tokens reads).  The same on every rank (the routing of every
        gathered token is recorded)."""
        lw = self.lw
        ids = self.ids[:min(steps, self.max_steps)].cpu().numpy()
        total = 0
        for step_ids in ids:
            total += len(np.unique(step_ids[step_ids >= 0])) * lw.expert_bytes
        total += steps * (lw.shared_bytes + lw.router.nbytes + lw.hidden * 4)
        return int(total)

    def algorithmic_bytes(self, steps: int) -> int:
        """Packed weight + router + gate-vector bytes this rank's steps must
        read: the distinct held experts each step's tokens select, the
        shared expert and router once per step."""
        lw = self.lw
        per_expert = lw.expert_bytes
        ids = self.ids[:min(steps, self.max_steps)].cpu().numpy()
        dl = self.be.store.layer(self.layers[0])
        total = 0
        for step_ids in ids:
            sel = np.unique(step_ids[step_ids >= 0])
            held = sel[(sel >= dl.expert_begin) & (sel < dl.expert_begin + dl.expert_count)]
            total += len(held) * per_expert
        total += steps * (lw.shared_bytes + lw.router.nbytes + lw.hidden * 4)
        return int(total)

    # ------------------------------------------------------------------ e2e

    def e2e(self, steps: int, warmup: int) -> dict:
        """The same steps through host memory: each step's token starts in
        pinned host memory and its result ends there, synchronised like a
        caller that consumes the result.  One GPU: one ``moe_b200_decode_host``
        call per step (the device reads the token and writes the result
        through the pinned mapping); expert-parallel: host copies around the
        rank's exchange step."""
        H = self.lw.hidden
        n = self.tokens.shape[0]
        host_x = torch.empty((n, H), dtype=torch.float32).pin_memory()
        host_x.copy_(self.tokens.cpu())
        host_y = torch.empty((1, H), dtype=torch.float32).pin_memory()
        xd = torch.empty((1, H), dtype=torch.float32, device=self.dev)
        stream = torch.cuda.current_stream(self.dev)

        xrow = [host_x[j].data_ptr() for j in range(n)]
        yptr = host_y.data_ptr()
        sh = stream.cuda_stream

        def one(i):
            if self.world == 1:
                # one synchronous library call on the pinned rows: token in,
                # result out
                self.be.decode_host_ptrs(self.layers[i % len(self.layers)], xrow[i % n], 1, yptr,
                                         stream_handle=sh)
                return
            xd.copy_(host_x[i % n].view(1, -1), non_blocking=True)
            self.step(i, x=xd)
            host_y.copy_(self.y, non_blocking=True)
            stream.synchronize()

        for i in range(warmup):
            one(i)
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            one(i)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], device=self.dev)
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        byts = self.algorithmic_bytes(steps)
        bt = torch.tensor([float(byts)], device=self.dev, dtype=torch.float64)
        if self.world > 1:
            dist.all_reduce(bt)
        return {"value": round(float(bt.item()) / (ms / 1e3) / 1e9, 3), "unit": "GB/s",
                "us_per_token": round(ms * 1e3 / steps, 3),
                "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4}

    def close(self):
        self._graph = None
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None
