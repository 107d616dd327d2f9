"""Worker of test_gpu_ep.py, one process per GPU under torchrun.

Rank r holds experts [r*E/N, (r+1)*E/N) of the config-2 layer.  Decode:
DecodeRunner steps for 4 tokens per rank, with the dispatch and combine
inside the fused kernel over peer memory (also replayed from a CUDA graph),
and with collectives around the kernel.  Prefill: the same exchange with
moe_b200_prefill for 64 tokens per rank.  Rank 0 compares every rank's
outputs with a single-GPU run of the whole layer and prints EP_OK."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "intel-optimized-moe-streaming_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def max_rel(a, b) -> float:
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    from flash_moe_b200 import _lib, synth
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.ep import DecodeRunner, ep_exchange_step, expert_range
    from flash_moe_b200.store import ExpertArena

    lw = synth.make_layer(seed=0)
    H = lw.hidden
    begin, count = expert_range(lw.n_experts, world, rank)
    arena = ExpertArena(dev)
    arena.add_layer(0, lw, expert_begin=begin, expert_count=count)
    be = B200ExpertBackend(arena)

    # ---- decode: 4 tokens per rank, one DecodeRunner step each, with the
    # exchange inside the kernel (peer memory) and around it (collectives)
    n_dec = 4
    toks = torch.from_numpy(synth.make_tokens(500 + rank, n_dec, H)).to(dev)
    runner = DecodeRunner(be, [0], toks, world, rank)
    assert runner.xchg is not None and runner.launches_per_step == 1
    y_dec = torch.empty((n_dec, H), dtype=torch.float32, device=dev)
    for i in range(n_dec):
        runner.step(i, x=toks[i:i + 1], y=y_dec[i:i + 1])
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    # the same steps replayed from a CUDA graph (no collective inside): the
    # last step's output is bit-identical
    graph = runner.capture(n_dec)
    graph.replay()
    torch.cuda.synchronize()
    assert be.device_errors() == 0
    assert torch.equal(runner.y[0], y_dec[n_dec - 1])
    del graph
    runner._graph = None
    runner_c = DecodeRunner(be, [0], toks, world, rank, peer_exchange=False)
    assert runner_c.xchg is None and runner_c.fused_ep
    y_col = torch.empty_like(y_dec)
    for i in range(n_dec):
        runner_c.step(i, x=toks[i:i + 1], y=y_col[i:i + 1])
    torch.cuda.synchronize()
    assert be.device_errors() == 0

    # ---- prefill: 64 tokens per rank through the tensor-core path
    n_pf = 64
    xp = torch.from_numpy(synth.make_tokens(600 + rank, n_pf, H)).to(dev)
    x_all = torch.empty((world * n_pf, H), dtype=torch.float32, device=dev)
    y_part = torch.empty_like(x_all)
    y_routed, y_sh, y_pf = (torch.empty((n_pf, H), dtype=torch.float32, device=dev)
                            for _ in range(3))
    ep_exchange_step(
        xp,
        lambda xa, yp: be.prefill_device(0, xa, yp, flags=_lib.NO_SHARED),
        lambda xo, ys: be.prefill_device(0, xo, ys, flags=_lib.SHARED_ONLY),
        x_all, y_part, y_routed, y_sh, y_pf)
    torch.cuda.synchronize()
    assert be.prefill_errors() == 0

    # gather every rank's inputs and outputs on rank 0
    g = lambda t: [torch.empty_like(t) for _ in range(world)]  # noqa: E731
    xs_dec, ys_dec, ys_col, xs_pf, ys_pf = g(toks), g(y_dec), g(y_col), g(xp), g(y_pf)
    dist.all_gather(xs_dec, toks)
    dist.all_gather(ys_dec, y_dec)
    dist.all_gather(ys_col, y_col)
    dist.all_gather(xs_pf, xp)
    dist.all_gather(ys_pf, y_pf)
    runner.close()
    runner_c.close()
    ok = True
    if rank == 0:
        full = ExpertArena(dev)
        full.add_layer(0, lw)
        ref = B200ExpertBackend(full)
        xd = torch.cat(xs_dec)
        want = torch.empty_like(xd)
        ref.forward_layer_device(0, xd, want, flags=_lib.EXACT)
        e_dec = max_rel(torch.cat(ys_dec).cpu().numpy(), want.cpu().numpy())
        e_col = max_rel(torch.cat(ys_col).cpu().numpy(), want.cpu().numpy())
        xa = torch.cat(xs_pf)
        want_pf = torch.empty_like(xa)
        ref.prefill_device(0, xa, want_pf)
        e_pf = max_rel(torch.cat(ys_pf).cpu().numpy(), want_pf.cpu().numpy())
        torch.cuda.synchronize()
        print(f"ep decode max rel {e_dec:.3e} (peer memory) {e_col:.3e} (collectives)  "
              f"ep prefill max rel {e_pf:.3e}", flush=True)
        # decode: the fused kernel's integer dot products (activations
        # quantised to 16 bits per 256-value block) against the exact engine,
        # at the layer tolerance; prefill: the same tensor-core arithmetic
        # on both sides, summed in another order
        ok = e_dec <= 1e-3 and e_col <= 1e-3 and e_pf <= 1e-5
        if ok:
            print("EP_OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
