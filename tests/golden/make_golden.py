"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference project checked out (by default
the directory ``reference`` beside this repository, or
``$FLASH_MOE_REFERENCE_ROOT``) and the reference library built from its own
sources (``make -C oracle ref``):

    python tests/golden/make_golden.py [--reference <reference checkout>]

What produces the expected values:
  * dequantised blocks: ``gguf.quants.dequantize`` (gguf-py 0.19.0, the
    package the reference pins its decoders against,
    ``tools/test_dequant_k.py:121``) for f32, and the reference's own
    ``dequant_k`` export (compiled from ``cpp/dequant_k.cpp``) for binary16;
  * single experts: the reference's ``moe_quant_expert`` export
    (``cpp/moe_quant_dot.cpp:171``), both ``fp16_graph`` modes;
  * DeltaNet steps: the reference's ``moe_delta_heads`` export
    (``cpp/moe_delta.cpp:18-69``), several steps on one state per case;
  * MoE layers and sequences: the reference's own Python
    (``flash_moe.moe_layer.run_moe_layer`` / ``run_moe_sequence``,
    ``flash_moe.router.ExpertRouter``, ``flash_moe.shared_expert.SharedExpert``,
    ``flash_moe.native_expert.NativeExpert``), imported from the reference
    tree with a stub ``openvino`` module (OpenVINO is not installed and is not
    on the path these functions take), driving the reference library.

Inputs are regenerated from seeds by ``flash_moe_b200.synth``; each fixture
stores a sha256 of its inputs so a drift in the generator is detected rather
than silently compared.  Only small arrays (outputs, a few raw blocks) are
stored.
"""
from __future__ import annotations

import argparse
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "intel-optimized-moe-streaming_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))

from cases import DELTA_SPECS, LAYER_SPECS, delta_case, TRIPLES, layer_case, layer_digest, small_expert_inputs  # noqa: E402
from flash_moe_b200 import synth  # noqa: E402
from flash_moe_b200.formats import BLOCK, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0  # noqa: E402

TYPES = [Q8_0, Q3_K, Q4_K, Q5_K, Q6_K]


def stub_openvino(tmp: Path) -> None:
    """A minimal importable ``openvino`` package: enough for ``flash_moe``'s
    package ``__init__`` to import; none of its objects are used here."""
    pkg = tmp / "openvino"
    pkg.mkdir()
    (pkg / "__init__.py").write_text(
        "class Type:\n    f16='f16'; f32='f32'; bf16='bf16'; i8='i8'; u8='u8'\n"
        "class Core:\n    available_devices=['CPU']\n"
        "    def set_property(self,*a,**k): pass\n"
        "class Model:\n    def __init__(self,*a,**k): pass\n"
        "class Tensor:\n    def __init__(self,*a,**k): pass\n")
    (pkg / "opset13.py").write_text("")
    sys.path.insert(0, str(tmp))


def golden_dequant(ref, gguf) -> None:
    out = {}
    for t in TYPES:
        rng = np.random.default_rng(np.random.SeedSequence([23, t]))
        raw = synth.quant_blocks(rng, t, 8)
        bs, pb = BLOCK[t]
        # round trip of real quantisation where gguf-py implements it
        vals = (rng.standard_normal(bs * 4) * 0.05).astype(np.float32)
        try:
            rt = np.ascontiguousarray(
                gguf.quants.quantize(vals, gguf.GGMLQuantizationType(t))).view(np.uint8).reshape(-1, pb)
            raw = np.concatenate([raw, rt])
        except Exception:  # gguf-py has no quantiser for this type
            pass
        n = raw.shape[0] * bs
        f32 = gguf.quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(t)).reshape(-1)
        rc, f16 = ref.dequant(t, raw, want_f16=True)
        assert rc == 0
        rc32, r32 = ref.dequant(t, raw)
        assert rc32 == 0 and np.array_equal(r32.view(np.uint32), f32.astype(np.float32).view(np.uint32))
        bad, _ = ref.dequant(t, raw, n=n + 1)
        out[f"raw_{t}"] = raw.reshape(-1)
        out[f"f32_{t}"] = f32.astype(np.float32)
        out[f"f16_{t}"] = f16.view(np.uint16).copy()
        out[f"bad_n_status_{t}"] = np.int32(bad)
    np.savez_compressed(OUT / "dequant_blocks.npz", **out)


def golden_expert_small(ref) -> None:
    out = {}
    for i, kinds in enumerate(TRIPLES):
        tensors, x = small_expert_inputs(kinds, i)
        k = dict(zip(("gate", "up", "down"), kinds))
        for fg in (0, 1):
            rc, y = ref.expert(tensors, k, x, 256, 256, fg)
            out[f"y{fg}_{i}"] = y
            out[f"rc{fg}_{i}"] = np.int32(rc)
        out[f"digest_{i}"] = np.array(synth.digest(tensors["gate"], tensors["up"], tensors["down"], x))
    # status codes of malformed calls, on the first triple
    tensors, x = small_expert_inputs(TRIPLES[0], 0)
    k = dict(zip(("gate", "up", "down"), TRIPLES[0]))
    out["rc_bad_type"] = np.int32(ref.expert(tensors, dict(k, gate=999), x, 256, 256)[0])
    short = dict(tensors, up=tensors["up"][:-1])
    out["rc_bad_bytes"] = np.int32(ref.expert(short, k, x, 256, 256)[0])
    out["rc_bad_graph"] = np.int32(ref.expert(tensors, k, x, 256, 256, 2)[0])
    out["rc_bad_cols"] = np.int32(ref.expert(tensors, k, x, 256, 128)[0])
    np.savez_compressed(OUT / "expert_small.npz", **out)


def golden_expert_cfg1(ref) -> None:
    tensors, kinds, x = synth.make_expert_q4k(seed=1)
    out = {"digest": np.array(synth.digest(tensors["gate"], tensors["up"], tensors["down"], x))}
    for fg in (0, 1):
        rc, y = ref.expert(tensors, kinds, x, 2048, 512, fg)
        out[f"y{fg}"] = y
        out[f"rc{fg}"] = np.int32(rc)
    np.savez_compressed(OUT / "expert_cfg1.npz", **out)


def golden_delta(ref) -> None:
    out = {}
    for name in DELTA_SPECS:
        state, steps = delta_case(name)
        out[f"{name}_digest"] = np.array(synth.digest(state, *[a for st in steps for a in st]))
        ys, rcs = [], []
        for q, k, v, beta, gate in steps:
            rc, y = ref.delta_heads(state, q, k, v, beta, gate)
            ys.append(y)
            rcs.append(rc)
        out[f"{name}_y"] = np.stack(ys)
        out[f"{name}_rc"] = np.array(rcs, np.int32)
        out[f"{name}_state_sha"] = np.array(synth.digest(state))
        if state.size <= 4096:
            out[f"{name}_state"] = state.copy()
    # argument checks: one head of 8 x 8, then each limit crossed
    state, steps = delta_case("many_heads")
    q, k, v, beta, gate = steps[0]
    bad = {"heads0": (0, 8, 8), "heads257": (257, 8, 8), "dk0": (1, 0, 8),
           "dk1025": (1, 1025, 8), "dv0": (1, 8, 0), "dv1025": (1, 8, 1025)}
    for key, (h, dk, dv) in bad.items():
        out[f"rc_{key}"] = np.int32(ref._delta(state.ctypes.data, q.ctypes.data, k.ctypes.data,
                                               v.ctypes.data, beta.ctypes.data, gate.ctypes.data,
                                               v.ctypes.data, h, dk, dv))
    out["rc_null"] = np.int32(ref._delta(None, q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                         beta.ctypes.data, gate.ctypes.data, v.ctypes.data, 1, 8, 8))
    np.savez_compressed(OUT / "delta.npz", **out)
    print("delta ok", {n: out[f"{n}_rc"].tolist() for n in DELTA_SPECS})


class RefBackend:
    """Backend duck type over the reference library.  ``forward`` is the
    reference kernel per token; ``forward_batch`` runs it per row (the
    reference's batched path is OpenVINO, which is not available)."""

    def __init__(self, ref, lw, fp16_graph: int):
        self.ref, self.lw, self.fg = ref, lw, fp16_graph

    def forward(self, key, x, hidden, inter):
        rc, y = self.ref.expert(self.lw.expert(key.expert), self.lw.kinds, x, hidden, inter, self.fg)
        if rc:
            raise RuntimeError(f"native expert failed with status {rc}")
        return y

    def forward_batch(self, key, xs, hidden, inter):
        return np.stack([self.forward(key, row, hidden, inter) for row in xs])


def ref_layer_objects(ref, lw, layer: int = 0):
    from flash_moe.router import ExpertRouter
    from flash_moe.shared_expert import SharedExpert
    router = ExpertRouter(lw.hidden, lw.n_experts, top_k=lw.top_k,
                          gate_weights=lw.router, gate_dtype=np.float32)
    shared = None
    if lw.shared_inter:
        shared = SharedExpert.__new__(SharedExpert)
        shared.hidden_size = lw.hidden
        shared.intermediate_size = lw.shared_inter
        sk = lw.shared_kinds
        weights = {"gate_inp": lw.shared_gate_inp}
        for role, packed, shape in (("gate", lw.shared_gate, (lw.shared_inter, lw.hidden)),
                                    ("up", lw.shared_up, (lw.shared_inter, lw.hidden)),
                                    ("down", lw.shared_down, (lw.hidden, lw.shared_inter))):
            rc, v = ref.dequant(sk[role], packed, shape[0] * shape[1], want_f16=True)
            assert rc == 0
            weights[role] = np.ascontiguousarray(v.astype(np.float32).reshape(shape))
        shared.layers = {layer: weights}
    return router, shared


def golden_layers(ref) -> None:
    from flash_moe.moe_layer import run_moe_layer, run_moe_sequence
    from flash_moe.native_expert import NativeExpert
    from flash_moe.norm import RMSNorm

    for name, (kw, count) in LAYER_SPECS.items():
        lw, xs = layer_case(name)
        router, shared = ref_layer_objects(ref, lw)
        backend = RefBackend(ref, lw, 0)
        ys, ids, ws = [], [], []
        for x in xs:
            ys.append(run_moe_layer(0, x, router, backend, lw.hidden, lw.inter, shared))
            i, w = router.route(x)
            ids.append(i)
            ws.append(w)
        out = {"digest": np.array(layer_digest(lw, xs)),
               "y": np.stack(ys), "ids": np.array(ids, np.int64), "w": np.array(ws),
               "scores": np.stack([router.scores(x) for x in xs])}
        if name == "small":
            # the stock NativeExpert path (always fp16_graph=1)
            native = NativeExpert(ref.path)
            stock = type("Stock", (), {})()
            stock.forward = lambda key, x, h, i: native.forward(
                {k: v.tobytes() for k, v in lw.expert(key.expert).items()}, lw.kinds, x, h, i)
            out["y_stock"] = np.stack([run_moe_layer(0, x, router, stock, lw.hidden, lw.inter, shared)
                                       for x in xs])
            # sequences: per-token shared (8 tokens) and batched shared (20)
            for t in (8, 20):
                seq = synth.make_tokens(kw["seed"], t, lw.hidden, stream=1 + t)
                out[f"seq{t}"] = run_moe_sequence(0, seq, router, backend, lw.hidden, lw.inter, shared)
                out[f"seq{t}_digest"] = np.array(synth.digest(seq))
            # RMSNorm with unit weight, the identity-mixer stack's norm
            norm = RMSNorm(np.ones(lw.hidden, np.float32))
            out["norm_in"] = xs * 3.0
            out["norm_out"] = norm.forward(xs * 3.0).view(np.uint16)
        np.savez_compressed(OUT / f"layer_{name}.npz", **out)
        print(name, "ok", out["y"].shape)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: $FLASH_MOE_REFERENCE_ROOT or the "
                         "sibling directory 'reference')")
    ap.add_argument("--only", nargs="*", default=None,
                    help="regenerate only these fixture groups "
                         "(delta dequant expert_small expert_cfg1 layers)")
    args = ap.parse_args()
    import oracle as O
    if args.reference is None:
        args.reference = str(O.reference_root())
    O.build_oracle()
    if O.build_reference(args.reference) is None:
        print("reference sources not found", file=sys.stderr)
        return 2
    ref = O.ReferenceLibrary()
    import gguf
    with tempfile.TemporaryDirectory() as tmp:
        stub_openvino(Path(tmp))
        sys.path.insert(0, str(Path(args.reference) / "src"))
        groups = {"delta": lambda: golden_delta(ref),
                  "dequant": lambda: golden_dequant(ref, gguf),
                  "expert_small": lambda: golden_expert_small(ref),
                  "expert_cfg1": lambda: golden_expert_cfg1(ref),
                  "layers": lambda: golden_layers(ref)}
        for name, make in groups.items():
            if args.only is None or name in args.only:
                make()
    print("fixtures written to", OUT)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
