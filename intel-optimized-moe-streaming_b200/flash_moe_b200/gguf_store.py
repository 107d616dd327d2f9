"""MoE layers read from a GGUF file straight into the HBM arena.

The tensors are the ones the reference slices from the model file:

- ``blk.L.ffn_{gate,up,down}_exps.weight``: all routed experts of layer L,
  GGUF shape ne = [cols, rows, experts], packed blocks row-major, expert e
  the e-th equal slice (reference ``build_manifest_from_gguf``,
  ``src/run_q4k_f16_openvino.py:88-133``);
- ``blk.L.ffn_gate_inp.weight``: the router, ne = [hidden, experts], i.e.
  (experts, hidden) in memory (``ExpertRouter.from_gguf_tensor``,
  ``src/flash_moe/router.py:92-138``), F32 or F16;
- ``blk.L.ffn_{gate,up,down}_shexp.weight`` and
  ``blk.L.ffn_gate_inp_shexp.weight``: the shared expert and its gate
  vector (``src/flash_moe/shared_expert.py:45-62``), when present.

Block formats are read per layer and per tensor, as the reference insists
(``expert_tensor_types``, ``src/run_q4k_f16_openvino.py:136-155``): in the
real model they change from layer to layer.  The packed bytes are memory-
mapped by gguf-py and copied to the device once.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from .formats import BLOCK, SUPPORTED_TYPES
from .synth import LayerWeights

_ROLES = ("gate", "up", "down")
F32, F16 = 0, 1


def _reader(src):
    import gguf
    return src if hasattr(src, "tensors") else gguf.GGUFReader(str(src))


def _tmap(reader) -> dict:
    return {t.name: t for t in reader.tensors}


def expert_tensor_types(src, max_layers: int = 4096) -> dict[int, dict[str, int]]:
    """ggml type of gate/up/down of every layer that has routed experts
    (same result as the reference's ``expert_tensor_types``)."""
    tmap = _tmap(_reader(src))
    out: dict[int, dict[str, int]] = {}
    for layer in range(max_layers):
        types = {}
        for role in _ROLES:
            t = tmap.get(f"blk.{layer}.ffn_{role}_exps.weight")
            if t is not None:
                types[role] = int(t.tensor_type)
        if types:
            out[layer] = types
    return out


def moe_layers(src) -> list[int]:
    """Layer indices that hold a routed-expert block."""
    return sorted(expert_tensor_types(src))


def _packed(t, what: str) -> np.ndarray:
    ty = int(t.tensor_type)
    if ty not in SUPPORTED_TYPES:
        raise ValueError(f"{what}: ggml type {ty} is not one of the supported block formats")
    data = np.asarray(t.data)
    if data.dtype != np.uint8:
        raise ValueError(f"{what}: expected packed bytes, got {data.dtype}")
    return data.reshape(-1)


def _floats(t, what: str) -> np.ndarray:
    ty = int(t.tensor_type)
    if ty not in (F32, F16):
        raise ValueError(f"{what}: ggml type {ty}, expected F32 or F16")
    return np.asarray(t.data).astype(np.float32, copy=False).reshape(-1)


def layer_weights(src, layer: int, top_k: int = 8) -> LayerWeights:
    """The routed experts, router and shared expert of one layer as a
    ``LayerWeights`` over the file's memory-mapped bytes."""
    tmap = _tmap(_reader(src))
    name = lambda role: f"blk.{layer}.ffn_{role}_exps.weight"  # noqa: E731
    missing = [name(r) for r in _ROLES if name(r) not in tmap]
    if missing:
        raise KeyError(f"layer {layer} has no routed experts ({', '.join(missing)} missing)")
    tg, tu, td = (tmap[name(r)] for r in _ROLES)
    hidden, inter, n_exp = (int(v) for v in tg.shape[:3])
    if tuple(int(v) for v in tu.shape[:3]) != (hidden, inter, n_exp) or \
            tuple(int(v) for v in td.shape[:3]) != (inter, hidden, n_exp):
        raise ValueError(f"layer {layer}: gate {tg.shape}, up {tu.shape}, down {td.shape} "
                         "do not describe one expert FFN")
    for t, cols in ((tg, hidden), (tu, hidden), (td, inter)):
        ty = int(t.tensor_type)
        if ty not in SUPPORTED_TYPES:
            raise ValueError(f"{t.name}: ggml type {ty} is not one of the supported block formats")
        if cols % BLOCK[ty][0]:
            raise ValueError(f"{t.name}: {cols} columns are not whole blocks of type {ty}")
    tr = tmap.get(f"blk.{layer}.ffn_gate_inp.weight")
    if tr is None:
        raise KeyError(f"layer {layer}: blk.{layer}.ffn_gate_inp.weight missing")
    router = _floats(tr, tr.name)
    if router.size != n_exp * hidden:
        raise ValueError(f"{tr.name}: {router.size} values for {n_exp} experts x {hidden}")
    lw = LayerWeights(
        hidden=hidden, inter=inter, n_experts=n_exp, top_k=int(top_k),
        gate_type=int(tg.tensor_type), up_type=int(tu.tensor_type), down_type=int(td.tensor_type),
        gate=_packed(tg, tg.name), up=_packed(tu, tu.name), down=_packed(td, td.name),
        router=router.reshape(n_exp, hidden),
        meta={"source": "gguf", "layer": layer},
    )
    sh = {r: tmap.get(f"blk.{layer}.ffn_{r}_shexp.weight") for r in _ROLES}
    ginp = tmap.get(f"blk.{layer}.ffn_gate_inp_shexp.weight")
    if all(t is not None for t in sh.values()) and ginp is not None:
        s_inter = int(sh["gate"].shape[1])
        lw.shared_inter = s_inter
        lw.shared_types = tuple(int(sh[r].tensor_type) for r in _ROLES)
        lw.shared_gate = _packed(sh["gate"], sh["gate"].name)
        lw.shared_up = _packed(sh["up"], sh["up"].name)
        lw.shared_down = _packed(sh["down"], sh["down"].name)
        lw.shared_gate_inp = _floats(ginp, ginp.name)
        if lw.shared_gate_inp.size != hidden:
            raise ValueError(f"{ginp.name}: {lw.shared_gate_inp.size} values, expected {hidden}")
    return lw


def load_arena(src, device=None, layers=None, top_k: int = 8, expert_begin: int = 0,
               expert_count: int | None = None):
    """An ``ExpertArena`` holding `layers` (default: every MoE layer of the
    file) of a GGUF model, each under its own layer index; expert parallel
    ranks pass their ``expert_begin`` / ``expert_count`` slice."""
    from .store import ExpertArena
    reader = _reader(src)
    arena = ExpertArena(device)
    for layer in (moe_layers(reader) if layers is None else layers):
        arena.add_layer(layer, layer_weights(reader, layer, top_k), expert_begin=expert_begin,
                        expert_count=expert_count)
    return arena


def write_layers(path, layers: dict[int, LayerWeights], arch: str = "qwen35moe") -> Path:
    """Write layers in the model file's tensor naming and layout (for tests
    and for exporting synthetic models)."""
    import gguf
    from gguf import GGMLQuantizationType as Q
    path = Path(path)
    w = gguf.GGUFWriter(str(path), arch)

    def packed(name, arr, t, rows_shape, cols):
        rb = BLOCK[t][1] * (cols // BLOCK[t][0])
        w.add_tensor(name, np.asarray(arr, np.uint8).reshape(*rows_shape, rb),
                     raw_shape=(*rows_shape, rb), raw_dtype=Q(t))

    for layer, lw in sorted(layers.items()):
        E, I, H = lw.n_experts, lw.inter, lw.hidden
        packed(f"blk.{layer}.ffn_gate_exps.weight", lw.gate, lw.gate_type, (E, I), H)
        packed(f"blk.{layer}.ffn_up_exps.weight", lw.up, lw.up_type, (E, I), H)
        packed(f"blk.{layer}.ffn_down_exps.weight", lw.down, lw.down_type, (E, H), I)
        w.add_tensor(f"blk.{layer}.ffn_gate_inp.weight", np.ascontiguousarray(lw.router, np.float32))
        if lw.shared_inter:
            g, u, d = lw.shared_types
            Is = lw.shared_inter
            packed(f"blk.{layer}.ffn_gate_shexp.weight", lw.shared_gate, g, (Is,), H)
            packed(f"blk.{layer}.ffn_up_shexp.weight", lw.shared_up, u, (Is,), H)
            packed(f"blk.{layer}.ffn_down_shexp.weight", lw.shared_down, d, (H,), Is)
            w.add_tensor(f"blk.{layer}.ffn_gate_inp_shexp.weight",
                         np.ascontiguousarray(lw.shared_gate_inp, np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path
