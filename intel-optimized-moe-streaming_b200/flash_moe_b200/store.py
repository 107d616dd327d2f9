"""HBM-resident expert store.

The reference streams each expert's byte range out of the GGUF file into a
bounded RAM LRU with async prefetch (``src/flash_moe/store.py:138-239``) and
hands ``read_all(key) -> {"gate", "up", "down": bytes}`` to the kernel
(``backend_ov.py:373-377``).  On a B200 the whole routed-expert set of a
layer (~381 MB for 256 Qwen3.6 experts, ~15.5 GB for 40 layers) fits in HBM
many times over, so ``ExpertArena`` uploads every layer once, in its native
GGUF block layout, and the kernels read it in place: no per-token host
traffic, no cache, and prefetch is a no-op.

Per layer the arena holds one contiguous device buffer per tensor family,
exactly as the GGUF ``ffn_{gate,up,down}_exps`` tensors are laid out
(expert ``e`` at ``e * per_expert_bytes``), the fp32 router ``[E x H]``, an
optional router bias, and the shared expert.  Under expert parallelism a GPU
holds only the slice ``[expert_begin, expert_begin + expert_count)`` of the
routed experts and a full copy of the router and shared expert.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .key import ArenaStats, ExpertKey
from .synth import LayerWeights


def _to_device(arr: np.ndarray, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.to(device)


class DeviceLayer:
    """Device copy of one layer plus the ``moe_b200_layer`` struct that
    points at it (valid while this object is alive)."""

    def __init__(self, lw: LayerWeights, device, expert_begin: int = 0,
                 expert_count: int | None = None, flags: int = 0):
        count = lw.n_experts - expert_begin if expert_count is None else expert_count
        if expert_begin < 0 or count < 1 or expert_begin + count > lw.n_experts:
            raise ValueError(f"expert slice [{expert_begin}, {expert_begin + count}) outside "
                             f"0..{lw.n_experts}")
        self.weights = lw
        self.device = torch.device(device)
        self.expert_begin, self.expert_count = expert_begin, count
        b, e = expert_begin, expert_begin + count
        self.gate = _to_device(lw.gate[b * lw.gate_stride:e * lw.gate_stride], self.device)
        self.up = _to_device(lw.up[b * lw.up_stride:e * lw.up_stride], self.device)
        self.down = _to_device(lw.down[b * lw.down_stride:e * lw.down_stride], self.device)
        self.router = _to_device(lw.router, self.device)
        self.router_bias = (_to_device(lw.router_bias, self.device)
                            if lw.router_bias is not None else None)
        self.shared = None
        if lw.shared_inter:
            self.shared = {
                "gate": _to_device(lw.shared_gate, self.device),
                "up": _to_device(lw.shared_up, self.device),
                "down": _to_device(lw.shared_down, self.device),
                "gate_inp": _to_device(lw.shared_gate_inp, self.device),
            }
        self.struct = self._make_struct(flags)

    def _make_struct(self, flags: int) -> _lib.Layer:
        lw = self.weights
        s = _lib.Layer()
        s.hidden, s.intermediate = lw.hidden, lw.inter
        s.n_experts, s.top_k = lw.n_experts, lw.top_k
        s.expert_begin, s.expert_count = self.expert_begin, self.expert_count
        s.gate_type, s.up_type, s.down_type = lw.gate_type, lw.up_type, lw.down_type
        s.flags = flags
        s.gate, s.up, s.down = self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr()
        s.router = self.router.data_ptr()
        s.router_bias = self.router_bias.data_ptr() if self.router_bias is not None else None
        if self.shared is not None:
            s.shared_intermediate = lw.shared_inter
            s.shared_gate_type, s.shared_up_type, s.shared_down_type = lw.shared_types
            s.shared_gate = self.shared["gate"].data_ptr()
            s.shared_up = self.shared["up"].data_ptr()
            s.shared_down = self.shared["down"].data_ptr()
            s.shared_gate_inp = self.shared["gate_inp"].data_ptr()
        return s

    def clone(self) -> "DeviceLayer":
        """A second resident copy of this layer at distinct device addresses
        (same values); used to rotate benchmark steps over more bytes than L2
        holds without regenerating weights on the host."""
        other = object.__new__(DeviceLayer)
        other.weights = self.weights
        other.device = self.device
        other.expert_begin, other.expert_count = self.expert_begin, self.expert_count
        other.gate, other.up, other.down = self.gate.clone(), self.up.clone(), self.down.clone()
        other.router = self.router.clone()
        other.router_bias = self.router_bias.clone() if self.router_bias is not None else None
        other.shared = ({k: v.clone() for k, v in self.shared.items()}
                        if self.shared is not None else None)
        other.struct = other._make_struct(self.struct.flags)
        return other

    def reshuffled(self, seed: int) -> "DeviceLayer":
        """Another layer of the same construction, made on the device: the
        rows of every packed tensor permuted by a seeded permutation (each row
        keeps its blocks, so every block keeps its drawn scales and quants)
        and a fresh N(0, 0.02) router and shared-gate vector.  Used to fill a
        deep stack of distinct resident layers without generating gigabytes
        on the host; the values are not those of synth.make_layer(seed)."""
        lw = self.weights
        g = torch.Generator(device=self.device)
        g.manual_seed(int(seed))

        def rows(t: torch.Tensor, row_bytes: int) -> torch.Tensor:
            r = t.view(-1, row_bytes)
            return r[torch.randperm(r.shape[0], generator=g, device=self.device)].reshape(-1)

        other = object.__new__(DeviceLayer)
        other.weights = lw
        other.device = self.device
        other.expert_begin, other.expert_count = self.expert_begin, self.expert_count
        other.gate = rows(self.gate, lw.gate_stride // lw.inter)
        other.up = rows(self.up, lw.up_stride // lw.inter)
        other.down = rows(self.down, lw.down_stride // lw.hidden)
        other.router = torch.randn(self.router.shape, generator=g, device=self.device) * 0.02
        other.router_bias = self.router_bias.clone() if self.router_bias is not None else None
        other.shared = None
        if self.shared is not None:
            sh = self.shared
            other.shared = {
                "gate": rows(sh["gate"], sh["gate"].numel() // lw.shared_inter),
                "up": rows(sh["up"], sh["up"].numel() // lw.shared_inter),
                "down": rows(sh["down"], sh["down"].numel() // lw.hidden),
                "gate_inp": torch.randn(sh["gate_inp"].shape, generator=g, device=self.device) * 0.02,
            }
        other.struct = other._make_struct(self.struct.flags)
        return other

    def with_flags(self, flags: int) -> _lib.Layer:
        s = _lib.Layer.from_buffer_copy(self.struct)
        s.flags = flags
        return s

    @property
    def resident_bytes(self) -> int:
        n = self.gate.numel() + self.up.numel() + self.down.numel() + self.router.numel() * 4
        if self.router_bias is not None:
            n += self.router_bias.numel() * 4
        if self.shared is not None:
            n += sum(t.numel() * t.element_size() for t in self.shared.values())
        return n

    def holds(self, expert: int) -> bool:
        return self.expert_begin <= expert < self.expert_begin + self.expert_count

    def expert_views(self, expert: int) -> dict[str, torch.Tensor]:
        """Device byte views of one held routed expert."""
        if not self.holds(expert):
            raise KeyError(f"expert {expert} is not held on this device")
        lw, i = self.weights, expert - self.expert_begin
        return {
            "gate": self.gate[i * lw.gate_stride:(i + 1) * lw.gate_stride],
            "up": self.up[i * lw.up_stride:(i + 1) * lw.up_stride],
            "down": self.down[i * lw.down_stride:(i + 1) * lw.down_stride],
        }


class ExpertArena:
    """All layers' experts resident in one GPU's HBM.

    Offers the read side of the reference store interface
    (``read_all``/``read_tensor``/``prefetch_many``, ``src/flash_moe/store.py:
    178-217``) so existing callers keep working; the kernels never go through
    it."""

    def __init__(self, device=None):
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self.layers: dict[int, DeviceLayer] = {}
        self.stats = ArenaStats()

    def add_layer(self, index: int, lw: LayerWeights, expert_begin: int = 0,
                  expert_count: int | None = None, flags: int = 0) -> DeviceLayer:
        dl = DeviceLayer(lw, self.device, expert_begin, expert_count, flags)
        old = self.layers.get(index)
        if old is not None:
            self.stats.resident_bytes -= old.resident_bytes
            self.stats.layers -= 1
        self.layers[index] = dl
        self.stats.resident_bytes += dl.resident_bytes
        self.stats.layers += 1
        return dl

    def add_device_layer(self, index: int, dl: DeviceLayer) -> DeviceLayer:
        old = self.layers.get(index)
        if old is not None:
            self.stats.resident_bytes -= old.resident_bytes
            self.stats.layers -= 1
        self.layers[index] = dl
        self.stats.resident_bytes += dl.resident_bytes
        self.stats.layers += 1
        return dl

    def drop_layer(self, index: int) -> None:
        """Release a resident layer (its device memory returns to the pool)."""
        old = self.layers.pop(index, None)
        if old is not None:
            self.stats.resident_bytes -= old.resident_bytes
            self.stats.layers -= 1

    def layer(self, index: int) -> DeviceLayer:
        try:
            return self.layers[index]
        except KeyError:
            raise KeyError(f"layer {index} is not resident") from None

    def tensor_types(self) -> dict[int, dict[str, int]]:
        """Per-layer ggml types, the shape of ``expert_tensor_types``
        (reference ``src/run_q4k_f16_openvino.py:136-155``)."""
        return {i: dict(dl.weights.kinds) for i, dl in self.layers.items()}

    def read_all(self, key: ExpertKey) -> dict[str, bytes]:
        self.stats.host_reads += 1
        views = self.layer(key.layer).expert_views(key.expert)
        return {name: t.cpu().numpy().tobytes() for name, t in views.items()}

    def read_tensor(self, key: ExpertKey, name: str) -> bytes:
        self.stats.host_reads += 1
        return self.layer(key.layer).expert_views(key.expert)[name].cpu().numpy().tobytes()

    def prefetch_many(self, keys) -> int:
        """Every expert is resident: nothing to fetch."""
        self.stats.prefetch_calls += 1
        return 0

    def prefetch(self, key) -> None:
        self.stats.prefetch_calls += 1

    def close(self) -> None:
        self.layers.clear()
