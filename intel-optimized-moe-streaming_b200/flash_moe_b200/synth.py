"""Seeded synthetic MoE layers in native GGUF block layout.

The real Qwen3.6-35B-A3B GGUF is not available, so benchmarks and tests use
random weights with the shapes and value distributions of the benchmark
configurations.  Every draw comes from ``numpy.random.default_rng`` seeded by
``SeedSequence([seed, layer, stream])`` with a fixed stream number per tensor,
so each tensor can be regenerated on its own and independently of draw order
elsewhere.

Distributions (per tensor, per block):
  * Q4_K / Q5_K: uniform random bytes (nibbles uniform 0..15, packed 6-bit
    scales/mins uniform 0..63), then d = f16(|N(0,1)|*2e-3) and
    dmin = f16(|N(0,1)|*1e-3).
  * Q3_K: uniform random bytes, then d (bytes 108..109) = f16(|N(0,1)|*2e-3).
  * Q6_K: uniform random bytes, then d (bytes 208..209) = f16(|N(0,1)|*2e-3).
  * Q8_0: d = f16(|N(0,1)|*2e-3), quants int8 uniform in [-127, 127].
  * router: fp32 (experts, hidden) ~ N(0, 0.02), the GGUF ``ffn_gate_inp``
    orientation.
  * shared-expert gate vector: fp32 [hidden] ~ N(0, 0.02).
  * optional Zipf(s) popularity bias added to the router logits:
    bias_e = log(p_rank(e)), p_r proportional to r^-s, ranks assigned to
    experts by a seeded permutation.
  * tokens: fp32 ~ N(0, 1).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .formats import BLOCK, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0, tensor_bytes

# stream ids of SeedSequence([seed, layer, stream])
S_ROUTER, S_GATE, S_UP, S_DOWN = 0, 1, 2, 3
S_SH_GATE, S_SH_UP, S_SH_DOWN, S_SH_INP, S_ZIPF = 4, 5, 6, 7, 8
S_TOKENS = 100


def _rng(seed: int, layer: int, stream: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([int(seed), int(layer), int(stream)]))


def _f16_bytes(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(-1, 2)


def quant_blocks(rng: np.random.Generator, type_id: int, nblocks: int,
                 d_scale: float = 2e-3, dmin_scale: float = 1e-3) -> np.ndarray:
    """``nblocks`` random blocks of ``type_id`` as a (nblocks, bytes) array."""
    _, pb = BLOCK[type_id]
    raw = rng.integers(0, 256, size=(nblocks, pb), dtype=np.uint8)
    d = np.abs(rng.standard_normal(nblocks)) * d_scale
    if type_id in (Q4_K, Q5_K):
        raw[:, 0:2] = _f16_bytes(d)
        raw[:, 2:4] = _f16_bytes(np.abs(rng.standard_normal(nblocks)) * dmin_scale)
    elif type_id == Q3_K:
        raw[:, 108:110] = _f16_bytes(d)
    elif type_id == Q6_K:
        raw[:, 208:210] = _f16_bytes(d)
    elif type_id == Q8_0:
        raw[:, 0:2] = _f16_bytes(d)
        raw[:, 2:34] = rng.integers(-127, 128, size=(nblocks, 32), dtype=np.int8).view(np.uint8)
    else:
        raise ValueError(f"unsupported type {type_id}")
    return raw


def quant_tensor(rng: np.random.Generator, type_id: int, rows: int, cols: int) -> np.ndarray:
    """A packed [rows x cols] tensor as flat uint8, GGUF row-major block order."""
    bs, _ = BLOCK[type_id]
    return quant_blocks(rng, type_id, rows * (cols // bs)).reshape(-1)


@dataclass
class LayerWeights:
    """One MoE layer in host memory, in the layout it has inside a GGUF file.

    ``gate``/``up`` hold ``n_experts`` consecutive [inter x hidden] tensors and
    ``down`` ``n_experts`` consecutive [hidden x inter] tensors; expert ``e``
    is the byte slice ``[e*stride, (e+1)*stride)`` exactly as
    ``build_manifest_from_gguf`` slices ``ffn_*_exps`` (reference
    ``src/run_q4k_f16_openvino.py:112-122``)."""

    hidden: int
    inter: int
    n_experts: int
    top_k: int
    gate_type: int
    up_type: int
    down_type: int
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    router: np.ndarray                       # fp32 (n_experts, hidden)
    router_bias: np.ndarray | None = None    # fp32 (n_experts,) or None
    shared_inter: int = 0
    shared_types: tuple[int, int, int] = (Q8_0, Q8_0, Q8_0)
    shared_gate: np.ndarray | None = None
    shared_up: np.ndarray | None = None
    shared_down: np.ndarray | None = None
    shared_gate_inp: np.ndarray | None = None  # fp32 (hidden,)
    meta: dict = field(default_factory=dict)

    @property
    def gate_stride(self) -> int:
        return tensor_bytes(self.gate_type, self.inter, self.hidden)

    @property
    def up_stride(self) -> int:
        return tensor_bytes(self.up_type, self.inter, self.hidden)

    @property
    def down_stride(self) -> int:
        return tensor_bytes(self.down_type, self.hidden, self.inter)

    @property
    def kinds(self) -> dict[str, int]:
        return {"gate": self.gate_type, "up": self.up_type, "down": self.down_type}

    @property
    def shared_kinds(self) -> dict[str, int]:
        g, u, d = self.shared_types
        return {"gate": g, "up": u, "down": d}

    def expert(self, e: int) -> dict[str, np.ndarray]:
        """Packed bytes of routed expert ``e`` (views, no copy)."""
        return {
            "gate": self.gate[e * self.gate_stride:(e + 1) * self.gate_stride],
            "up": self.up[e * self.up_stride:(e + 1) * self.up_stride],
            "down": self.down[e * self.down_stride:(e + 1) * self.down_stride],
        }

    def shared(self) -> dict[str, np.ndarray] | None:
        if not self.shared_inter:
            return None
        return {"gate": self.shared_gate, "up": self.shared_up, "down": self.shared_down}

    def gate_he(self) -> np.ndarray:
        """Router weights as (hidden, experts), the orientation
        ``ExpertRouter`` multiplies with (reference ``router.py:176-191``)."""
        return np.ascontiguousarray(self.router.T, dtype=np.float32)

    @property
    def expert_bytes(self) -> int:
        return self.gate_stride + self.up_stride + self.down_stride

    @property
    def shared_bytes(self) -> int:
        if not self.shared_inter:
            return 0
        return int(self.shared_gate.nbytes + self.shared_up.nbytes + self.shared_down.nbytes)


def zipf_bias(seed: int, layer: int, n_experts: int, s: float = 1.1) -> np.ndarray:
    """log-popularity per expert: p_r ~ r^-s over ranks, ranks permuted."""
    ranks = np.arange(1, n_experts + 1, dtype=np.float64)
    p = ranks ** -s
    p /= p.sum()
    perm = _rng(seed, layer, S_ZIPF).permutation(n_experts)
    bias = np.empty(n_experts, np.float64)
    bias[perm] = np.log(p)
    return bias.astype(np.float32)


def make_layer(seed: int = 0, layer: int = 0, hidden: int = 2048, inter: int = 512,
               n_experts: int = 256, top_k: int = 8, gate_type: int = Q3_K,
               up_type: int = Q3_K, down_type: int = Q4_K, shared_inter: int = 512,
               shared_types: tuple[int, int, int] = (Q8_0, Q8_0, Q8_0),
               router_std: float = 0.02, zipf_s: float | None = None) -> LayerWeights:
    """A seeded MoE layer.  Defaults are the one-layer decode configuration:
    256 experts, top-8, Q3_K gate/up, Q4_K down, Q8_0 shared expert."""
    router = (_rng(seed, layer, S_ROUTER).standard_normal((n_experts, hidden))
              * router_std).astype(np.float32)
    lw = LayerWeights(
        hidden=hidden, inter=inter, n_experts=n_experts, top_k=top_k,
        gate_type=gate_type, up_type=up_type, down_type=down_type,
        gate=quant_tensor(_rng(seed, layer, S_GATE), gate_type, n_experts * inter, hidden),
        up=quant_tensor(_rng(seed, layer, S_UP), up_type, n_experts * inter, hidden),
        down=quant_tensor(_rng(seed, layer, S_DOWN), down_type, n_experts * hidden, inter),
        router=router,
        router_bias=zipf_bias(seed, layer, n_experts, zipf_s) if zipf_s else None,
        meta={"seed": seed, "layer": layer, "zipf_s": zipf_s, "router_std": router_std},
    )
    if shared_inter:
        g, u, d = shared_types
        lw.shared_inter = shared_inter
        lw.shared_types = tuple(shared_types)
        lw.shared_gate = quant_tensor(_rng(seed, layer, S_SH_GATE), g, shared_inter, hidden)
        lw.shared_up = quant_tensor(_rng(seed, layer, S_SH_UP), u, shared_inter, hidden)
        lw.shared_down = quant_tensor(_rng(seed, layer, S_SH_DOWN), d, hidden, shared_inter)
        lw.shared_gate_inp = (_rng(seed, layer, S_SH_INP).standard_normal(hidden)
                              * 0.02).astype(np.float32)
    return lw


def make_expert_q4k(seed: int = 0, hidden: int = 2048, inter: int = 512):
    """Single routed expert of the one-expert decode configuration: gate, up
    and down all Q4_K, plus one fp32 token ~ N(0, 1)."""
    tensors = {
        "gate": quant_tensor(_rng(seed, 0, S_GATE), Q4_K, inter, hidden),
        "up": quant_tensor(_rng(seed, 0, S_UP), Q4_K, inter, hidden),
        "down": quant_tensor(_rng(seed, 0, S_DOWN), Q4_K, hidden, inter),
    }
    x = make_tokens(seed, 1, hidden)[0]
    return tensors, {"gate": Q4_K, "up": Q4_K, "down": Q4_K}, x


def make_tokens(seed: int, count: int, hidden: int, stream: int = 0,
                dtype=np.float32) -> np.ndarray:
    """``count`` tokens ~ N(0, 1), shape (count, hidden)."""
    x = _rng(seed, 0, S_TOKENS + stream).standard_normal((count, hidden)).astype(np.float32)
    if dtype is not np.float32:
        x = x.astype(dtype)
    return x


def digest(*arrays: np.ndarray) -> str:
    """sha256 over the bytes of ``arrays``, to pin regenerated inputs."""
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).view(np.uint8).tobytes())
    return h.hexdigest()


S_DELTA_STATE, S_DELTA_STEP = 200, 201


def make_delta_state(seed: int, heads: int, key_dim: int, value_dim: int,
                     scale: float = 0.1) -> np.ndarray:
    """A DeltaNet recurrent state [heads, value_dim, key_dim] ~ N(0, scale)."""
    rng = _rng(seed, 0, S_DELTA_STATE)
    return (rng.standard_normal((heads, value_dim, key_dim)) * scale).astype(np.float32)


def make_delta_step(seed: int, step: int, heads: int, key_dim: int, value_dim: int):
    """Per-token DeltaNet inputs with the value ranges of the reference's
    caller (``src/flash_moe/gated_deltanet.py:340-386``): q and k L2-normalised
    per head, q scaled by 1/sqrt(key_dim), v ~ N(0, 1), beta = sigmoid(.) in
    (0, 1), gate = a log-decay <= 0 (decay = exp(gate) in (0, 1]).
    Returns (q, k, v, beta, gate) as float32 arrays."""
    rng = _rng(seed, step, S_DELTA_STEP)
    q = rng.standard_normal((heads, key_dim))
    k = rng.standard_normal((heads, key_dim))
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6) / np.sqrt(key_dim)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    v = rng.standard_normal((heads, value_dim))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal(heads)))
    gate = -np.log1p(np.exp(rng.standard_normal(heads))) * rng.uniform(0.05, 1.5, heads)
    return tuple(np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, beta, gate))
