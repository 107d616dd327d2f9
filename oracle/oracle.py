"""CPU oracle for the routed-expert MoE hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference legs may import this module, and only
to check or time against; the shipped package never imports it.

Two layers:

* ``KQuantOracle`` -- ctypes binding of ``libkquant_oracle.so`` (the scalar C
  restatement of ``cpp/dequant_k.cpp`` and ``cpp/moe_quant_dot.cpp`` in
  ``kquant_oracle.c``), plus ``ReferenceLibrary`` for the reference's own
  sources compiled in place into ``_ref/`` (``make ref``).
* numpy restatements of the Python MoE layer the native kernel sits in:
  ``route`` (``src/flash_moe/router.py:140-170``), ``run_moe_layer``
  (``src/flash_moe/moe_layer.py:39-107``), ``run_moe_sequence``
  (``moe_layer.py:110-195``), the shared expert (``shared_expert.py:200-251``)
  and RMSNorm (``norm.py:21-30``).  They perform the same numpy operations in
  the same order, so on one host they give the reference's bits.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "libkquant_oracle.so"
REF_LIB = HERE / "_ref" / "libmoe_quant_dot_ref.so"

Q8_0, Q3_K, Q4_K, Q5_K, Q6_K = 8, 11, 12, 13, 14
BLOCK = {Q8_0: (32, 34), Q3_K: (256, 110), Q4_K: (256, 144),
         Q5_K: (256, 176), Q6_K: (256, 210)}


def build_oracle(force: bool = False) -> Path:
    """Compile ``libkquant_oracle.so`` with the committed Makefile if absent."""
    if force or not ORACLE_LIB.exists():
        subprocess.run(["make", "-C", str(HERE), "libkquant_oracle.so"],
                       check=True, capture_output=True)
    return ORACLE_LIB


def reference_root() -> Path:
    """The reference checkout: ``$FLASH_MOE_REFERENCE_ROOT``, else a sibling
    directory ``reference`` of this repository."""
    env = os.environ.get("FLASH_MOE_REFERENCE_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"


def build_reference(ref_root: str | Path | None = None) -> Path | None:
    """Compile the reference's own ``cpp/moe_quant_dot.cpp`` into ``_ref/``.

    Returns None when the reference sources are not present (GPU boxes only
    carry the already-built library)."""
    if REF_LIB.exists():
        return REF_LIB
    ref_root = reference_root() if ref_root is None else ref_root
    if not (Path(ref_root) / "cpp" / "moe_quant_dot.cpp").exists():
        return None
    subprocess.run(["make", "-C", str(HERE), "ref", f"REF={ref_root}"],
                   check=True, capture_output=True)
    return REF_LIB


def _bind(lib: C.CDLL, dequant: str, expert: str):
    fd = getattr(lib, dequant)
    fd.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_int]
    fd.restype = C.c_int
    fe = getattr(lib, expert)
    fe.argtypes = [C.c_int, C.c_void_p, C.c_int64] * 3 + [
        C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
    fe.restype = C.c_int
    return fd, fe


class _KQuantLib:
    """Common numpy-facing wrapper over a library with the reference ABI."""

    def __init__(self, path: Path, dequant: str, expert: str, delta: str):
        self.path = Path(path)
        self.lib = C.CDLL(str(self.path))
        self._dequant, self._expert = _bind(self.lib, dequant, expert)
        self._delta = getattr(self.lib, delta)
        self._delta.argtypes = [C.c_void_p] * 7 + [C.c_int] * 3
        self._delta.restype = C.c_int

    def dequant(self, type_id: int, raw: np.ndarray, n: int | None = None,
                want_f16: bool = False) -> tuple[int, np.ndarray]:
        raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
        bs, pb = BLOCK.get(type_id, (1, 1))
        if n is None:
            n = raw.size // pb * bs
        out = np.zeros(max(n, 1), np.uint16 if want_f16 else np.float32)
        rc = self._dequant(type_id, raw.ctypes.data, out.ctypes.data, n, int(want_f16))
        return rc, (out.view(np.float16) if want_f16 else out)

    def expert(self, tensors: dict, kinds: dict, x: np.ndarray, hidden: int,
               intermediate: int, fp16_graph: int = 0) -> tuple[int, np.ndarray]:
        arrays = [np.ascontiguousarray(np.frombuffer(tensors[k], np.uint8)
                                       if isinstance(tensors[k], (bytes, bytearray))
                                       else tensors[k], dtype=np.uint8).reshape(-1)
                  for k in ("gate", "up", "down")]
        args = []
        for name, raw in zip(("gate", "up", "down"), arrays):
            args.extend((kinds[name], raw.ctypes.data, raw.nbytes))
        xv = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.full(hidden, np.nan, np.float32)
        rc = self._expert(*args, xv.ctypes.data, hidden, intermediate,
                          out.ctypes.data, fp16_graph)
        return rc, out

    def delta_heads(self, state: np.ndarray, q, k, v, beta, gate,
                    out: np.ndarray | None = None) -> tuple[int, np.ndarray]:
        """One DeltaNet step in place on ``state`` [heads, value_dim, key_dim]
        (``cpp/moe_delta.cpp:18-69``).  ``out`` [heads, value_dim] defaults to
        NaN so rows the call does not write are visible."""
        if state.dtype != np.float32 or not state.flags.c_contiguous:
            raise ValueError("state must be contiguous float32")
        heads, dv, dk = state.shape
        arrays = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, beta, gate)]
        if out is None:
            out = np.full((heads, dv), np.nan, np.float32)
        rc = self._delta(state.ctypes.data, *(a.ctypes.data for a in arrays),
                         out.ctypes.data, heads, dk, dv)
        return rc, out


class KQuantOracle(_KQuantLib):
    """The scalar C restatement (``kquant_oracle.c``)."""

    def __init__(self, path: Path | None = None):
        super().__init__(path or build_oracle(), "kq_dequant", "kq_expert",
                         "kq_delta_heads")


class ReferenceLibrary(_KQuantLib):
    """The reference's own AVX2 sources, compiled here (``make ref``)."""

    def __init__(self, path: Path | None = None):
        path = path or REF_LIB
        if not Path(path).exists():
            raise FileNotFoundError(f"reference library not built: {path}")
        super().__init__(path, "dequant_k", "moe_quant_expert", "moe_delta_heads")


# ---------------------------------------------------------------- numpy layer

def route(x: np.ndarray, gate_he: np.ndarray, top_k: int, bias: np.ndarray | None = None):
    """Top-k ids and softmax weights of one token.

    Restates ``ExpertRouter.scores/route`` (``src/flash_moe/router.py:140-170``):
    fp32 ``x @ W`` with W laid out (hidden, experts), ``argsort`` ascending,
    the last k reversed, a float64 softmax over those k only.  ``bias`` (an
    fp32 per-expert logit offset, the popularity skew of the batched-decode
    benchmark; the reference router has none) is added to the fp32 scores."""
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    scores = (x @ np.asarray(gate_he, dtype=np.float32)).astype(np.float32)
    if bias is not None:
        scores = (scores + np.asarray(bias, dtype=np.float32)).astype(np.float32)
    ids = np.argsort(scores)[-top_k:][::-1].astype(np.int64).tolist()
    top = scores[ids].astype(np.float64)
    e = np.exp(top - np.max(top))
    total = e.sum()
    if not np.isfinite(total) or total <= 0.0:
        w = np.full(len(ids), 1.0 / len(ids))
    else:
        w = e / total
    return ids, [float(v) for v in w], scores


def sigmoid(x: np.ndarray) -> np.ndarray:
    """Restates ``_sigmoid`` (``src/flash_moe/shared_expert.py:55-62``)."""
    out = np.empty_like(x)
    pos = x >= 0
    out[pos] = 1.0 / (1.0 + np.exp(-x[pos]))
    e = np.exp(x[~pos])
    out[~pos] = e / (1.0 + e)
    return out


def shared_forward(x: np.ndarray, w: dict) -> np.ndarray:
    """Restates ``SharedExpert.forward`` (``shared_expert.py:221-251``).

    ``w`` holds fp32 arrays ``gate_inp`` [H], ``gate``/``up`` [I, H] and
    ``down`` [H, I] (the reference keeps them as fp16-rounded values promoted
    to fp32, ``shared_expert.py:157-195 and the fp32 views at :242-249``)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    gate = sigmoid((x @ np.asarray(w["gate_inp"], dtype=np.float32)).reshape(()))
    g = x @ np.asarray(w["gate"], dtype=np.float32).T
    act = (g * sigmoid(g)) * (x @ np.asarray(w["up"], dtype=np.float32).T)
    out = act @ np.asarray(w["down"], dtype=np.float32).T
    return (gate * out).astype(np.float32)


def shared_forward_batch(x: np.ndarray, w: dict) -> np.ndarray:
    """Restates ``SharedExpert.forward_batch`` (``shared_expert.py:200-219``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gate = sigmoid(x @ np.asarray(w["gate_inp"], dtype=np.float32).reshape(-1))
    g = x @ np.asarray(w["gate"], dtype=np.float32).T
    u = x @ np.asarray(w["up"], dtype=np.float32).T
    out = ((g * sigmoid(g)) * u) @ np.asarray(w["down"], dtype=np.float32).T
    return (out * gate[:, None]).astype(np.float32)


def shared_weights_from_packed(lib: _KQuantLib, packed: dict, kinds: dict,
                               hidden: int, inter: int, gate_inp) -> dict:
    """fp32 shared-expert weights as the reference loads them: dequantised to
    binary16 by ``dequant_k(..., want_f16=1)`` then promoted to fp32
    (``shared_expert.py:157-195`` and the fp32 views at ``:242-249``)."""
    shapes = {"gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
    out = {"gate_inp": np.asarray(gate_inp, dtype=np.float32).reshape(-1)}
    for role, shape in shapes.items():
        rc, v = lib.dequant(kinds[role], packed[role], shape[0] * shape[1], want_f16=True)
        if rc != 0:
            raise RuntimeError(f"dequant of shared {role} failed: {rc}")
        out[role] = np.ascontiguousarray(v.astype(np.float32).reshape(shape))
    return out


def run_moe_layer(x, gate_he, top_k, expert_fn, shared=None, workers: int = 4,
                  selection=None, bias=None):
    """One token through one MoE layer.

    Restates ``run_moe_layer`` (``src/flash_moe/moe_layer.py:39-107``): the k
    experts run on a thread pool, ``combined += weight * out`` in top-k order
    in fp32, then ``combined + shared_out``.  ``expert_fn(expert_id, x)``
    returns the expert's fp32 output.  ``selection`` optionally forces the
    (ids, weights) pair, used when the device's routing resolved a near tie
    differently.  Returns (y, ids, weights)."""
    if selection is None:
        ids, weights, _ = route(x, gate_he, top_k, bias)
    else:
        ids, weights = selection
    combined = np.zeros(np.asarray(x).size, dtype=np.float32)
    if workers > 1 and len(ids) > 1:
        with ThreadPoolExecutor(max_workers=workers) as pool:
            outs = list(pool.map(lambda e: expert_fn(e, x), ids))
    else:
        outs = [expert_fn(e, x) for e in ids]
    for out, w in zip(outs, weights):
        combined += w * np.asarray(out, dtype=np.float32)
    if shared is not None:
        combined = combined + shared_forward(x, shared)
    return combined, ids, weights


def run_moe_sequence(xs, gate_he, top_k, expert_fn, shared=None):
    """Many tokens through one MoE layer, grouped by expert.

    Restates ``run_moe_sequence`` (``moe_layer.py:110-195``) for a backend
    whose batched call equals its per-token call: per-token weighted sums in
    slot order, shared expert batched for 16..128 tokens, per token otherwise."""
    xs = np.asarray(xs, dtype=np.float32)
    t = xs.shape[0]
    outs = np.empty((t, top_k, xs.shape[1]), np.float32)
    routed = []
    for i in range(t):
        ids, w, _ = route(xs[i], gate_he, top_k)
        routed.append((ids, w))
        for slot, e in enumerate(ids):
            outs[i, slot] = expert_fn(e, xs[i])
    batch_shared = shared is not None and 16 <= t <= 128
    result = np.zeros_like(xs)
    for i, (ids, w) in enumerate(routed):
        for slot, wk in enumerate(w):
            result[i] += wk * outs[i, slot]
        if shared is not None and not batch_shared:
            result[i] += shared_forward(xs[i], shared)
    if batch_shared:
        result += shared_forward_batch(xs, shared)
    return result, routed


def rmsnorm_f16(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm with unit weight: fp32 reduction, binary16 output.

    Restates ``RMSNorm.forward`` (``src/flash_moe/norm.py:28-30``) with the
    weight fixed to 1."""
    x32 = np.ascontiguousarray(x, dtype=np.float32)
    rms = np.sqrt(np.mean(x32 * x32, axis=-1, keepdims=True) + eps)
    return ((x32 / rms) * np.float32(1.0)).astype(np.float16)


def stack_block(x: np.ndarray, moe_fn, eps: float = 1e-6) -> np.ndarray:
    """One block of the identity-mixer stack, decode of one token.

    Restates ``TransformerBlock.forward`` (``src/flash_moe/transformer.py:
    229-247``) with the mixer replaced by identity: ``h = x + norm(x)``,
    ``out = h + moe(norm2(h))``.  In decode ``_moe_forward`` stores the MoE
    output into an array shaped like its binary16 input (``:192-204``), so the
    MoE output is rounded to binary16 before the residual add."""
    x = np.asarray(x, dtype=np.float32)
    h = x + rmsnorm_f16(x, eps)
    n2 = rmsnorm_f16(h, eps)
    moe = np.asarray(moe_fn(n2.astype(np.float32)), dtype=np.float32).astype(np.float16)
    return h + moe


def max_relative_error(actual: np.ndarray, reference: np.ndarray) -> float:
    """``max|a - r| / max|r|`` (``src/flash_moe/dequant.py:198-202``)."""
    reference = np.asarray(reference, dtype=np.float64)
    scale = float(np.abs(reference).max()) if reference.size else 0.0
    if scale == 0.0:
        return float(np.abs(actual).max()) if np.asarray(actual).size else 0.0
    return float(np.abs(np.asarray(actual, dtype=np.float64) - reference).max() / scale)
