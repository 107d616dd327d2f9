"""Expert execution backend for the B200.

Drop-in for the backend object the reference's MoE layer drives
(``OpenVINOExpertBackend``, ``src/flash_moe/backend_ov.py:91-431``): it has
``forward``, ``forward_batch``, ``prefetch_weights``, ``store``,
``_moe_executor``, ``begin_decode`` and ``begin_prefill`` with the same
arguments and results, so ``run_moe_layer`` / ``run_moe_sequence`` (the
reference's or ``flash_moe_b200.moe_layer``'s) work unchanged.  It adds
``forward_layer``: the whole layer (routing, the top-k experts, the weighted
sum and the shared expert) for a batch of tokens in one device call, which
``flash_moe_b200.moe_layer.run_moe_layer`` uses when present.

Weights never leave HBM; a call moves only the activations (8 KB per token
in, 8 KB out).
"""
from __future__ import annotations

import ctypes as C
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from . import _lib
from .key import ExpertKey
from .store import ExpertArena


def _host_ptr(a, np_dtype, torch_dtype, shape, what):
    """Address of a contiguous host buffer of `shape` (numpy array or CPU
    tensor), or None for None."""
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        if (a.dtype == torch_dtype and a.device.type == "cpu" and tuple(a.shape) == shape
                and a.is_contiguous()):
            return a.data_ptr()
    elif (isinstance(a, np.ndarray) and a.dtype == np_dtype and a.shape == shape
          and a.flags.c_contiguous):
        return a.ctypes.data
    raise ValueError(f"{what}: contiguous host {np.dtype(np_dtype)} array of shape {shape} needed")


class B200ExpertBackend:
    """Expert backend over an ``ExpertArena``.

    ``fp16_graph`` selects the reference native kernel's binary16 rounding
    (``cpp/moe_quant_dot.cpp:192-209``) for routed experts; the default is
    the fp32 arithmetic of ``fp16_graph=0``."""

    def __init__(self, arena: ExpertArena, expert_workers: int = 4,
                 fp16_graph: bool = False, exact: bool = False,
                 prefill_min_tokens: int | None = None):
        if expert_workers < 1:
            raise ValueError("thread and worker counts must be positive")
        self.lib = _lib.load()
        self.store = arena
        self.device = arena.device
        self.tensor_types = arena.tensor_types()
        self.fp16_graph = bool(fp16_graph)
        self.exact = bool(exact)
        self._moe_executor = ThreadPoolExecutor(max_workers=expert_workers)
        self._native_enabled = False
        self._tls = threading.local()
        # forward_layer uses the tensor-core prefill kernels from this many
        # tokens on (when the layer's shapes and formats allow it); None: for
        # every token count the single-launch decode kernels do not take
        self.prefill_min_tokens = None if prefill_min_tokens is None else int(prefill_min_tokens)

    # ---------------------------------------------------------------- policy

    def begin_decode(self):
        self._native_enabled = True

    def begin_prefill(self):
        self._native_enabled = False

    def prefetch_weights(self, keys):
        return self.store.prefetch_many(keys)

    def close(self):
        self._moe_executor.shutdown(wait=True)

    @property
    def flags(self) -> int:
        return (_lib.FP16_GRAPH if self.fp16_graph else 0) | (_lib.EXACT if self.exact else 0)

    # ------------------------------------------------------------ workspaces

    def _workspace(self, dl, tokens: int) -> torch.Tensor:
        cache = getattr(self._tls, "ws", None)
        if cache is None:
            cache = self._tls.ws = {}
        need = C.c_size_t(0)
        _lib.check(self.lib.moe_b200_decode_workspace(C.byref(dl.struct), tokens, C.byref(need)),
                   "moe_b200_decode_workspace")
        ws = cache.get(self.device)
        if ws is None or ws.numel() < need.value:
            ws = torch.zeros(max(need.value, 256), dtype=torch.uint8, device=self.device)
            cache[self.device] = ws
        return ws

    def _host_workspace(self, dl, tokens: int) -> torch.Tensor:
        cache = getattr(self._tls, "host_ws", None)
        if cache is None:
            cache = self._tls.host_ws = {}
        need = C.c_size_t(0)
        _lib.check(self.lib.moe_b200_decode_host_workspace(C.byref(dl.struct), tokens,
                                                           C.byref(need)),
                   "moe_b200_decode_host_workspace")
        ws = cache.get(self.device)
        if ws is None or ws.numel() < need.value:
            ws = torch.zeros(max(need.value, 256), dtype=torch.uint8, device=self.device)
            cache[self.device] = ws
        return ws

    def _prefill_workspace(self, s, tokens: int) -> torch.Tensor:
        cache = getattr(self._tls, "pf_ws", None)
        if cache is None:
            cache = self._tls.pf_ws = {}
        need = C.c_size_t(0)
        _lib.check(self.lib.moe_b200_prefill_workspace(C.byref(s), tokens, C.byref(need)),
                   "moe_b200_prefill_workspace")
        ws = cache.get(self.device)
        if ws is None or ws.numel() < need.value:
            ws = torch.zeros(max(need.value, 256), dtype=torch.uint8, device=self.device)
            cache[self.device] = ws
        return ws

    def prefill_supported(self, layer: int, flags: int | None = None) -> bool:
        """Whether the tensor-core prefill path takes this layer and flags."""
        s = self.store.layer(layer).with_flags(self.flags if flags is None else flags)
        return bool(self.lib.moe_b200_prefill_supported(C.byref(s)))

    def prefill_device(self, layer: int, x: torch.Tensor, y: torch.Tensor,
                       topk_ids: torch.Tensor | None = None,
                       topk_weights: torch.Tensor | None = None,
                       flags: int | None = None, stream=None) -> None:
        """Asynchronous many-token layer on the tensor cores: x fp32 or bf16
        [T, H], y fp32 [T, H] (``moe_b200_prefill``)."""
        dl = self.store.layer(layer)
        t = x.shape[0]
        s = dl.with_flags(self.flags if flags is None else flags)
        if x.dtype == torch.float32:
            xdt = 0
        elif x.dtype == torch.bfloat16:
            xdt = 1
        else:
            raise TypeError("prefill input must be fp32 or bf16")
        ws = self._prefill_workspace(s, t)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_prefill(
            C.byref(s), x.data_ptr(), xdt, t, y.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_weights.data_ptr() if topk_weights is not None else None,
            ws.data_ptr(), ws.numel(), stream.cuda_stream)
        _lib.check(st, "moe_b200_prefill")

    def prefill_errors(self) -> int:
        """Read and clear the device error word of this thread's prefill
        workspace (-9 wait timeout, -10 activation outside fp16)."""
        cache = getattr(self._tls, "pf_ws", None) or {}
        ws = cache.get(self.device)
        if ws is None:
            return 0
        err = C.c_int(0)
        _lib.check(self.lib.moe_b200_workspace_error(
            ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream, C.byref(err)),
            "moe_b200_workspace_error")
        return err.value

    def prefill_kernels(self, layer: int, tokens: int, flags: int | None = None) -> int:
        """Kernels one prefill_device call of `tokens` tokens launches (from
        the library)."""
        s = self.store.layer(layer).with_flags(self.flags if flags is None else flags)
        n = C.c_int(0)
        _lib.check(self.lib.moe_b200_prefill_kernels(C.byref(s), tokens, C.byref(n)),
                   "moe_b200_prefill_kernels")
        return n.value

    def uses_tensor_path(self, layer: int, tokens: int) -> bool:
        """Whether forward_layer runs these tokens on the tensor-core prefill
        path.  With the default threshold that is every token count the
        one-launch decode kernels (fused, multi-token) do not take: from there
        on the decode engine is four launches with a pass over the routed rows
        per token, 1.7-2.6x the tensor path's time for 9 to 31 tokens of a
        256-expert layer on a B200."""
        if not self.prefill_supported(layer):
            return False
        if self.prefill_min_tokens is not None:
            return tokens >= self.prefill_min_tokens
        return self.kernels_per_call(layer, tokens) > 1

    def kernels_per_call(self, layer: int, tokens: int, flags: int | None = None) -> int:
        """Kernels one forward_layer_device call launches (from the library)."""
        dl = self.store.layer(layer)
        s = dl.with_flags(self.flags if flags is None else flags)
        n = C.c_int(0)
        _lib.check(self.lib.moe_b200_decode_kernels(C.byref(s), tokens, C.byref(n)),
                   "moe_b200_decode_kernels")
        return n.value

    def device_errors(self) -> int:
        """Read and clear the device error word of this thread's workspace
        (-9 when a bounded wait inside a decode kernel gave up)."""
        cache = getattr(self._tls, "ws", None) or {}
        ws = cache.get(self.device)
        if ws is None:
            return 0
        err = C.c_int(0)
        _lib.check(self.lib.moe_b200_workspace_error(
            ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream, C.byref(err)),
            "moe_b200_workspace_error")
        return err.value

    # -------------------------------------------------------------- forward

    def forward_layer_device(self, layer: int, x: torch.Tensor, y: torch.Tensor,
                             topk_ids: torch.Tensor | None = None,
                             topk_weights: torch.Tensor | None = None,
                             flags: int | None = None, stream=None) -> None:
        """Asynchronous layer decode on device tensors: x, y fp32 [T, H]."""
        dl = self.store.layer(layer)
        t = x.shape[0]
        s = dl.with_flags(self.flags if flags is None else flags)
        ws = self._workspace(dl, t)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_decode(
            C.byref(s), x.data_ptr(), t, y.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_weights.data_ptr() if topk_weights is not None else None,
            ws.data_ptr(), ws.numel(), stream.cuda_stream)
        _lib.check(st, "moe_b200_decode")

    def _host_call(self, layer: int, flags: int, tokens: int):
        """(layer struct reference, workspace pointer, workspace bytes) of a
        moe_b200_decode_host call, cached per thread, layer object and flags."""
        cache = getattr(self._tls, "host_calls", None)
        if cache is None:
            cache = self._tls.host_calls = {}
        dl = self.store.layer(layer)
        key = (layer, flags, tokens)
        ent = cache.get(key)
        if ent is None or ent[0] is not dl:
            s = dl.with_flags(flags)
            ws = self._host_workspace(dl, tokens)
            ent = cache[key] = (dl, s, C.byref(s), ws, ws.data_ptr(), ws.numel())
        return ent

    def decode_host_ptrs(self, layer: int, x_ptr: int, tokens: int, y_ptr: int,
                         ids_ptr: int | None = None, w_ptr: int | None = None,
                         stream_handle: int = 0) -> None:
        """``moe_b200_decode_host`` on raw host addresses, like the reference's
        ctypes binding of moe_quant_expert (src/flash_moe/native_expert.py:23-37):
        the caller guarantees fp32 x / y rows of [tokens, H] (and int32 /
        fp32 [tokens, K] routing rows when given); `stream_handle` is a
        cudaStream_t (0: the legacy default stream)."""
        ent = self._host_call(layer, self.flags, tokens)
        st = self.lib.moe_b200_decode_host(ent[2], x_ptr, tokens, y_ptr, ids_ptr, w_ptr, ent[4],
                                           ent[5], stream_handle)
        if st:
            _lib.check(st, "moe_b200_decode_host")

    def forward_layer_host(self, layer: int, x, y, topk_ids=None, topk_weights=None,
                           flags: int | None = None, stream=None) -> None:
        """Synchronous layer decode with host buffers (``moe_b200_decode_host``):
        x and y fp32 [T, H], topk_ids int32 / topk_weights fp32 [T, K] when
        given -- numpy arrays or CPU tensors, pinned for asynchronous copies."""
        t = x.shape[0] if len(x.shape) == 2 else 0
        ent = self._host_call(layer, self.flags if flags is None else flags, t)
        w = ent[0].weights
        shp_x, shp_k = (t, w.hidden), (t, w.top_k)
        xp = _host_ptr(x, np.float32, torch.float32, shp_x, "x")
        yp = _host_ptr(y, np.float32, torch.float32, shp_x, "y")
        ip = _host_ptr(topk_ids, np.int32, torch.int32, shp_k, "topk_ids")
        wp = _host_ptr(topk_weights, np.float32, torch.float32, shp_k, "topk_weights")
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_decode_host(ent[2], xp, t, yp, ip, wp, ent[4], ent[5],
                                           stream.cuda_stream)
        if st:
            _lib.check(st, "moe_b200_decode_host")

    def ep_fused_supported(self, layer: int, tokens: int) -> bool:
        """True when ``decode_ep_device`` takes `tokens` gathered tokens of
        `layer` (the fused multi-token kernel: at most 8 tokens)."""
        if tokens < 2 or tokens > 8 or self.flags & (_lib.EXACT | _lib.FP16_GRAPH):
            return False
        return self.kernels_per_call(layer, tokens) == 1

    def decode_ep_device(self, layer: int, x: torch.Tensor, y: torch.Tensor, shared_begin: int,
                         shared_count: int, topk_ids: torch.Tensor | None = None,
                         topk_weights: torch.Tensor | None = None, stream=None) -> None:
        """One rank's expert-parallel step over the gathered tokens x [T, H]
        (``moe_b200_decode_ep``): the held routed experts of every token,
        and the shared expert of tokens [shared_begin, shared_begin +
        shared_count) only; y [T, H] is this rank's partial output."""
        dl = self.store.layer(layer)
        t = x.shape[0]
        s = dl.with_flags(self.flags)
        ws = self._workspace(dl, t)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_decode_ep(
            C.byref(s), x.data_ptr(), t, shared_begin, shared_count, y.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_weights.data_ptr() if topk_weights is not None else None,
            ws.data_ptr(), ws.numel(), stream.cuda_stream)
        _lib.check(st, "moe_b200_decode_ep")

    def decode_ep_p2p_device(self, layer: int, exchange, x: torch.Tensor, y: torch.Tensor,
                             topk_ids: torch.Tensor | None = None,
                             topk_weights: torch.Tensor | None = None, stream=None) -> None:
        """One expert-parallel step with dispatch and combine over peer
        memory (``moe_b200_decode_ep_p2p``): x, y [tokens_per_rank, H] are
        this rank's tokens; topk_ids / topk_weights [world * tokens_per_rank,
        K] receive the routing of every gathered token."""
        dl = self.store.layer(layer)
        s = dl.with_flags(self.flags)
        ws = self._workspace(dl, exchange.world * exchange.tokens_per_rank)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_decode_ep_p2p(
            C.byref(s), exchange.handle, x.data_ptr(), y.data_ptr(),
            topk_ids.data_ptr() if topk_ids is not None else None,
            topk_weights.data_ptr() if topk_weights is not None else None,
            ws.data_ptr(), ws.numel(), stream.cuda_stream)
        _lib.check(st, "moe_b200_decode_ep_p2p")

    # ---------------------------------------------------- multi-step decode

    def layer_table(self, layers) -> torch.Tensor:
        """Device copy of the ``moe_b200_layer`` structs of `layers` (cached
        per tuple of layer ids and flags)."""
        key = (tuple(layers), self.flags)
        cache = getattr(self, "_layer_tables", None)
        if cache is None:
            cache = self._layer_tables = {}
        t = cache.get(key)
        if t is None:
            raw = b"".join(bytes(self.store.layer(l).with_flags(self.flags)) for l in layers)
            t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
            cache[key] = t
        return t

    def step_table(self, steps) -> torch.Tensor:
        """Device array of ``moe_b200_step`` for `steps`, a list of
        (table index, flags, x, y, topk_ids, topk_weights) with device
        tensors (or None)."""
        arr = (_lib.Step * len(steps))()
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        for i, (li, fl, x, y, ids, w) in enumerate(steps):
            arr[i] = _lib.Step(li, fl, ptr(x), ptr(y), ptr(ids), ptr(w))
        return torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(self.device)

    def decode_steps_device(self, layer_table: torch.Tensor, step_table: torch.Tensor,
                            n_steps: int, layer0: int, eps: float = 1e-6, stream=None) -> None:
        """All steps of the tables in one launch (``moe_b200_decode_steps``)."""
        dl = self.store.layer(layer0)
        s = dl.with_flags(self.flags)
        ws = self._workspace(dl, 1)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        st = self.lib.moe_b200_decode_steps(C.byref(s), layer_table.data_ptr(),
                                            step_table.data_ptr(), n_steps, eps, ws.data_ptr(),
                                            ws.numel(), stream.cuda_stream)
        _lib.check(st, "moe_b200_decode_steps")

    def decode_stack(self, layers, x: torch.Tensor, y: torch.Tensor, eps: float = 1e-6) -> None:
        """One token through a stack of blocks with identity mixers (the
        40-layer configuration): h = x + rmsnorm16(x); out = h +
        f16(MoE(rmsnorm16(h))), layer after layer, in one launch."""
        H = x.shape[-1]
        tmp = torch.empty((2, H), dtype=torch.float32, device=self.device)
        steps = []
        for i, _ in enumerate(layers):
            out = y.view(-1) if i == len(layers) - 1 else tmp[i % 2]
            fl = _lib.STEP_BLOCK | (_lib.STEP_CHAIN if i else 0)
            steps.append((i, fl, x.view(-1) if i == 0 else None, out, None, None))
        lt = self.layer_table(layers)
        stt = self.step_table(steps)
        self.decode_steps_device(lt, stt, len(steps), layers[0], eps)
        self._keep = (tmp, stt)  # alive until the stream has run the launch

    def decode_stack_batch(self, layers, x: torch.Tensor, y: torch.Tensor, eps: float = 1e-6,
                           prefill: bool = True) -> None:
        """T tokens through the identity-mixer block stack: per layer
        moe_b200_block_prepare, the MoE layer (tensor-core prefill path, or
        the decode engines), moe_b200_block_finish."""
        T, H = x.shape
        dev = self.device
        h = torch.empty((T, H), dtype=torch.float32, device=dev)
        n = torch.empty_like(h)
        m = torch.empty_like(h)
        scratch = torch.empty_like(h)  # layer outputs between layers
        stream = torch.cuda.current_stream(dev).cuda_stream
        for i, layer in enumerate(layers):
            src = x if i == 0 else scratch
            dst = y if i == len(layers) - 1 else scratch
            _lib.check(self.lib.moe_b200_block_prepare(src.data_ptr(), h.data_ptr(), n.data_ptr(),
                                                       T, H, eps, stream), "moe_b200_block_prepare")
            if prefill:
                self.prefill_device(layer, n, m)
            else:
                self.forward_layer_device(layer, n, m)
            _lib.check(self.lib.moe_b200_block_finish(h.data_ptr(), m.data_ptr(), dst.data_ptr(),
                                                      T, H, stream), "moe_b200_block_finish")

    def forward_layer(self, layer: int, activations, return_routing: bool = False):
        """Whole MoE layer for T tokens (host arrays in, host array out)."""
        x = np.ascontiguousarray(activations, dtype=np.float32)
        squeeze = x.ndim == 1
        x = x.reshape(-1, self.store.layer(layer).weights.hidden)
        k = self.store.layer(layer).weights.top_k
        if not self.uses_tensor_path(layer, x.shape[0]):
            # decode: one synchronous call with the host arrays
            t = x.shape[0]
            y = np.empty_like(x)
            ids = np.empty((t, k), np.int32)
            w = np.empty((t, k), np.float32)
            with torch.cuda.device(self.device):
                self.forward_layer_host(layer, x, y, ids, w)
            y = y[0] if squeeze else y
            return (y, (ids, w)) if return_routing else y
        with torch.cuda.device(self.device):
            xd = torch.from_numpy(x).to(self.device, non_blocking=False)
            yd = torch.empty_like(xd)
            ids = torch.empty((x.shape[0], k), dtype=torch.int32, device=self.device)
            w = torch.empty((x.shape[0], k), dtype=torch.float32, device=self.device)
            self.prefill_device(layer, xd, yd, ids, w)
            err = self.prefill_errors()
            if err == -10:   # an activation outside fp16: fp32 engine instead
                self.forward_layer_device(layer, xd, yd, ids, w)
            elif err:
                _lib.check(err, "moe_b200_prefill")
            y = yd.cpu().numpy()
            routing = (ids.cpu().numpy(), w.cpu().numpy())
        y = y[0] if squeeze else y
        return (y, routing) if return_routing else y

    def forward(self, key: ExpertKey, activation, hidden_size: int,
                intermediate_size: int) -> np.ndarray:
        """One routed expert for one token (reference ``backend_ov.py:385-405``)."""
        dl = self.store.layer(key.layer)
        lw = dl.weights
        if hidden_size != lw.hidden or intermediate_size != lw.inter:
            raise ValueError("expert shape does not match the resident layer")
        views = dl.expert_views(key.expert)
        x = np.ascontiguousarray(activation, dtype=np.float32).reshape(-1)
        if x.size != hidden_size:
            raise ValueError("native expert activation shape mismatch")
        out = np.empty(hidden_size, np.float32)
        with torch.cuda.device(self.device):
            st = self.lib.moe_quant_expert(
                lw.gate_type, views["gate"].data_ptr(), views["gate"].numel(),
                lw.up_type, views["up"].data_ptr(), views["up"].numel(),
                lw.down_type, views["down"].data_ptr(), views["down"].numel(),
                x.ctypes.data, hidden_size, intermediate_size, out.ctypes.data,
                1 if self.fp16_graph else 0)
        _lib.check(st, "native expert")
        return out

    def forward_batch(self, key: ExpertKey, activations: np.ndarray, hidden_size: int,
                      intermediate_size: int) -> np.ndarray:
        """One expert for several tokens (reference ``backend_ov.py:407-431``)."""
        x = np.ascontiguousarray(activations, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != hidden_size:
            raise ValueError(f"expert activations must have shape (tokens, {hidden_size}), "
                             f"got {x.shape}")
        if x.shape[0] == 0:
            return np.empty((0, hidden_size), dtype=np.float32)
        return np.stack([self.forward(key, row, hidden_size, intermediate_size) for row in x])
