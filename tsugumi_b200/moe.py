"""Host-side mirror of the reference's MoE encoder classes over the C ABI.

The reference's Swift classes (Sources/Tsugumi/Kernels/MoE/MoE.swift,
Sources/Tsugumi/Kernels/Prefill/MoE/*.swift) encode Metal kernels into a
command buffer.  These classes keep their names and argument meaning and
call libtsugumi_cuda.so instead; buffers are torch CUDA tensors (device
memory only -- torch is plumbing here, no torch op computes the block).
Errors surface as exceptions named like the reference's thrown errors.
"""

from __future__ import annotations

import ctypes as C
import weakref
from dataclasses import dataclass

import numpy as np

from . import _abi
from ._abi import check

try:
    import torch
except ImportError:  # pragma: no cover - torch is present in this image
    torch = None


def _ptr(t) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("device tensor required")
    if not t.is_contiguous():
        raise ValueError("contiguous tensor required")
    return t.data_ptr()


class PrefillMoEGroupingError(Exception):
    """PrefillMoEGroupingError (PrefillMoEGrouping.swift:52-88)."""


class Context:
    """MetalContext analogue: device, stream, workspace and device error word."""

    def __init__(self, device: int = 0, stream=None):
        self.lib = _abi.load()
        self.device = device
        h = C.c_void_p()
        s = None if stream is None else C.c_void_p(stream.cuda_stream)
        check(self.lib.tsg_ctx_create(device, s, C.byref(h)))
        self.h = h
        self._layers = weakref.WeakSet()

    def set_stream(self, stream) -> None:
        check(self.lib.tsg_ctx_set_stream(self.h, C.c_void_p(stream.cuda_stream)), self.h)

    def set_decode_max_tokens(self, t: int) -> None:
        check(self.lib.tsg_ctx_set_decode_max_tokens(self.h, t), self.h)

    def set_option(self, name: str, value: int) -> None:
        check(self.lib.tsg_ctx_set_option(self.h, name.encode(), int(value)), self.h)

    def reserve(self, layer: "MoELayer", max_tokens: int) -> None:
        check(self.lib.tsg_ctx_reserve(self.h, layer.h, max_tokens), self.h)

    def sync(self) -> None:
        """checkCommandBufferError (MetalContext.swift:40-45) analogue."""
        st = self.lib.tsg_sync(self.h)
        if st == 7:
            raise PrefillMoEGroupingError(self.last_error())
        check(st, self.h)

    def last_error(self) -> str:
        raw = self.lib.tsg_last_error_string(self.h)
        return raw.decode() if raw else ""

    def close(self) -> None:
        if self.h:
            for layer in list(self._layers):
                layer.close()
            self.lib.tsg_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoELayer:
    """One layer's resident weights (device tensors) bound to a context."""

    def __init__(self, ctx: Context, t: dict, router_norm: bool = True, norm_eps: float = 1e-6,
                 effective_scale=None, per_expert_scale=None):
        self.ctx = ctx
        self.t = t  # keeps the tensors alive
        d = _abi.LayerDesc()
        d.d, d.f, d.num_experts, d.top_k = t["d"], t["f"], t["num_experts"], t["top_k"]
        d.group_size = 32
        d.activation = t["act"]
        d.experts = _ptr(t["experts"])
        d.expert_stride = t["expert_stride"]
        d.offsets = _abi.ExpertOffsets(*t["offsets"])
        self._router_w = t["router_w"].float().contiguous()
        d.router_weight = _ptr(self._router_w)
        self._eff = None if effective_scale is None else effective_scale.float().contiguous()
        d.effective_scale = _ptr(self._eff)
        self._pes = None if per_expert_scale is None else per_expert_scale.float().contiguous()
        d.per_expert_scale = _ptr(self._pes)
        self._bias = t.get("logit_bias")
        d.logit_bias = _ptr(self._bias)
        d.router_norm = 1 if router_norm else 0
        d.norm_eps = norm_eps
        if t.get("shared") is not None:
            d.shared_expert = _ptr(t["shared"])
            d.shared_f = t["shared_f"]
            d.shared_offsets = _abi.ExpertOffsets(*t["shared_offsets"])
            self._sg = t.get("shared_gate")
            if self._sg is not None:
                self._sg = self._sg.float().contiguous()
            d.shared_gate = _ptr(self._sg)
        self.desc = d
        h = C.c_void_p()
        check(ctx.lib.tsg_moe_layer_create(ctx.h, C.byref(d), C.byref(h)), ctx.h)
        self.h = h
        ctx._layers.add(self)
        self.d, self.f = t["d"], t["f"]
        self.num_experts, self.top_k = t["num_experts"], t["top_k"]

    def forward(self, hidden, y=None, residual=None, out_dtype=None):
        """tsg_moe_block_forward: the whole block."""
        T = hidden.shape[0]
        if y is None:
            y = torch.empty((T, self.d), dtype=out_dtype or torch.bfloat16, device=hidden.device)
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.ctx.lib.tsg_moe_block_forward(self.ctx.h, self.h, _ptr(hidden), hidden.stride(0),
                                                 T, _ptr(residual), _ptr(y), y.stride(0), dt),
              self.ctx.h)
        return y

    def gemma_ffn(self, hidden, attn, norms: dict, eps: float = 1e-6,
                  layer_scalar: float = 1.0):
        """tsg_gemma_ffn_forward: Gemma's layer FFN with the adjacent norms
        fused (fused_post_attn_setup / fused_layer_tail, fused.metal:190-374);
        `hidden` (bf16 [T, D]) is updated in place.  `norms` holds bf16 [D]
        tensors post_attn, pre_ffn, pre_ffn2, post_dense, post_routed,
        post_ffn.  The layer is created with router_norm=False."""
        keys = ("post_attn", "pre_ffn", "pre_ffn2", "post_dense", "post_routed", "post_ffn")
        w = {k: norms[k].to(torch.bfloat16).contiguous() for k in keys}
        n = _abi.GemmaNorms(*[_ptr(w[k]) for k in keys], float(eps), float(layer_scalar))
        check(self.ctx.lib.tsg_gemma_ffn_forward(self.ctx.h, self.h, C.byref(n), _ptr(hidden),
                                                 hidden.stride(0), _ptr(attn), attn.stride(0),
                                                 hidden.shape[0]),
              self.ctx.h)
        self._gemma_norms = w  # alive until the stream has used them
        return hidden

    def verify_rows(self, hidden, y=None, residual=None, out_dtype=None):
        """tsg_moe_verify_rows_forward: a speculative-verify block, each row
        bit-equal to forward() on that row alone (PrefillGroupedRoutedMoE
        .encodeStreamedRows, PrefillGroupedRoutedMoE.swift:768-800)."""
        T = hidden.shape[0]
        if y is None:
            y = torch.empty((T, self.d), dtype=out_dtype or torch.bfloat16, device=hidden.device)
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.ctx.lib.tsg_moe_verify_rows_forward(self.ctx.h, self.h, _ptr(hidden),
                                                       hidden.stride(0), T, _ptr(residual),
                                                       _ptr(y), y.stride(0), dt),
              self.ctx.h)
        return y

    def close(self) -> None:
        if self.h:
            self.ctx.lib.tsg_moe_layer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MoE:
    """MoE (Sources/Tsugumi/Kernels/MoE/MoE.swift:42): decode router and
    routed phases for one layer."""

    def __init__(self, context: Context, layer: MoELayer):
        self.context, self.layer = context, layer

    def encode_router_gemma4_bf16(self, hidden, out_indices, out_weights, out_weights_f16=None):
        """encodeRouterGemma4BF16 / ...Rows (MoE.swift:259-302, :413-466)."""
        T = hidden.shape[0]
        check(self.context.lib.tsg_router_topk(self.context.h, self.layer.h, _ptr(hidden),
                                               hidden.stride(0), T, _ptr(out_indices),
                                               _ptr(out_weights), _ptr(out_weights_f16)),
              self.context.h)

    def encode_router_logits_bf16(self, hidden, out_logits):
        """encodeRouterLogitsBF16 (MoE.swift:316-345): the router's fp32
        logits [T, E] alone, no selection."""
        T = hidden.shape[0]
        check(self.context.lib.tsg_router_logits(self.context.h, self.layer.h, _ptr(hidden),
                                                 hidden.stride(0), T, _ptr(out_logits)),
              self.context.h)

    def encode_routed_phases(self, x, indices, routing_weights, y, residual=None):
        """encodeRoutedPersistentPhase1U16Load + encodeRoutedPersistentPhase2Reduce
        (MoE.swift:529-644) for caller-supplied routing."""
        T = x.shape[0]
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.context.lib.tsg_moe_experts_decode(self.context.h, self.layer.h, _ptr(x),
                                                      x.stride(0), T, _ptr(indices),
                                                      _ptr(routing_weights), _ptr(residual),
                                                      _ptr(y), y.stride(0), dt),
              self.context.h)


class PrefillRouter:
    """PrefillRouter (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillRouter.swift:30)."""

    def __init__(self, context: Context, layer: MoELayer):
        self.context, self.layer = context, layer

    def encode_gemma4_bf16_gemm(self, hidden, out_indices, out_weights, out_weights_f16=None):
        MoE(self.context, self.layer).encode_router_gemma4_bf16(hidden, out_indices, out_weights,
                                                                out_weights_f16)

    encode_gemma4_bf16_block = encode_gemma4_bf16_gemm

    @staticmethod
    def make_token_expert_pairs(context: Context, indices, weights_f16, query_count: int,
                                top_k: int):
        """makeTokenExpertPairs (PrefillRouter.swift:238-258): int32 [T*K, 4]."""
        out = torch.empty((query_count * top_k, 4), dtype=torch.int32, device=indices.device)
        check(context.lib.tsg_make_token_expert_pairs(context.h, _ptr(indices), _ptr(weights_f16),
                                                      query_count, top_k, _ptr(out)), context.h)
        return out


@dataclass
class PrefillMoEGroupedRoutes:
    """PrefillMoEGroupedRoutes (PrefillMoEGrouping.swift:32-50), host copies."""

    sorted_pairs: np.ndarray       # [n, 4] (token, expert, rank, weight bits)
    per_expert_offsets: np.ndarray
    per_expert_counts: np.ndarray
    groups: np.ndarray             # [g, 3] (expert, pair_start, pair_count)
    tiles: np.ndarray              # [t, 4]
    query_count: int

    @property
    def max_pairs_per_expert(self) -> int:
        return int(self.groups[:, 2].max()) if len(self.groups) else 0

    @property
    def max_pairs_per_tile(self) -> int:
        return int(self.tiles[:, 3].max()) if len(self.tiles) else 0

    @property
    def max_live_experts_per_tile(self) -> int:
        return int(self.tiles[:, 1].max()) if len(self.tiles) else 0


class PrefillMoEGrouping:
    """PrefillMoEGrouping (PrefillMoEGrouping.swift:90): the permutation, on
    the GPU."""

    @staticmethod
    def group_token_expert_pairs(context: Context, pairs, query_count: int, top_k: int,
                                 num_experts: int, tile_expert_count: int = 16,
                                 expert_sort_keys=None, tile_break_after_group=None):
        n = 0 if pairs is None else int(pairs.shape[0])
        dev = torch.device("cuda", context.device)
        ne = max(num_experts, 1)
        sorted_pairs = torch.zeros((max(n, 1), 4), dtype=torch.int32, device=dev)
        offsets = torch.zeros(ne, dtype=torch.int32, device=dev)
        counts = torch.zeros(ne, dtype=torch.int32, device=dev)
        groups = torch.zeros((ne, 3), dtype=torch.int32, device=dev)
        tiles = torch.zeros((ne, 4), dtype=torch.int32, device=dev)
        ng = torch.zeros(1, dtype=torch.int32, device=dev)
        nt = torch.zeros(1, dtype=torch.int32, device=dev)
        keys = None
        if expert_sort_keys is not None:
            keys = torch.as_tensor(np.asarray(expert_sort_keys, np.uint64).view(np.int64),
                                   device=dev)
        st = context.lib.tsg_moe_group_pairs(
            context.h, _ptr(pairs) if n else None, n, query_count, top_k, num_experts,
            tile_expert_count, _ptr(keys), 0 if keys is None else int(keys.numel()),
            -1 if tile_break_after_group is None else tile_break_after_group,
            _ptr(sorted_pairs), _ptr(offsets), _ptr(counts), _ptr(groups), _ptr(ng), _ptr(tiles),
            _ptr(nt))
        if st == 1:
            raise PrefillMoEGroupingError(context.last_error())
        check(st, context.h)
        context.sync()  # per-pair validation errors surface here
        g = int(ng.item())
        t = int(nt.item())
        as_u32 = lambda a: a.cpu().numpy().view(np.uint32)
        return PrefillMoEGroupedRoutes(
            sorted_pairs=as_u32(sorted_pairs[:n]), per_expert_offsets=as_u32(offsets[:num_experts]),
            per_expert_counts=as_u32(counts[:num_experts]), groups=as_u32(groups[:g]),
            tiles=as_u32(tiles[:t]), query_count=query_count)


class PrefillRoutedGEMMPlanner:
    """PrefillRoutedGEMMPlanner (PrefillGroupedRoutedMoE.swift:42-83), host."""

    tile_rows = 64

    @staticmethod
    def plan(groups: np.ndarray, max_rows_per_batch: int, tile_rows: int = 64):
        lib = _abi.load()
        groups = np.ascontiguousarray(np.asarray(groups, np.uint32).reshape(-1, 3))
        ng = groups.shape[0]
        cap = int(groups[:, 2].sum()) + ng + 4 if ng else 4
        blocks = np.zeros((cap, 4), np.uint32)
        rows = np.zeros(cap, np.uint32)
        first = np.zeros(cap, np.uint32)
        cnt = np.zeros(cap, np.uint32)
        nb, nbatch = C.c_uint32(), C.c_uint32()
        gp = groups.ctypes.data_as(C.c_void_p) if ng else None
        check(lib.tsg_plan_routed_gemm(gp, ng, max_rows_per_batch, tile_rows,
                                       blocks.ctypes.data_as(C.c_void_p), cap, C.byref(nb),
                                       rows.ctypes.data_as(C.c_void_p),
                                       first.ctypes.data_as(C.c_void_p),
                                       cnt.ctypes.data_as(C.c_void_p), cap, C.byref(nbatch)))
        return [{"rows": int(rows[i]), "blocks": blocks[first[i]:first[i] + cnt[i]]}
                for i in range(nbatch.value)]


class PrefillGroupedRoutedMoE:
    """PrefillGroupedRoutedMoE (PrefillGroupedRoutedMoE.swift:414): grouped
    routed experts for caller-supplied routing, on tcgen05."""

    def __init__(self, context: Context, layer: MoELayer):
        self.context, self.layer = context, layer

    def encode_streamed_tiled(self, x, indices, routing_weights, y, residual=None):
        T = x.shape[0]
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.context.lib.tsg_moe_experts_prefill(self.context.h, self.layer.h, _ptr(x),
                                                       x.stride(0), T, _ptr(indices),
                                                       _ptr(routing_weights), _ptr(residual),
                                                       _ptr(y), y.stride(0), dt),
              self.context.h)


class PrefillMoE:
    """PrefillMoE (PrefillMoE.swift:1-40)."""

    @staticmethod
    def encode_reduce_token_major(context: Context, route_partials, route_weights, h2):
        T, K = route_weights.shape
        D = route_partials.shape[-1]
        dt = _abi.DTYPE_F32 if h2.dtype == torch.float32 else _abi.DTYPE_F16
        check(context.lib.tsg_moe_reduce_token_major(context.h, _ptr(route_partials),
                                                     _ptr(route_weights), T, K, D, _ptr(h2), dt),
              context.h)


class SharedExpertRuntime:
    """SharedExpertRuntime (SharedExpertInt4.swift:115-136) plus the Qwen
    sigmoid gate (QwenKernels.encodeMoESharedGate, QwenKernels.swift:311-355)."""

    def __init__(self, context: Context, layer: MoELayer):
        self.context, self.layer = context, layer

    def encode(self, x, y):
        T = x.shape[0]
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.context.lib.tsg_shared_expert(self.context.h, self.layer.h, _ptr(x),
                                                 x.stride(0), T, _ptr(y), y.stride(0), dt),
              self.context.h)


def last_routing(context: Context):
    lib = _abi.load()
    ids, w, sp = C.c_void_p(), C.c_void_p(), C.c_void_p()
    T, K = C.c_uint32(), C.c_uint32()
    check(lib.tsg_last_routing(context.h, C.byref(ids), C.byref(w), C.byref(sp), C.byref(T),
                               C.byref(K)), context.h)
    return ids.value, w.value, sp.value, T.value, K.value
