"""ctypes bindings of libtsugumi_cuda.so (include/tsugumi_cuda.h).

The library is built in-tree by tsugumi_b200/build.py.  Loading fails with an
ImportError-like RuntimeError when it is missing: there is no fallback path.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtsugumi_cuda.so"

TSG_OK = 0
STATUS_NAMES = {
    0: "TSG_OK",
    1: "TSG_ERR_INVALID_ARG",
    2: "TSG_ERR_UNSUPPORTED_SHAPE",
    3: "TSG_ERR_OOM",
    4: "TSG_ERR_CUDA",
    5: "TSG_ERR_NCCL",
    6: "TSG_ERR_TIMEOUT",
    7: "TSG_ERR_METADATA",
}

DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2
ACT_GELU_TANH, ACT_SILU = 0, 1


class ExpertOffsets(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "gate_w_off", "gate_s_off", "gate_b_off", "up_w_off", "up_s_off", "up_b_off",
        "down_w_off", "down_s_off", "down_b_off")]


class TokenExpertPair(C.Structure):
    _fields_ = [("token", C.c_uint32), ("expert", C.c_uint32), ("rank", C.c_uint32),
                ("weight_bits_and_reserved", C.c_uint32)]


class MoEGroup(C.Structure):
    _fields_ = [("expert", C.c_uint32), ("pair_start", C.c_uint32), ("pair_count", C.c_uint32)]


class MoETile(C.Structure):
    _fields_ = [("group_start", C.c_uint32), ("group_count", C.c_uint32),
                ("pair_start", C.c_uint32), ("pair_count", C.c_uint32)]


class RoutedGemmBlock(C.Structure):
    _fields_ = [("local_slot", C.c_uint32), ("pair_start", C.c_uint32),
                ("row_count", C.c_uint32), ("local_row", C.c_uint32)]


class LayerDesc(C.Structure):
    _fields_ = [
        ("d", C.c_uint32), ("f", C.c_uint32), ("num_experts", C.c_uint32),
        ("top_k", C.c_uint32), ("group_size", C.c_uint32), ("activation", C.c_int),
        ("experts", C.c_void_p), ("expert_stride", C.c_uint64), ("offsets", ExpertOffsets),
        ("router_weight", C.c_void_p), ("effective_scale", C.c_void_p),
        ("per_expert_scale", C.c_void_p), ("logit_bias", C.c_void_p),
        ("router_norm", C.c_uint32), ("norm_eps", C.c_float),
        ("shared_expert", C.c_void_p), ("shared_f", C.c_uint32),
        ("shared_offsets", ExpertOffsets), ("shared_gate", C.c_void_p),
    ]


# (name, restype, argtypes) for every symbol the header declares.
class GemmaNorms(C.Structure):
    _fields_ = [("post_attn", C.c_void_p), ("pre_ffn", C.c_void_p), ("pre_ffn2", C.c_void_p),
                ("post_dense", C.c_void_p), ("post_routed", C.c_void_p),
                ("post_ffn", C.c_void_p), ("eps", C.c_float), ("layer_scalar", C.c_float)]


_P = C.c_void_p
_U = C.c_uint32
_I = C.c_int32
_S = C.c_int
SIGNATURES = [
    ("tsg_abi_version", C.c_int, []),
    ("tsg_ctx_create", _S, [C.c_int, _P, C.POINTER(_P)]),
    ("tsg_ctx_destroy", _S, [_P]),
    ("tsg_ctx_set_stream", _S, [_P, _P]),
    ("tsg_ctx_set_decode_max_tokens", _S, [_P, _U]),
    ("tsg_ctx_set_option", _S, [_P, C.c_char_p, C.c_int64]),
    ("tsg_ctx_reserve", _S, [_P, _P, _U]),
    ("tsg_sync", _S, [_P]),
    ("tsg_last_error_string", C.c_char_p, [_P]),
    ("tsg_moe_layer_create", _S, [_P, C.POINTER(LayerDesc), C.POINTER(_P)]),
    ("tsg_moe_layer_destroy", _S, [_P]),
    ("tsg_moe_block_forward", _S, [_P, _P, _P, _U, _U, _P, _P, _U, C.c_int]),
    ("tsg_moe_verify_rows_forward", _S, [_P, _P, _P, _U, _U, _P, _P, _U, C.c_int]),
    ("tsg_router_topk", _S, [_P, _P, _P, _U, _U, _P, _P, _P]),
    ("tsg_router_logits", _S, [_P, _P, _P, _U, _U, _P]),
    ("tsg_make_token_expert_pairs", _S, [_P, _P, _P, _U, _U, _P]),
    ("tsg_moe_group_pairs", _S, [_P, _P, _U, _I, _I, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P,
                                 _P, _P]),
    ("tsg_moe_group_pairs_noalloc", _S, [_P, _P, _U, _I, _I, _I, _I, _P, _I, _I, _P, _P, _P,
                                         _P, _P, _P, _P]),
    ("tsg_ep_unique_id", _S, [_P]),
    ("tsg_ep_init", _S, [_P, _P, C.c_int, C.c_int]),
    ("tsg_ep_moe_block_forward", _S, [_P, _P, _U, _P, _U, _U, _P, _P, _U, C.c_int]),
    ("tsg_ep_phase_ms", _S, [_P, _P, C.c_int]),
    ("tsg_plan_routed_gemm", _S, [_P, _U, _U, _U, _P, _U, C.POINTER(_U), _P, _P, _P, _U,
                                  C.POINTER(_U)]),
    ("tsg_moe_experts_decode", _S, [_P, _P, _P, _U, _U, _P, _P, _P, _P, _U, C.c_int]),
    ("tsg_moe_experts_prefill", _S, [_P, _P, _P, _U, _U, _P, _P, _P, _P, _U, C.c_int]),
    ("tsg_moe_reduce_token_major", _S, [_P, _P, _P, _U, _U, _U, _P, C.c_int]),
    ("tsg_shared_expert", _S, [_P, _P, _P, _U, _U, _P, _U, C.c_int]),
    ("tsg_import_int4_affine", _S, [_P, _P, _P, _P, _U, _U, _U, _P, _P]),
    ("tsg_gemma_ffn_forward", _S, [_P, _P, C.POINTER(GemmaNorms), _P, _U, _P, _U, _U]),
    ("tsg_ctx_profile_begin", _S, [_P, _U]),
    ("tsg_ctx_profile_end", _S, [_P, C.POINTER(C.c_float), C.POINTER(_U)]),
    ("tsg_last_routing", _S, [_P, C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_U),
                              C.POINTER(_U)]),
]

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Loads the library (building nothing); raises if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m tsugumi_b200.build` "
                "(the MoE block has no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class TsgError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


def check(status: int, ctx=None) -> None:
    if status != TSG_OK:
        msg = ""
        if ctx is not None:
            raw = load().tsg_last_error_string(ctx)
            msg = raw.decode() if raw else ""
        raise TsgError(status, msg)
