"""ctypes front end of the CPU oracle (oracle/tsg_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker.  Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
may import this module.  The product path (tsugumi_b200) never does.

Parity status: the oracle restates the reference's Swift CPU reference
(Sources/TsugumiValidation/Support/Reference/MoE/Moe.swift) and host
algorithms; it is pinned against the reference's own known-answer tests
(grouping / planner golden arrays, router tie rule, GELU points) restated in
tests/test_oracle_golden.py, and against fixtures produced by the reference's
numpy forward (Scripts/qwen35/reference_forward.py, ReferenceModel._moe) in
tests/golden/.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libtsg_oracle.so"

ORC_ERRORS = {
    1: "invalidQueryCount",
    2: "invalidTopK",
    3: "invalidNumExperts",
    4: "invalidTileExpertCount",
    5: "pairCountMismatch",
    6: "tokenOutOfRange",
    7: "rankOutOfRange",
    8: "expertOutOfRange",
    9: "duplicateTokenRank",
    10: "expertSortKeyCountMismatch",
}


class OracleError(Exception):
    def __init__(self, code: int, value: int):
        self.code = code
        self.name = ORC_ERRORS.get(code, f"error{code}")
        self.value = value
        super().__init__(f"{self.name}({value})")


class ExpertOffsets(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "gate_w_off", "gate_s_off", "gate_b_off", "up_w_off", "up_s_off", "up_b_off",
        "down_w_off", "down_s_off", "down_b_off")]


class Layer(C.Structure):
    _fields_ = [
        ("d", C.c_int), ("f", C.c_int), ("num_experts", C.c_int), ("top_k", C.c_int),
        ("group", C.c_int), ("act", C.c_int),
        ("experts", C.c_void_p), ("expert_stride", C.c_uint64), ("off", ExpertOffsets),
        ("router_w", C.c_void_p), ("effective_scale", C.c_void_p),
        ("per_expert_scale", C.c_void_p), ("logit_bias", C.c_void_p),
        ("router_norm", C.c_int), ("norm_eps", C.c_float),
        ("shared", C.c_void_p), ("shared_f", C.c_int), ("shared_off", ExpertOffsets),
        ("shared_gate_w", C.c_void_p),
    ]


class Pair(C.Structure):
    _fields_ = [("token", C.c_uint32), ("expert", C.c_uint32), ("rank", C.c_uint32),
                ("weight_bits", C.c_uint32)]


PAIR_DTYPE = np.dtype([("token", "<u4"), ("expert", "<u4"), ("rank", "<u4"),
                       ("weight_bits", "<u4")])
GROUP_DTYPE = np.dtype([("expert", "<u4"), ("pair_start", "<u4"), ("pair_count", "<u4")])
TILE_DTYPE = np.dtype([("group_start", "<u4"), ("group_count", "<u4"), ("pair_start", "<u4"),
                       ("pair_count", "<u4")])
BLOCK_DTYPE = np.dtype([("local_slot", "<u4"), ("pair_start", "<u4"), ("row_count", "<u4"),
                        ("local_row", "<u4")])

_lib = None


def build() -> Path:
    env = dict(os.environ)
    env.pop("CC", None)
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.orc_splitmix64_next.restype = C.c_uint64
        L.orc_splitmix64_next.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_splitmix64_uniform.restype = C.c_float
        L.orc_splitmix64_uniform.argtypes = [C.POINTER(C.c_uint64), C.c_float, C.c_float]
        L.orc_seedtree_key.restype = C.c_uint64
        L.orc_seedtree_key.argtypes = [C.c_uint64, C.c_char_p]
        L.orc_bf16_bits.restype = C.c_uint16
        L.orc_bf16_bits.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_gelu_tanh.restype = C.c_double
        L.orc_gelu_tanh.argtypes = [C.c_double]
        L.orc_silu.restype = C.c_double
        L.orc_silu.argtypes = [C.c_double]
        L.orc_quantize_int4_sym.restype = None
        L.orc_quantize_int4_sym.argtypes = [P, C.c_int, C.c_int, P, P]
        L.orc_dequant_int4_sym_row.restype = None
        L.orc_dequant_int4_sym_row.argtypes = [P, P, C.c_int, C.c_int, P]
        L.orc_topk_select.restype = C.c_double
        L.orc_topk_select.argtypes = [P, C.c_int, C.c_int, P, P, P]
        L.orc_router.restype = None
        L.orc_router.argtypes = [C.POINTER(Layer), P, C.c_int, P, P, P, P]
        L.orc_moe_block.restype = None
        L.orc_moe_block.argtypes = [C.POINTER(Layer), P, C.c_int, P, P, P, P, P]
        L.orc_shared_expert.restype = None
        L.orc_shared_expert.argtypes = [C.POINTER(Layer), P, C.c_int, P]
        L.orc_make_pairs.restype = None
        L.orc_make_pairs.argtypes = [P, P, C.c_int, C.c_int, P]
        L.orc_group_pairs.restype = C.c_int
        L.orc_group_pairs.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, C.c_int,
                                      C.c_int, P, P, P, P, C.POINTER(C.c_int), P,
                                      C.POINTER(C.c_int), C.POINTER(C.c_uint32)]
        L.orc_plan_routed_gemm.restype = C.c_int
        L.orc_plan_routed_gemm.argtypes = [P, C.c_int, C.c_int, C.c_int, P, C.POINTER(C.c_int),
                                           P, P, P]
        L.orc_reduce_token_major.restype = None
        L.orc_reduce_token_major.argtypes = [P, P, C.c_int, C.c_int, C.c_int, P]
        L.orc_num_threads.restype = C.c_int
        L.orc_set_num_threads.restype = None
        L.orc_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def splitmix64_stream(seed: int, n: int) -> list[int]:
    st = C.c_uint64(seed)
    return [lib().orc_splitmix64_next(C.byref(st)) for _ in range(n)]


def seedtree_key(root: int, label: str) -> int:
    return int(lib().orc_seedtree_key(root, label.encode()))


def gelu_tanh(x: float) -> float:
    return float(lib().orc_gelu_tanh(x))


def quantize_int4_sym(row: np.ndarray, group: int = 32):
    row = np.ascontiguousarray(row, dtype=np.float32)
    packed = np.zeros(row.size // 2, np.uint8)
    scales = np.zeros(row.size // group, np.uint16)
    lib().orc_quantize_int4_sym(_p(row), row.size, group, _p(packed), _p(scales))
    return packed, scales


def dequant_int4_sym(packed: np.ndarray, scales: np.ndarray, n: int, group: int = 32):
    out = np.zeros(n, np.float32)
    lib().orc_dequant_int4_sym_row(_p(np.ascontiguousarray(packed)),
                                   _p(np.ascontiguousarray(scales)), n, group, _p(out))
    return out


def topk_select(logits: np.ndarray, k: int, per_expert_scale: np.ndarray | None = None):
    lg = np.ascontiguousarray(logits, dtype=np.float64)
    ids = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    pes = None if per_expert_scale is None else np.ascontiguousarray(per_expert_scale, np.float32)
    gap = lib().orc_topk_select(_p(lg), lg.size, k, _p(pes), _p(ids), _p(w))
    return ids, w, gap


class OracleLayer:
    """Host copy of one layer in the blob format, bound for the oracle."""

    def __init__(self, layer):
        # `layer` is a tsugumi_b200.synthetic.HostLayer (numpy arrays)
        self.h = layer
        s = Layer()
        s.d, s.f, s.num_experts, s.top_k = layer.d, layer.f, layer.num_experts, layer.top_k
        s.group = 32
        s.act = layer.act
        s.experts = _p(layer.experts)
        s.expert_stride = layer.expert_stride
        s.off = ExpertOffsets(*layer.offsets)
        s.router_w = _p(layer.router_w)
        s.effective_scale = _p(layer.effective_scale)
        s.per_expert_scale = _p(layer.per_expert_scale)
        s.logit_bias = _p(layer.logit_bias)
        s.router_norm = int(layer.router_norm)
        s.norm_eps = layer.norm_eps
        s.shared = _p(layer.shared)
        s.shared_f = layer.shared_f if layer.shared is not None else 0
        s.shared_off = ExpertOffsets(*(layer.shared_offsets or (0,) * 9))
        s.shared_gate_w = _p(layer.shared_gate)
        self.s = s

    def router(self, x_bf16: np.ndarray):
        T = x_bf16.shape[0]
        K, E = self.h.top_k, self.h.num_experts
        ids = np.zeros((T, K), np.uint32)
        w = np.zeros((T, K), np.float32)
        gap = np.zeros(T, np.float64)
        logits = np.zeros((T, E), np.float32)
        lib().orc_router(C.byref(self.s), _p(np.ascontiguousarray(x_bf16)), T, _p(ids), _p(w),
                         _p(gap), _p(logits))
        return ids, w, gap, logits

    def block(self, x_bf16: np.ndarray, ids: np.ndarray | None = None,
              w: np.ndarray | None = None):
        T = x_bf16.shape[0]
        K = self.h.top_k
        y = np.zeros((T, self.h.d), np.float32)
        ids_out = np.zeros((T, K), np.uint32)
        w_out = np.zeros((T, K), np.float32)
        ids_in = None if ids is None else np.ascontiguousarray(ids, np.uint32)
        w_in = None if w is None else np.ascontiguousarray(w, np.float32)
        lib().orc_moe_block(C.byref(self.s), _p(np.ascontiguousarray(x_bf16)), T, _p(ids_in),
                            _p(w_in), _p(y), _p(ids_out), _p(w_out))
        return y, ids_out, w_out

    def shared_expert(self, x_bf16: np.ndarray):
        T = x_bf16.shape[0]
        y = np.zeros((T, self.h.d), np.float32)
        lib().orc_shared_expert(C.byref(self.s), _p(np.ascontiguousarray(x_bf16)), T, _p(y))
        return y


def make_pairs(ids: np.ndarray, w_f16_bits: np.ndarray | None = None) -> np.ndarray:
    T, K = ids.shape
    out = np.zeros(T * K, PAIR_DTYPE)
    w = None if w_f16_bits is None else np.ascontiguousarray(w_f16_bits, np.uint16)
    lib().orc_make_pairs(_p(np.ascontiguousarray(ids, np.uint32)), _p(w), T, K, _p(out))
    return out


def group_pairs(pairs: np.ndarray, query_count: int, top_k: int, num_experts: int,
                tile_expert_count: int = 16, sort_keys=None, tile_break: int | None = None):
    """PrefillMoEGrouping.groupTokenExpertPairs; raises OracleError like the
    reference throws PrefillMoEGroupingError."""
    pairs = np.ascontiguousarray(pairs, PAIR_DTYPE)
    n = pairs.size
    ne = max(num_experts, 1)
    sorted_pairs = np.zeros(max(n, 1), PAIR_DTYPE)
    offsets = np.zeros(ne, np.uint32)
    counts = np.zeros(ne, np.uint32)
    groups = np.zeros(ne, GROUP_DTYPE)
    tiles = np.zeros(ne, TILE_DTYPE)
    ng, nt = C.c_int(0), C.c_int(0)
    errv = C.c_uint32(0)
    keys = None if sort_keys is None else np.ascontiguousarray(sort_keys, np.uint64)
    rc = lib().orc_group_pairs(_p(pairs) if n else None, n, query_count, top_k, num_experts,
                               tile_expert_count, _p(keys), 0 if keys is None else keys.size,
                               -1 if tile_break is None else tile_break, _p(sorted_pairs),
                               _p(offsets), _p(counts), _p(groups), C.byref(ng), _p(tiles),
                               C.byref(nt), C.byref(errv))
    if rc != 0:
        raise OracleError(rc, errv.value)
    return {
        "sorted_pairs": sorted_pairs[:n],
        "offsets": offsets[:num_experts],
        "counts": counts[:num_experts],
        "groups": groups[:ng.value],
        "tiles": tiles[:nt.value],
    }


def plan_routed_gemm(groups: np.ndarray, max_rows_per_batch: int, tile_rows: int = 64):
    groups = np.ascontiguousarray(groups, GROUP_DTYPE)
    total = int(groups["pair_count"].sum()) if groups.size else 0
    cap = total + groups.size + 4
    blocks = np.zeros(cap, BLOCK_DTYPE)
    rows = np.zeros(cap, np.int32)
    first = np.zeros(cap, np.int32)
    cnt = np.zeros(cap, np.int32)
    nb = C.c_int(0)
    nbatch = lib().orc_plan_routed_gemm(_p(groups) if groups.size else None, groups.size,
                                        max_rows_per_batch, tile_rows, _p(blocks), C.byref(nb),
                                        _p(rows), _p(first), _p(cnt))
    return [
        {"rows": int(rows[i]), "blocks": blocks[first[i]:first[i] + cnt[i]]}
        for i in range(nbatch)
    ]


def reduce_token_major(partials: np.ndarray, w: np.ndarray) -> np.ndarray:
    T, K = w.shape
    D = partials.shape[-1]
    h2 = np.zeros((T, D), np.float32)
    lib().orc_reduce_token_major(_p(np.ascontiguousarray(partials, np.float32)),
                                 _p(np.ascontiguousarray(w, np.float32)), T, K, D, _p(h2))
    return h2


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(n)


def num_threads() -> int:
    return int(lib().orc_num_threads())
