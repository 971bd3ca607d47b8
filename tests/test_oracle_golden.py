"""Pins the CPU oracle to the reference (no GPU needed).

Every known answer here comes from the reference project: its own test
expectations (restated as data, file:line given per test) and fixtures made
by running its numpy MoE forward (tests/golden/make_golden.py).
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tsugumi_b200.synthetic import bf16_bits_to_f32, host_layer, host_tokens

GOLDEN = Path(__file__).resolve().parent / "golden"


# --------------------------------------------------------------------------
# PRNG (Sources/TsugumiValidation/Support/PRNG/*.swift)
# --------------------------------------------------------------------------
def test_splitmix64_known_answers():
    # SplitMix64 from state 0: the published first outputs of the generator
    assert [hex(v) for v in O.splitmix64_stream(0, 3)] == [
        "0xe220a8397b1dcdaf", "0x6e789e6aa1b965f4", "0x6c45d188009454f"]


def test_seedtree_is_fnv1a_of_label_xor_root():
    h = 0xCBF29CE484222325
    for b in b"production-routed-moe":
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    assert O.seedtree_key(0x2D3, "production-routed-moe") == (0x2D3 ^ h)


# --------------------------------------------------------------------------
# Activations (Tests/Tsugumi/Core/Validation/Reference/MoEReferenceTests.swift:7-17)
# --------------------------------------------------------------------------
def test_gelu_tanh_matches_scalar_definition():
    assert abs(O.gelu_tanh(0.0)) < 1e-7
    expected_at_1 = 0.5 * (1 + math.tanh(0.7978845608028654 * (1 + 0.044715)))
    assert abs(O.gelu_tanh(1.0) - expected_at_1) < 1e-5
    assert O.gelu_tanh(1.0) > 0
    assert O.gelu_tanh(-1.0) < 0
    assert O.gelu_tanh(2.0) > O.gelu_tanh(1.0)


# --------------------------------------------------------------------------
# Weight format (Quantization.swift:166-227)
# --------------------------------------------------------------------------
def test_symmetric_quantization_round_trip_and_bias_identity():
    rng = np.random.default_rng(3)
    row = rng.uniform(-0.3, 0.3, 256).astype(np.float32)
    packed, scales = O.quantize_int4_sym(row)
    back = O.dequant_int4_sym(packed, scales, 256)
    s = np.repeat(scales.view(np.float16).astype(np.float32), 32)
    # within half a step where the value is inside the lattice -8..7
    assert np.all(np.abs(back - row) <= s * 0.5 + 1e-7)
    # codes are nibbles, low nibble = even element
    q0 = packed[0] & 0x0F
    assert back[0] == pytest.approx((float(q0) - 8.0) * s[0], abs=0)


def test_fp16_conversion_round_trips_all_finite_values():
    bits = np.arange(0, 0x7C00, 7, dtype=np.uint16)
    for b in bits[:2000]:
        f = O.lib().orc_f16_to_f32(int(b))
        assert O.lib().orc_f32_to_f16(f) == b


# --------------------------------------------------------------------------
# Router tie rule (Tests/Tsugumi/Core/Kernels/MoE/RouterTopKTests.swift:215-295)
# --------------------------------------------------------------------------
def _sort_reference(logits, k, expert_scale=None):
    """RouterTopKTests.reference: sort by logit descending, index ascending,
    softmax over the selected, times the expert scale."""
    paired = sorted(((float(v), e) for e, v in enumerate(logits)), key=lambda p: (-p[0], p[1]))
    sel = paired[:k]
    mx = sel[0][0]
    ex = [math.exp(v - mx) for v, _ in sel]
    s = sum(ex)
    w = [ex[i] / s * (1.0 if expert_scale is None else float(expert_scale[e]))
         for i, (_, e) in enumerate(sel)]
    return [e for _, e in sel], w


def _uniform(state, lo, hi, n):
    out = []
    st = state
    import ctypes as C
    s = C.c_uint64(st)
    for _ in range(n):
        out.append(O.lib().orc_splitmix64_uniform(C.byref(s), lo, hi))
    return out, s.value


def test_router_matches_sort_reference():
    experts, dim, k = 16, 128, 8
    import ctypes as C
    s = C.c_uint64(0xA5B61234)
    uni = lambda lo, hi: O.lib().orc_splitmix64_uniform(C.byref(s), lo, hi)
    weights = [[uni(-0.05, 0.05) + e * 0.01 for _ in range(dim)] for e in range(experts)]
    hidden = [uni(-1.0, 1.0) for _ in range(dim)]
    inv_sqrt_d = 1.0 / math.sqrt(dim)
    eff = [uni(0.5, 1.5) * inv_sqrt_d for _ in range(dim)]
    expert_scale = np.array([uni(0.6, 1.4) for _ in range(experts)], np.float32)
    logits = np.array([sum(w * h * e for w, h, e in zip(row, hidden, eff)) for row in weights])
    ids, w, _ = O.topk_select(logits, k, expert_scale)
    ref_ids, ref_w = _sort_reference(logits, k, expert_scale)
    assert list(ids) == ref_ids
    assert np.max(np.abs(w - np.array(ref_w))) < 1e-6


def test_router_resolves_near_tie_like_reference():
    experts, dim, k = 16, 128, 8
    import ctypes as C
    s = C.c_uint64(0x71E0F4A)
    uni = lambda lo, hi: O.lib().orc_splitmix64_uniform(C.byref(s), lo, hi)
    pattern = [uni(0.2, 1.0) for _ in range(dim)]
    hidden = [uni(0.5, 1.5) for _ in range(dim)]
    gains = [0.0] * experts
    for e in range(7):
        gains[e] = 1.0 - e * 0.05
    gains[7] = 0.5
    gains[8] = 0.5 * (1.0 + 1e-4)
    for e in range(9, experts):
        gains[e] = 0.4 - (e - 9) * 0.02
    logits = np.array([sum(g * p * h for p, h in zip(pattern, hidden)) for g in gains])
    ids, _, _ = O.topk_select(logits, k)
    assert list(ids) == _sort_reference(logits, k)[0]
    assert 8 in ids and 7 not in ids  # the larger gain wins the last slot


def test_exact_tie_keeps_lower_index():
    logits = np.array([0.5, 1.0, 1.0, 0.2, 1.0])
    ids, _, gap = O.topk_select(logits, 2)
    assert list(ids) == [1, 2]
    assert gap == 0.0


# --------------------------------------------------------------------------
# Reference forward fixtures (Scripts/qwen35/reference_forward.py:300-334)
# --------------------------------------------------------------------------
FIXTURES = ["tiny_swiglu", "tiny_shared", "small_qwenlike", "small_gemmalike_geglu",
            "gemma_geglu"]


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_reference_numpy_forward(name):
    fx = np.load(GOLDEN / f"{name}.npz")
    cfg = tuple(int(v) for v in fx["config"])
    layer = host_layer(cfg, int(fx["layer_seed"]))
    x = host_tokens(int(fx["T"]), cfg[0], int(fx["token_seed"]))
    ol = O.OracleLayer(layer)
    y, ids, w = ol.block(x)
    # the reference orders its picks by probability; ours by logit (same order)
    assert np.array_equal(ids.astype(np.int32), fx["router_idx"])
    assert np.max(np.abs(w - fx["router_w"])) < 1e-6
    rel = np.linalg.norm(y - fx["y"]) / np.linalg.norm(fx["y"])
    assert rel < 2e-6, rel


@pytest.mark.parametrize("name", FIXTURES)
def test_numpy_restatement_matches_reference_numpy_forward(name):
    """The second CPU reference (oracle/numpy_moe.py) reproduces the
    reference's own numpy forward on every fixture, GeGLU included."""
    from oracle import numpy_moe as NM

    fx = np.load(GOLDEN / f"{name}.npz")
    cfg = tuple(int(v) for v in fx["config"])
    layer = host_layer(cfg, int(fx["layer_seed"]))
    x = host_tokens(int(fx["T"]), cfg[0], int(fx["token_seed"]))
    ids, w, _ = NM.route(layer, NM.normalise(layer, x))
    assert np.array_equal(ids.astype(np.int32), fx["router_idx"])
    assert np.max(np.abs(w - fx["router_w"])) < 1e-6
    y = NM.moe_block(layer, x)
    rel = np.linalg.norm(y - fx["y"]) / np.linalg.norm(fx["y"])
    assert rel < 2e-6, rel


def test_numpy_restatement_matches_oracle_on_skewed_gemma_shape():
    """Two independent restatements agree on a Zipf-skewed GeGLU layer."""
    from oracle import numpy_moe as NM

    layer = host_layer((1024, 256, 64, 8, 0, 0), 5, skew=1.1)
    x = host_tokens(12, 1024, 3)
    y_c, ids_c, _ = O.OracleLayer(layer).block(x)
    ids_n, _, _ = NM.route(layer, NM.normalise(layer, x))
    assert np.array_equal(ids_n, ids_c)
    y_n = NM.moe_block(layer, x)
    assert np.linalg.norm(y_n - y_c) / np.linalg.norm(y_c) < 2e-6


# --------------------------------------------------------------------------
# Grouping (Tests/Tsugumi/Core/Kernels/Prefill/PrefillMoEGroupingTests.swift)
# --------------------------------------------------------------------------
def _pairs(rows):
    a = np.zeros(len(rows), O.PAIR_DTYPE)
    for i, (t, e, r, wb) in enumerate(rows):
        a[i] = (t, e, r, wb)
    return a


GROUPING_CASE_1 = [
    (0, 3, 0, 10), (0, 1, 1, 11), (0, 4, 2, 12), (1, 1, 0, 13), (1, 3, 1, 14), (1, 2, 2, 15),
    (2, 4, 0, 16), (2, 3, 1, 17), (2, 1, 2, 18), (3, 5, 0, 19), (3, 1, 1, 20), (3, 4, 2, 21),
]


def test_grouping_sorts_pairs_and_builds_offsets_counts_and_tiles():  # :6-54
    g = O.group_pairs(_pairs(GROUPING_CASE_1[::-1]), 4, 3, 6, tile_expert_count=2)
    sp = g["sorted_pairs"]
    assert list(sp["expert"]) == [1, 1, 1, 1, 2, 3, 3, 3, 4, 4, 4, 5]
    assert [[int(t), int(r)] for t, r in zip(sp["token"], sp["rank"])] == [
        [0, 1], [1, 0], [2, 2], [3, 1], [1, 2], [0, 0], [1, 1], [2, 1], [0, 2], [2, 0], [3, 2],
        [3, 0]]
    assert list(g["offsets"]) == [0xFFFFFFFF, 0, 4, 5, 8, 11]
    assert list(g["counts"]) == [0, 4, 1, 3, 3, 1]
    assert [tuple(x) for x in g["groups"].tolist()] == [
        (1, 0, 4), (2, 4, 1), (3, 5, 3), (4, 8, 3), (5, 11, 1)]
    assert [tuple(x) for x in g["tiles"].tolist()] == [(0, 2, 0, 5), (2, 2, 5, 6), (4, 1, 11, 1)]
    assert int(g["groups"]["pair_count"].max()) == 4
    assert int(g["tiles"]["pair_count"].max()) == 6
    assert int(g["tiles"]["group_count"].max()) == 2


def test_grouping_is_deterministic_and_preserves_weight_bits():  # :56-87
    tm = [(0, 2, 0, 101), (0, 1, 1, 102), (1, 2, 0, 103), (1, 0, 1, 104), (2, 1, 0, 105),
          (2, 2, 1, 106)]
    shuffled = [tm[5], tm[1], tm[3], tm[0], tm[4], tm[2]]
    a = O.group_pairs(_pairs(tm), 3, 2, 3, tile_expert_count=2)
    b = O.group_pairs(_pairs(shuffled), 3, 2, 3, tile_expert_count=2)
    for key in a:
        assert np.array_equal(a[key], b[key])
    assert list(a["sorted_pairs"]["weight_bits"]) == [104, 102, 105, 101, 103, 106]


def test_grouping_orders_by_expert_sort_keys():  # :89-121
    p = _pairs([(0, 1, 0, 10), (0, 2, 1, 20), (1, 3, 0, 30), (1, 1, 1, 11), (2, 2, 0, 21),
                (2, 3, 1, 31)])
    g = O.group_pairs(p, 3, 2, 4, tile_expert_count=2, sort_keys=[0, 30, 10, 20])
    assert list(g["groups"]["expert"]) == [2, 3, 1]
    assert list(g["sorted_pairs"]["expert"]) == [2, 2, 3, 3, 1, 1]
    assert list(g["offsets"]) == [0xFFFFFFFF, 4, 0, 2]
    assert [tuple(x) for x in g["tiles"].tolist()] == [(0, 2, 0, 4), (2, 1, 4, 2)]


@pytest.mark.parametrize("kwargs,pairs,err,value", [
    (dict(query_count=1, top_k=1, num_experts=1, tile_expert_count=17), [(0, 0, 0, 1)],
     "invalidTileExpertCount", 17),
    (dict(query_count=1, top_k=1, num_experts=2, tile_expert_count=1), [(0, 2, 0, 1)],
     "expertOutOfRange", 2),
    (dict(query_count=1, top_k=2, num_experts=2, tile_expert_count=1), [(0, 0, 0, 1), (0, 1, 0, 2)],
     "duplicateTokenRank", 0),
    (dict(query_count=1, top_k=1, num_experts=2, tile_expert_count=1, sort_keys=[0]),
     [(0, 0, 0, 1)], "expertSortKeyCountMismatch", 1),
])
def test_grouping_rejects_invalid_metadata(kwargs, pairs, err, value):  # :123-177
    with pytest.raises(O.OracleError) as ei:
        O.group_pairs(_pairs(pairs), **kwargs)
    assert ei.value.name == err and ei.value.value == value


def test_grouping_tolerates_real_trace_pressure_at_t32():  # :179-204
    rows = [(t, (t + r * 7) % 74, r, t * 8 + r) for t in range(32) for r in range(8)]
    g = O.group_pairs(_pairs(rows), 32, 8, 128, tile_expert_count=16)
    assert g["sorted_pairs"].size == 256
    assert g["groups"].size <= 74
    assert int(g["tiles"]["group_count"].max()) <= 16
    assert all(int(t["pair_count"]) > 0 for t in g["tiles"])


def test_tile_break_cuts_the_tile_at_the_requested_group():  # :206-238
    rows = [(t, (t * 5 + r) % 10, r, t * 5 + r) for t in range(4) for r in range(5)]
    g = O.group_pairs(_pairs(rows), 4, 5, 10, tile_expert_count=4, tile_break=3)
    assert g["groups"].size == 10
    assert list(g["tiles"]["group_count"]) == [3, 4, 3]
    assert list(g["tiles"]["group_start"]) == [0, 3, 7]
    assert int(g["tiles"]["pair_count"].sum()) == g["sorted_pairs"].size
    start = 0
    for t in g["tiles"]:
        assert int(t["pair_start"]) == start
        start += int(t["pair_count"])


def test_tile_break_beyond_the_groups_changes_nothing():  # :240-258
    rows = [(i // 2, i % 4, i % 2, i) for i in range(8)]
    a = O.group_pairs(_pairs(rows), 4, 2, 4, tile_expert_count=2)
    b = O.group_pairs(_pairs(rows), 4, 2, 4, tile_expert_count=2, tile_break=99)
    assert np.array_equal(a["tiles"], b["tiles"])


# --------------------------------------------------------------------------
# Planner (Tests/Tsugumi/Core/Kernels/Prefill/PrefillRoutedGEMMPlannerTests.swift)
# --------------------------------------------------------------------------
def _groups(rows):
    a = np.zeros(len(rows), O.GROUP_DTYPE)
    for i, r in enumerate(rows):
        a[i] = r
    return a


def _covers_once(batches, groups):
    seen = {}
    for b in batches:
        rows_seen = set()
        for blk in b["blocks"]:
            assert 1 <= blk["row_count"] <= 64
            assert int(blk["local_row"]) + int(blk["row_count"]) <= b["rows"]
            for i in range(int(blk["row_count"])):
                assert int(blk["local_row"]) + i not in rows_seen
                rows_seen.add(int(blk["local_row"]) + i)
                pair = int(blk["pair_start"]) + i
                seen[pair] = seen.get(pair, 0) + 1
                g = groups[int(blk["local_slot"])]
                assert int(g["pair_start"]) <= pair < int(g["pair_start"]) + int(g["pair_count"])
        assert len(rows_seen) == b["rows"]
    expected = [int(g["pair_start"]) + i for g in groups for i in range(int(g["pair_count"]))]
    assert sorted(seen) == sorted(expected) and all(v == 1 for v in seen.values())


def test_planner_packs_whole_groups_when_they_fit():  # :38-50
    g = _groups([(3, 0, 40), (7, 40, 20)])
    b = O.plan_routed_gemm(g, 128)
    assert len(b) == 1 and b[0]["rows"] == 60 and len(b[0]["blocks"]) == 2
    assert b[0]["blocks"][1]["local_row"] == 40 and b[0]["blocks"][1]["local_slot"] == 1
    _covers_once(b, g)


def test_planner_starts_new_batch_rather_than_splitting():  # :52-58
    g = _groups([(0, 0, 100), (1, 100, 100)])
    b = O.plan_routed_gemm(g, 128)
    assert [x["rows"] for x in b] == [100, 100]
    assert list(b[0]["blocks"]["row_count"]) == [64, 36]
    _covers_once(b, g)


def test_planner_splits_big_group_on_full_blocks():  # :60-67
    g = _groups([(0, 0, 300)])
    b = O.plan_routed_gemm(g, 128)
    assert [x["rows"] for x in b] == [128, 128, 44]
    assert list(b[0]["blocks"]["row_count"]) == [64, 64]
    assert list(b[2]["blocks"]["row_count"]) == [44]
    _covers_once(b, g)


def test_planner_rounds_budget_down_to_whole_blocks():  # :71-76
    g = _groups([(0, 0, 200)])
    b = O.plan_routed_gemm(g, 100)
    assert [x["rows"] for x in b] == [64, 64, 64, 8]
    _covers_once(b, g)


def test_planner_single_row_groups():  # :78-84
    g = _groups([(i, i, 1) for i in range(16)])
    b = O.plan_routed_gemm(g, 512)
    assert len(b) == 1 and len(b[0]["blocks"]) == 16
    _covers_once(b, g)


def test_planner_empty_groups():  # :86-88
    assert O.plan_routed_gemm(_groups([]), 512) == []


# --------------------------------------------------------------------------
# Pair layout (Tests/Tsugumi/Core/Kernels/Prefill/PrefillRouterTests.swift:12-30)
# --------------------------------------------------------------------------
def test_pair_layout_is_16_bytes_with_fields_at_0_4_8_12():
    import ctypes as C
    assert C.sizeof(O.Pair) == 16
    assert [O.Pair.token.offset, O.Pair.expert.offset, O.Pair.rank.offset,
            O.Pair.weight_bits.offset] == [0, 4, 8, 12]
    p = O.make_pairs(np.array([[3, 1], [0, 2]], np.uint32), np.array([[1, 2], [3, 4]], np.uint16))
    assert [tuple(int(v) for v in x) for x in p.tolist()] == [
        (0, 3, 0, 1), (0, 1, 1, 2), (1, 0, 0, 3), (1, 2, 1, 4)]


# --------------------------------------------------------------------------
# Reduce (prefill.metal:796-817)
# --------------------------------------------------------------------------
def test_reduce_token_major_sums_ranks_in_order():
    rng = np.random.default_rng(1)
    T, K, D = 5, 3, 16
    partials = rng.standard_normal((T * K, D)).astype(np.float32)
    w = rng.uniform(0, 1, (T, K)).astype(np.float32)
    h2 = O.reduce_token_major(partials, w)
    ref = np.einsum("tk,tkd->td", w.astype(np.float64),
                    partials.reshape(T, K, D).astype(np.float64))
    assert np.max(np.abs(h2 - ref)) < 1e-5


def test_oracle_router_norm_uses_no_scale_rmsnorm():
    layer = host_layer("tiny", 9)
    x = host_tokens(4, 512, 1)
    ids, w, gap, logits = O.OracleLayer(layer).router(x)
    xf = bf16_bits_to_f32(x).astype(np.float64)
    xn = xf / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + 1e-6)
    ref = xn @ layer.router_w.astype(np.float64).T
    assert np.max(np.abs(logits - ref)) < 1e-5
