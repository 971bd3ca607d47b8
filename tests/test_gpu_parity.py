"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bars:
  * expert ids and permutation / index arrays bit-exact, except tokens whose
    K-th / (K+1)-th logit gap is below 1e-6;
  * block outputs within relative L2 error 2e-3 of the fp32-accumulated
    oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsugumi_b200 as tb  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tsugumi_b200.synthetic import host_layer, host_tokens  # noqa: E402

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
TIE_GAP = 1e-6


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


_LAYERS: dict = {}


@pytest.fixture(scope="module")
def ctx():
    c = tb.Context(0)
    yield c
    _LAYERS.clear()
    c.close()


def layer_pair(ctx, name, seed, skew=None):
    key = (name, seed, skew)
    if key not in _LAYERS:
        host = host_layer(name, seed, skew=skew)
        dev = tb.MoELayer(ctx, tb.upload_host_layer(host))
        _LAYERS[key] = (host, dev, O.OracleLayer(host))
    return _LAYERS[key]


class regime:
    """Temporarily selects the regime: decode_max_tokens, the fused
    single-kernel decode switch and the largest batch the batched GEMVs
    take (0: small batches use the tensor-core contraction too)."""

    def __init__(self, ctx, dmax=4, fused=True, gemv=64):
        self.ctx, self.dmax, self.fused, self.gemv = ctx, dmax, fused, gemv

    def __enter__(self):
        self.ctx.set_decode_max_tokens(self.dmax)
        self.ctx.set_option("fused_decode", 1 if self.fused else 0)
        self.ctx.set_option("gemv_max_tokens", self.gemv)

    def __exit__(self, *exc):
        self.ctx.set_decode_max_tokens(3)  # the library's default
        self.ctx.set_option("fused_decode", 1)
        self.ctx.set_option("gemv_max_tokens", 16)


def gpu_route(ctx, layer, x_dev):
    T = x_dev.shape[0]
    ids = torch.empty((T, layer.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.top_k), dtype=torch.float32, device="cuda")
    w16 = torch.empty((T, layer.top_k), dtype=torch.float16, device="cuda")
    tb.MoE(ctx, layer).encode_router_gemma4_bf16(x_dev, ids, w, w16)
    ctx.sync()
    return ids, w, w16


def to_dev(x_np):
    return torch.from_numpy(x_np.view(np.int16)).to("cuda").view(torch.bfloat16)


ROUTER_CASES = [
    ("tiny", 16, None, 64),
    ("gemma", 1, None, 64),
    ("gemma", 4, None, 64),
    ("gemma", 64, None, 64),
    ("gemma", 256, 1.1, 64),
    ("qwen", 16, None, 64),
    ("qwen", 300, None, 64),
    ("tiny", 40, None, 0),  # prefill router kernels on a small batch
    # small-batch prefill router (T <= 64): ragged token passes, split D
    ("gemma", 8, None, 0),
    ("gemma", 64, 1.1, 0),
    ("qwen", 33, None, 0),
    # tensor-core prefill router: a partial second token tile, 16 experts in
    # a zero-padded 128-row tile, a large batch
    ("gemma", 200, None, 0),
    ("tiny", 300, None, 0),
    ("qwen", 4096, None, 0),
]


@pytest.mark.parametrize("name,T,skew,dmax", ROUTER_CASES)
def test_router_topk_matches_oracle(ctx, name, T, skew, dmax):
    host, dev, ol = layer_pair(ctx, name, 11, skew)
    x = host_tokens(T, host.d, 100 + T)
    with regime(ctx, dmax):
        ids, w, w16 = gpu_route(ctx, dev, to_dev(x))
    ref_ids, ref_w, gap, _ = ol.router(x)
    ok = gap >= TIE_GAP
    assert ok.sum() >= T - 1
    g_ids = ids.cpu().numpy().astype(np.uint32)
    assert np.array_equal(g_ids[ok], ref_ids[ok])
    assert np.max(np.abs(w.cpu().numpy()[ok] - ref_w[ok])) < 2e-6
    assert np.max(np.abs(w16.float().cpu().numpy()[ok] - ref_w[ok])) < 1e-3


@pytest.mark.parametrize("name,T,skew", [("gemma", 1, None), ("gemma", 200, 1.1),
                                         ("qwen", 33, None), ("tiny", 4096, None)])
def test_router_logits_match_oracle(ctx, name, T, skew):
    """tsg_router_logits (encodeRouterLogitsBF16) gives the scores the oracle
    ranks: normalised dot plus bias, fp32."""
    host, dev, ol = layer_pair(ctx, name, 11, skew)
    x = host_tokens(T, host.d, 300 + T)
    out = torch.empty((T, host.num_experts), dtype=torch.float32, device="cuda")
    tb.MoE(ctx, dev).encode_router_logits_bf16(to_dev(x), out)
    ctx.sync()
    _, _, _, ref = ol.router(x)
    got = out.cpu().numpy()
    assert np.max(np.abs(got - ref)) < 2e-6 * max(1.0, float(np.abs(ref).max()))


def _np_pairs(rows):
    a = np.zeros((len(rows), 4), np.int32)
    for i, r in enumerate(rows):
        a[i] = r
    return a


def test_grouping_golden_case_on_gpu(ctx):
    rows = [(0, 3, 0, 10), (0, 1, 1, 11), (0, 4, 2, 12), (1, 1, 0, 13), (1, 3, 1, 14),
            (1, 2, 2, 15), (2, 4, 0, 16), (2, 3, 1, 17), (2, 1, 2, 18), (3, 5, 0, 19),
            (3, 1, 1, 20), (3, 4, 2, 21)][::-1]
    pairs = torch.from_numpy(_np_pairs(rows)).cuda()
    g = tb.PrefillMoEGrouping.group_token_expert_pairs(ctx, pairs, 4, 3, 6, tile_expert_count=2)
    assert list(g.sorted_pairs[:, 1]) == [1, 1, 1, 1, 2, 3, 3, 3, 4, 4, 4, 5]
    assert g.sorted_pairs[:, [0, 2]].tolist() == [
        [0, 1], [1, 0], [2, 2], [3, 1], [1, 2], [0, 0], [1, 1], [2, 1], [0, 2], [2, 0], [3, 2],
        [3, 0]]
    assert list(g.per_expert_offsets) == [0xFFFFFFFF, 0, 4, 5, 8, 11]
    assert list(g.per_expert_counts) == [0, 4, 1, 3, 3, 1]
    assert g.groups.tolist() == [[1, 0, 4], [2, 4, 1], [3, 5, 3], [4, 8, 3], [5, 11, 1]]
    assert g.tiles.tolist() == [[0, 2, 0, 5], [2, 2, 5, 6], [4, 1, 11, 1]]
    assert g.max_pairs_per_expert == 4 and g.max_pairs_per_tile == 6
    assert g.max_live_experts_per_tile == 2


@pytest.mark.parametrize("T,K,E,tec,keys,brk", [
    (37, 4, 16, 16, False, None),
    (512, 8, 128, 16, False, None),
    (300, 8, 256, 5, True, None),
    (64, 6, 40, 4, False, 3),
    (4096, 8, 128, 16, False, None),
])
def test_grouping_matches_oracle(ctx, T, K, E, tec, keys, brk):
    rng = np.random.default_rng(T + K)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.uint32)
    w16 = rng.integers(0, 0x3C00, (T, K)).astype(np.uint16)
    pairs = O.make_pairs(ids, w16)
    perm = rng.permutation(T * K)
    shuffled = pairs[perm]
    sort_keys = rng.integers(0, 5, E).astype(np.uint64) if keys else None
    ref = O.group_pairs(shuffled, T, K, E, tec, sort_keys, brk)
    p = np.stack([shuffled[f].astype(np.int64) for f in ("token", "expert", "rank",
                                                          "weight_bits")], 1).astype(np.int32)
    g = tb.PrefillMoEGrouping.group_token_expert_pairs(
        ctx, torch.from_numpy(p).cuda(), T, K, E, tec,
        None if sort_keys is None else sort_keys, brk)
    got = g.sorted_pairs
    assert np.array_equal(got[:, 0], ref["sorted_pairs"]["token"])
    assert np.array_equal(got[:, 1], ref["sorted_pairs"]["expert"])
    assert np.array_equal(got[:, 2], ref["sorted_pairs"]["rank"])
    assert np.array_equal(got[:, 3], ref["sorted_pairs"]["weight_bits"])
    assert np.array_equal(g.per_expert_offsets, ref["offsets"])
    assert np.array_equal(g.per_expert_counts, ref["counts"])
    assert g.groups.tolist() == [list(x) for x in ref["groups"].tolist()]
    assert g.tiles.tolist() == [list(x) for x in ref["tiles"].tolist()]


@pytest.mark.parametrize("rows,args,msg", [
    ([(0, 2, 0, 1)], (1, 1, 2), "expert 2 is out of range"),
    ([(0, 0, 0, 1), (0, 1, 0, 2)], (1, 2, 2), "duplicate route pair for token 0"),
    ([(3, 0, 0, 1)], (1, 1, 2), "token 3 is out of range"),
])
def test_grouping_rejects_invalid_pairs(ctx, rows, args, msg):
    with pytest.raises(tb.PrefillMoEGroupingError, match=msg):
        tb.PrefillMoEGrouping.group_token_expert_pairs(
            ctx, torch.from_numpy(_np_pairs(rows)).cuda(), *args, tile_expert_count=1)


def test_grouping_rejects_bad_arguments(ctx):
    p = torch.from_numpy(_np_pairs([(0, 0, 0, 1)])).cuda()
    with pytest.raises(tb.PrefillMoEGroupingError, match="tileExpertCount must be in 1...16, got 17"):
        tb.PrefillMoEGrouping.group_token_expert_pairs(ctx, p, 1, 1, 1, tile_expert_count=17)
    with pytest.raises(tb.PrefillMoEGroupingError, match="expected 2 expert sort keys, got 1"):
        tb.PrefillMoEGrouping.group_token_expert_pairs(ctx, p, 1, 1, 2, 1, expert_sort_keys=[0])


BLOCK_CASES = [
    # name, T, skew, decode_max_tokens, fused, oracle token sample
    ("tiny", 4, None, 4, True, None),
    ("gemma", 1, None, 4, True, None),
    ("gemma", 2, None, 4, True, None),
    ("gemma", 4, None, 4, True, None),
    ("qwen", 1, None, 4, True, None),
    ("qwen", 4, None, 4, True, None),
    ("tiny", 16, None, 64, False, None),
    ("gemma", 1, None, 64, False, None),
    ("gemma", 16, None, 64, False, None),
    ("gemma", 64, None, 64, False, None),
    ("qwen", 64, None, 64, False, None),
    ("gemma", 16, None, 4, True, None),   # T > 4: grouped tcgen05 path
    ("tiny", 200, None, 4, True, None),
    ("gemma", 512, None, 4, True, 48),
    # the BASELINE prefill configs: Gemma-like T=4096 with Zipf(1.1) skew
    # (configs[2]) and Qwen-like T=4096, 512 sampled rows each
    # plus the first and last token of the hottest expert's segment
    ("gemma", 4096, 1.1, 4, True, 512),
    ("qwen", 1024, None, 4, True, 48),
    ("qwen", 4096, None, 4, True, 512),
    ("gemma", 48, None, 0, True, None),
    # 4 < T <= 64: batched GEMVs (ragged token blocks, few rows per expert)
    ("tiny", 5, None, 4, True, None),
    ("gemma", 9, None, 4, True, None),
    ("gemma", 64, 1.1, 4, True, None),
    ("qwen", 33, None, 4, True, None),
    ("qwen", 64, None, 4, True, None),
    # Gemma with its dense MLP branch (F = 2112 beside the experts' 704):
    # decode kernels, batched GEMVs and the tcgen05 contraction for the branch
    ("gemma_dense", 1, None, 4, True, None),
    ("gemma_dense", 3, None, 4, True, None),
    ("gemma_dense", 12, None, 4, True, None),
    ("gemma_dense", 300, None, 4, True, 48),
    ("gemma_dense", 8, None, 64, False, None),
]


def sample_rows(ids: np.ndarray, n: int) -> np.ndarray:
    """n evenly spaced tokens plus the first and last token routed to the
    most loaded expert (the two ends of its segment in the sorted pairs, so
    the first and the last row tile of the hottest expert are checked)."""
    T = ids.shape[0]
    counts = np.bincount(ids.ravel(), minlength=int(ids.max()) + 1)
    hot_tokens = np.nonzero((ids == int(np.argmax(counts))).any(axis=1))[0]
    rows = np.linspace(0, T - 1, n).astype(int)
    return np.unique(np.concatenate([rows, hot_tokens[:1], hot_tokens[-1:]]))


@pytest.mark.parametrize("name,T,skew,dmax,fused,sample", BLOCK_CASES)
def test_block_forward_matches_oracle(ctx, name, T, skew, dmax, fused, sample):
    host, dev, ol = layer_pair(ctx, name, 11, skew)
    x = host_tokens(T, host.d, 7 + T)
    xd = to_dev(x)
    with regime(ctx, dmax, fused):
        y = dev.forward(xd, out_dtype=torch.float32)
        ctx.sync()
    ids, w, _ = gpu_route(ctx, dev, xd)
    ref_ids, _, gap, _ = ol.router(x)
    ok = gap >= TIE_GAP
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32)[ok], ref_ids[ok])
    rows = np.arange(T) if sample is None else sample_rows(ids.cpu().numpy(), sample)
    y_ref, _, _ = ol.block(x[rows], ids.cpu().numpy()[rows].astype(np.uint32),
                           w.cpu().numpy()[rows])
    y_gpu = y.cpu().numpy()[rows]
    err = rel_l2(y_gpu, y_ref)
    print(f"{name} T={T} fused={fused} dmax={dmax}: rel L2 {err:.3e}")
    assert np.all(np.isfinite(y_gpu))
    assert err <= REL_L2


@pytest.mark.parametrize("name,T", [("gemma", 1), ("qwen", 3)])
def test_fused_decode_graph_replay_is_stable(ctx, name, T):
    """Replaying the fused kernel from a CUDA graph (its grid counters reset
    themselves at the end of every launch) gives the same bits every time,
    equal to a plain launch."""
    host, dev, ol = layer_pair(ctx, name, 11, None)
    xd = to_dev(host_tokens(T, host.d, 77))
    y0 = dev.forward(xd, out_dtype=torch.float32)
    ctx.sync()
    ctx.reserve(dev, T)
    y = torch.empty((T, host.d), dtype=torch.float32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        ctx.set_stream(side)
        with torch.cuda.graph(g, stream=side):
            dev.forward(xd, y=y)
    torch.cuda.current_stream().wait_stream(side)
    ctx.set_stream(torch.cuda.current_stream())
    for _ in range(5):
        y.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, y0)
    ctx.sync()
    del g


@pytest.mark.parametrize("name,T,coop", [("gemma", 1, 1), ("qwen", 1, 1), ("gemma", 2, 1),
                                         ("qwen", 4, 1), ("gemma", 1, 0), ("qwen", 3, 0)])
def test_programmatic_launch_chain_is_bit_equal(ctx, name, T, coop):
    """A chain of layers, each reading the previous one's output, launched
    with programmatic dependent launch (the next grid starts before this one
    ends and waits for it), cooperatively or not: the same bits as a plain
    cooperative launch, eager and from a CUDA graph."""
    lays = [layer_pair(ctx, name, 31 + l, None)[1] for l in range(6)]
    d = lays[0].d
    x0 = to_dev(host_tokens(T, d, 5))
    bufs = [torch.empty((T, d), dtype=torch.bfloat16, device="cuda") for _ in lays]

    def chain():
        x = x0
        for lay, b in zip(lays, bufs):
            lay.forward(x, y=b)
            x = b
        return bufs[-1]

    ctx.set_decode_max_tokens(4)  # the decode kernels for every T here
    ctx.set_option("programmatic_launch", 0)
    want = chain().clone()
    ctx.sync()
    ctx.set_option("programmatic_launch", 1)
    ctx.set_option("cooperative_launch", coop)
    try:
        for _ in range(3):
            got = chain()
            ctx.sync()
            assert torch.equal(got, want)
        for lay in lays:
            ctx.reserve(lay, T)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            ctx.set_stream(side)
            with torch.cuda.graph(g, stream=side):
                chain()
        torch.cuda.current_stream().wait_stream(side)
        ctx.set_stream(torch.cuda.current_stream())
        for _ in range(5):
            bufs[-1].zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(bufs[-1], want)
        ctx.sync()
        del g
    finally:
        ctx.set_option("programmatic_launch", 1)
        ctx.set_option("cooperative_launch", 1)
        ctx.set_decode_max_tokens(3)


@pytest.mark.parametrize("name,T", [("tiny", 1), ("gemma", 1), ("gemma", 3), ("qwen", 1),
                                    ("qwen", 4)])
def test_streaming_decode_matches_earlier_fused_kernel(ctx, name, T):
    """The streaming decode kernel (option fused_decode=1, the default) and
    the earlier single kernel with a grid-wide act exchange (fused_decode=2)
    give the same block output to the parity bar, and the same routing."""
    host, dev, ol = layer_pair(ctx, name, 11, None)
    xd = to_dev(host_tokens(T, host.d, 500 + T))
    ys = []
    for kind in (1, 2):
        with regime(ctx, dmax=4, gemv=16):
            ctx.set_option("fused_decode", kind)
            ys.append(dev.forward(xd, out_dtype=torch.float32))
            ctx.sync()
    err = rel_l2(ys[0].cpu().numpy(), ys[1].cpu().numpy())
    print(f"{name} T={T}: streaming vs earlier fused rel L2 {err:.3e}")
    assert err < REL_L2


@pytest.mark.parametrize("name,T", [("tiny", 7), ("gemma", 24), ("qwen", 64)])
def test_small_batch_gemv_matches_contraction(ctx, name, T):
    """The batched GEMVs and the tensor-core contraction compute the same
    expert products for a small router-driven batch."""
    host, dev, ol = layer_pair(ctx, name, 11, None)
    xd = to_dev(host_tokens(T, host.d, 5 + T))
    with regime(ctx, 4, True, 64):
        y_gemv = dev.forward(xd, out_dtype=torch.float32)
        ctx.sync()
    with regime(ctx, 4, True, 0):
        y_qmm = dev.forward(xd, out_dtype=torch.float32)
        ctx.sync()
    err = rel_l2(y_gemv.cpu().numpy(), y_qmm.cpu().numpy())
    print(f"{name} T={T}: gemv vs contraction rel L2 {err:.3e}")
    assert err < REL_L2


@pytest.mark.parametrize("name,T", [("gemma", 4), ("qwen", 32)])
def test_decode_and_prefill_regimes_agree(ctx, name, T):
    host, dev, ol = layer_pair(ctx, name, 11, None)
    xd = to_dev(host_tokens(T, host.d, 3))
    with regime(ctx, 64, False):
        y_dec = dev.forward(xd, out_dtype=torch.float32)
    with regime(ctx, 0):
        y_pre = dev.forward(xd, out_dtype=torch.float32)
        ctx.sync()
    assert rel_l2(y_pre.cpu().numpy(), y_dec.cpu().numpy()) < REL_L2


@pytest.mark.parametrize("which,T,hot", [
    ("decode", 3, False), ("decode", 8, False), ("prefill", 200, False),
    # caller routing may send every slot of every token to one expert: one
    # row tile of T*K rows with no more rows in the whole buffer (160: larger
    # than a 128-row token box, smaller than the 192-row one), exactly one
    # full tile (192), and a full tile plus a ragged one (240)
    ("prefill", 20, True), ("prefill", 24, True), ("prefill", 30, True)])
def test_experts_with_caller_routing(ctx, which, T, hot):
    host, dev, ol = layer_pair(ctx, "gemma", 11, None)
    x = host_tokens(T, host.d, 55)
    rng = np.random.default_rng(5)
    if hot:
        ids = np.full((T, host.top_k), 7, dtype=np.int64)
    else:
        ids = np.stack([rng.choice(host.num_experts, host.top_k, replace=False)
                        for _ in range(T)])
    w = rng.uniform(0.05, 0.3, (T, host.top_k)).astype(np.float32)
    resid = rng.standard_normal((T, host.d)).astype(np.float32)
    y = torch.empty((T, host.d), dtype=torch.float32, device="cuda")
    idt = torch.from_numpy(ids.astype(np.int32)).cuda()
    wt = torch.from_numpy(w).cuda()
    rt = torch.from_numpy(resid).cuda()
    if which == "decode":
        tb.MoE(ctx, dev).encode_routed_phases(to_dev(x), idt, wt, y, residual=rt)
    else:
        tb.PrefillGroupedRoutedMoE(ctx, dev).encode_streamed_tiled(to_dev(x), idt, wt, y,
                                                                   residual=rt)
    ctx.sync()
    y_ref, _, _ = ol.block(x, ids.astype(np.uint32), w)
    assert rel_l2(y.cpu().numpy(), y_ref + resid) <= REL_L2


@pytest.mark.parametrize("name,T", [("qwen", 1), ("qwen", 100), ("gemma_dense", 1),
                                    ("gemma_dense", 100)])
def test_shared_expert_alone(ctx, name, T):
    """SharedExpertRuntime alone: Qwen's shared expert, and Gemma's dense
    branch (SharedExpertInt4.swift:30-94) whose F differs from the experts'."""
    host, dev, ol = layer_pair(ctx, name, 11, None)
    x = host_tokens(T, host.d, 21)
    y = torch.empty((T, host.d), dtype=torch.float32, device="cuda")
    tb.SharedExpertRuntime(ctx, dev).encode(to_dev(x), y)
    ctx.sync()
    assert rel_l2(y.cpu().numpy(), ol.shared_expert(x)) <= REL_L2


def test_reduce_token_major(ctx):
    rng = np.random.default_rng(2)
    T, K, D = 33, 8, 512
    part = rng.standard_normal((T * K, D)).astype(np.float16)
    w = rng.uniform(0, 1, (T, K)).astype(np.float32)
    h2 = torch.empty((T, D), dtype=torch.float32, device="cuda")
    tb.PrefillMoE.encode_reduce_token_major(ctx, torch.from_numpy(part).cuda(),
                                            torch.from_numpy(w).cuda(), h2)
    ctx.sync()
    ref = O.reduce_token_major(part.astype(np.float32), w)
    assert np.max(np.abs(h2.cpu().numpy() - ref)) < 1e-5


def test_make_token_expert_pairs(ctx):
    ids = torch.tensor([[3, 1], [0, 2]], dtype=torch.int32, device="cuda")
    w16 = torch.tensor([[1, 2], [3, 4]], dtype=torch.int16, device="cuda")
    p = tb.PrefillRouter.make_token_expert_pairs(ctx, ids, w16, 2, 2)
    ctx.sync()
    assert p.cpu().tolist() == [[0, 3, 0, 1], [0, 1, 1, 2], [1, 0, 0, 3], [1, 2, 1, 4]]


def test_bf16_output_and_residual(ctx):
    host, dev, ol = layer_pair(ctx, "tiny", 11, None)
    T = 16
    x = host_tokens(T, host.d, 4)
    resid = np.random.default_rng(0).standard_normal((T, host.d)).astype(np.float32)
    xd = to_dev(x)
    ids, w, _ = gpu_route(ctx, dev, xd)
    y = dev.forward(xd, residual=torch.from_numpy(resid).cuda(), out_dtype=torch.bfloat16)
    ctx.sync()
    y_ref, _, _ = ol.block(x, ids.cpu().numpy().astype(np.uint32), w.cpu().numpy())
    assert rel_l2(y.float().cpu().numpy(), y_ref + resid) <= REL_L2


@pytest.mark.parametrize("name,T", [("gemma", 1), ("gemma", 2), ("gemma", 5), ("qwen", 3),
                                    ("qwen", 8), ("tiny", 4), ("gemma_dense", 3)])
def test_verify_rows_bit_equal_to_decode(ctx, name, T):
    """A speculative-verify block gives every row decode's bits: the rows
    path against T single-token forwards, compared bit for bit (as
    PrefillRoutedMoERowsVsDecodeTests.swift:23-166 compares the reference's
    rows path with its decode kernels), with and without a residual; and the
    block against the oracle."""
    host, dev, ol = layer_pair(ctx, name, 11, None)
    x = host_tokens(T, host.d, 300 + T)
    xd = to_dev(x)
    g = torch.Generator(device="cpu").manual_seed(5 + T)
    res = torch.randn((T, host.d), generator=g).cuda()
    with regime(ctx, 4, True):
        for r in (None, res):
            y = dev.verify_rows(xd, residual=r, out_dtype=torch.float32)
            ctx.sync()
            rows = [dev.forward(xd[i:i + 1], residual=None if r is None else r[i:i + 1],
                                out_dtype=torch.float32) for i in range(T)]
            ctx.sync()
            ref = torch.cat(rows)
            diff = (y != ref).sum().item()
            assert diff == 0, f"{diff} of {y.numel()} outputs differ from decode"
            if r is None:
                y0 = y
        ybf = dev.verify_rows(xd)
        ctx.sync()
        rows = [dev.forward(xd[i:i + 1]) for i in range(T)]
        ctx.sync()
        assert torch.equal(ybf.view(torch.int16), torch.cat(rows).view(torch.int16))
    ids, w, _ = gpu_route(ctx, dev, xd)
    ref_ids, _, gap, _ = ol.router(x)
    ok = gap >= TIE_GAP
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32)[ok], ref_ids[ok])
    y_ref, _, _ = ol.block(x, ids.cpu().numpy().astype(np.uint32), w.cpu().numpy())
    assert rel_l2(y0.cpu().numpy(), y_ref) <= REL_L2


@pytest.mark.parametrize("T,scalar", [(1, 1.0), (3, 0.5), (40, 1.0)])
def test_gemma_fused_norms_match_oracle(ctx, T, scalar):
    """Gemma's layer FFN with the adjacent norms and residuals fused
    (fused_post_attn_setup / fused_layer_tail, fused.metal:190-374) against
    the oracle's restatement: the new hidden rows, and the FFN's part of
    them (the new rows less the post-attention residual), over the fused
    decode kernel (T <= 4) and the batched GEMVs (T = 40)."""
    from oracle import numpy_moe as N

    key = ("gemma_dense_nonorm", 11)
    if key not in _LAYERS:
        host = host_layer("gemma_dense", 11)
        host.router_norm = False
        dev = tb.MoELayer(ctx, tb.upload_host_layer(host), router_norm=False)
        _LAYERS[key] = (host, dev, None)
    host, dev, _ = _LAYERS[key]
    rng = np.random.default_rng(40 + T)
    hidden = host_tokens(T, host.d, 60 + T)
    attn = host_tokens(T, host.d, 61 + T)
    from tsugumi_b200.synthetic import f32_to_bf16_bits

    names = ("post_attn", "pre_ffn", "pre_ffn2", "post_dense", "post_routed", "post_ffn")
    norms = {k: f32_to_bf16_bits(1.0 + 0.2 * rng.standard_normal(host.d).astype(np.float32))
             for k in names}
    want, h_ref = N.gemma_ffn(host, norms, hidden, attn, 1e-6, scalar)
    hd = to_dev(hidden)
    ad = to_dev(attn)
    nd = {k: torch.from_numpy(v.view(np.int16)).cuda().view(torch.bfloat16) for k, v in norms.items()}
    with regime(ctx, 4, True):
        dev.gemma_ffn(hd, ad, nd, eps=1e-6, layer_scalar=scalar)
        ctx.sync()
    got = hd.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert rel_l2(got, want) <= 1e-2
    # the FFN's part alone (the new rows less the post-attention residual)
    d_got, d_want = got / scalar - h_ref, want / scalar - h_ref
    err = rel_l2(d_got, d_want)
    print(f"gemma fused T={T}: rel L2 of the FFN part {err:.3e}")
    assert err <= 3e-2
