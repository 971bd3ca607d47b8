"""tsg_moe_group_pairs_noalloc: the permutation with static device scratch.

The variant must give exactly what tsg_moe_group_pairs gives (the grouping is
integer work, so the tolerance is zero), including on two calls enqueued back
to back, must reject inputs above its static limits with a clear error before
doing any work, and must not change the device's free memory.  This file
creates its own context, so it passes alone or after every other test.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tsugumi_b200 as tb  # noqa: E402
from tsugumi_b200 import _abi  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_PAIRS = 65536
TSG_ERR_UNSUPPORTED_SHAPE = 2


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _case(T, K, E, seed, keys=False):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w16 = rng.integers(0, 0x3C00, (T, K)).astype(np.int32)
    tok = np.repeat(np.arange(T, dtype=np.int32), K)
    rank = np.tile(np.arange(K, dtype=np.int32), T)
    pairs = np.stack([tok, ids.reshape(-1), rank, w16.reshape(-1)], 1)[rng.permutation(T * K)]
    sort_keys = rng.integers(0, 5, E).astype(np.uint64) if keys else None
    return np.ascontiguousarray(pairs), sort_keys


class _Out:
    def __init__(self, n, E):
        dev = torch.device("cuda", 0)
        self.sorted_pairs = torch.full((max(n, 1), 4), -7, dtype=torch.int32, device=dev)
        self.offsets = torch.full((E,), -7, dtype=torch.int32, device=dev)
        self.counts = torch.full((E,), -7, dtype=torch.int32, device=dev)
        self.groups = torch.full((E, 3), -7, dtype=torch.int32, device=dev)
        self.tiles = torch.full((E, 4), -7, dtype=torch.int32, device=dev)
        self.n_groups = torch.full((1,), -7, dtype=torch.int32, device=dev)
        self.n_tiles = torch.full((1,), -7, dtype=torch.int32, device=dev)

    def host(self, n):
        g = int(self.n_groups.item())
        t = int(self.n_tiles.item())
        return dict(sorted_pairs=self.sorted_pairs[:n].cpu().numpy(),
                    offsets=self.offsets.cpu().numpy(), counts=self.counts.cpu().numpy(),
                    groups=self.groups[:g].cpu().numpy(), tiles=self.tiles[:t].cpu().numpy(),
                    n_groups=g, n_tiles=t)


def _call(ctx, fn_name, pairs, T, K, E, tec, keys, brk, out):
    n = T * K
    fn = getattr(ctx.lib, fn_name)
    return fn(ctx.h, _ptr(pairs) if n else None, n, T, K, E, tec, _ptr(keys),
              0 if keys is None else int(keys.numel()), -1 if brk is None else brk,
              _ptr(out.sorted_pairs), _ptr(out.offsets), _ptr(out.counts), _ptr(out.groups),
              _ptr(out.n_groups), _ptr(out.tiles), _ptr(out.n_tiles))


CASES = [
    # T, K, E, tile_expert_count, sort keys, tile break, seed
    (4096, 8, 128, 16, False, None, 1),
    (300, 8, 256, 5, True, 3, 2),
    (8192, 8, 512, 16, True, None, 3),   # exactly the static limit of pairs
    (37, 4, 16, 2, False, None, 4),
]


@pytest.fixture(scope="module")
def ctx():
    c = tb.Context(0)
    yield c
    c.close()


def _dev(case):
    T, K, E, tec, keys, brk, seed = case
    pairs, sort_keys = _case(T, K, E, seed, keys)
    p = torch.from_numpy(pairs).cuda()
    k = None if sort_keys is None else torch.from_numpy(sort_keys.view(np.int64)).cuda()
    return (p, T, K, E, tec, k, brk)


def _assert_same(a, b):
    for key in ("sorted_pairs", "offsets", "counts", "groups", "tiles"):
        assert np.array_equal(a[key], b[key]), key
    assert a["n_groups"] == b["n_groups"] and a["n_tiles"] == b["n_tiles"]


@pytest.mark.parametrize("first,second", [(0, 1), (2, 3), (1, 0)])
def test_noalloc_matches_existing_entry_point_on_two_calls_in_a_row(ctx, first, second):
    args = [_dev(CASES[first]), _dev(CASES[second])]
    want = []
    for a in args:
        out = _Out(a[1] * a[2], a[3])
        _abi.check(_call(ctx, "tsg_moe_group_pairs", *a, out), ctx.h)
        ctx.sync()
        want.append(out.host(a[1] * a[2]))
    # the two no-alloc calls are enqueued back to back with no host sync
    outs = [_Out(a[1] * a[2], a[3]) for a in args]
    for a, out in zip(args, outs):
        _abi.check(_call(ctx, "tsg_moe_group_pairs_noalloc", *a, out), ctx.h)
    ctx.sync()
    for a, out, w in zip(args, outs, want):
        _assert_same(out.host(a[1] * a[2]), w)


@pytest.mark.parametrize("case", [
    CASES[0],                                # multi-chunk counting sort
    CASES[3],                                # one-CTA path (fits one chunk)
    (200, 8, 512, 16, False, None, 5),       # one-CTA path at 512 experts
])
def test_noalloc_leaves_free_device_memory_unchanged(case):
    c = tb.Context(0)  # fresh context: no workspace reserved yet
    try:
        a = _dev(case)
        out = _Out(a[1] * a[2], a[3])
        _abi.check(_call(c, "tsg_moe_group_pairs_noalloc", *a, out), c.h)
        c.sync()
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info(0)
        for _ in range(3):
            _abi.check(_call(c, "tsg_moe_group_pairs_noalloc", *a, out), c.h)
        c.sync()
        free1, _ = torch.cuda.mem_get_info(0)
        assert free1 == free0
    finally:
        c.close()


def test_noalloc_rejects_inputs_above_its_static_limits(ctx):
    out = _Out(1, 1)
    # no kernel runs: the limits are checked before any pointer is used
    st = _call(ctx, "tsg_moe_group_pairs_noalloc", None, MAX_PAIRS + 1, 1, 4, 16, None, None, out)
    assert st == TSG_ERR_UNSUPPORTED_SHAPE
    assert "static scratch limit of 65536 pairs" in ctx.last_error()
    st = _call(ctx, "tsg_moe_group_pairs_noalloc", None, 1, 1, 513, 16, None, None, out)
    assert st == TSG_ERR_UNSUPPORTED_SHAPE
    assert "513 experts exceed its static scratch limit of 512" in ctx.last_error()


def test_noalloc_reports_bad_pairs_like_the_existing_entry_point(ctx):
    dup = torch.tensor([[0, 0, 0, 1], [0, 1, 0, 2]], dtype=torch.int32, device="cuda")
    out = _Out(2, 2)
    _abi.check(_call(ctx, "tsg_moe_group_pairs_noalloc", dup, 1, 2, 2, 1, None, None, out), ctx.h)
    with pytest.raises(tb.PrefillMoEGroupingError, match="duplicate route pair for token 0"):
        ctx.sync()
    # the scratch is usable again afterwards
    a = _dev(CASES[3])
    want_out = _Out(a[1] * a[2], a[3])
    _abi.check(_call(ctx, "tsg_moe_group_pairs", *a, want_out), ctx.h)
    got_out = _Out(a[1] * a[2], a[3])
    _abi.check(_call(ctx, "tsg_moe_group_pairs_noalloc", *a, got_out), ctx.h)
    ctx.sync()
    _assert_same(got_out.host(a[1] * a[2]), want_out.host(a[1] * a[2]))
