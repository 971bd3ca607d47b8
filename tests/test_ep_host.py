"""The expert-parallel protocol on two CPU ranks (gloo), with the oracle
doing the arithmetic: route, sort the pairs by expert (so each owner's pairs
form one run), exchange per-expert counts with a status word, plan and size
the buffers, agree on a second status word, send each row to its expert's
owner, compute the owned experts on the received rows, return the outputs,
combine in rank order.  Each rank's result must equal the oracle's whole
block for its tokens; and a failure injected on one rank's host side (in its
routing, or in its plan and buffers) must end the call on every rank with an
error at the next agreement point -- no rank left waiting in an exchange.
The steps are those of tsg_ep_moe_block_forward; ep_forward_peer mirrors its
peer-memory transport the same way (one all-gather of counts and statuses,
a plan every rank computes alike, a growth agreed through its handle
exchange)."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class EPError(RuntimeError):
    pass


def ep_forward(layer, x_local: np.ndarray, rank: int, world: int, a2a,
               fail_at: str | None = None) -> np.ndarray:
    """One rank of the protocol.  `a2a(send, send_splits, recv_splits)` is an
    all-to-all of a 1-D or 2-D numpy array along axis 0.  `fail_at` injects
    a host-side failure on this rank: "route" (before the counts are sent) or
    "plan" (after them, while sizing the buffers)."""
    from oracle import oracle as O

    h = layer.h
    E, K, D = h.num_experts, h.top_k, h.d
    El = E // world
    T = x_local.shape[0]
    local_error = None
    counts = np.zeros(E, np.int64)
    try:
        if fail_at == "route":
            raise MemoryError("injected: routing launch failed")
        ids, w, _, _ = layer.router(x_local)
        pairs = O.make_pairs(ids)
        g = O.group_pairs(pairs, T, K, E, 16)
        sp = g["sorted_pairs"]
        counts = g["counts"].astype(np.int64)
    except MemoryError as exc:
        local_error = str(exc)
        counts = np.zeros(E, np.int64)  # (what is sent is not read)

    def agree(ok: bool) -> None:
        st = a2a(np.full(world, 1 if ok else 0, np.int64), [1] * world, [1] * world)
        if local_error:
            raise EPError(local_error)
        bad = [q for q in range(world) if st[q] == 0]
        if bad:
            raise EPError(f"rank {bad[0]} failed before the row exchange")

    # agreement 1: per-expert counts to the owners, with each rank's status
    recv_counts = a2a(counts, [El] * world, [El] * world).reshape(world, El)
    agree(local_error is None)
    send_cnt = [int(counts[q * El:(q + 1) * El].sum()) for q in range(world)]
    recv_cnt = [int(recv_counts[q].sum()) for q in range(world)]
    # the plan and its buffers (nothing is allocated after agreement 2)
    try:
        if fail_at == "plan":
            raise MemoryError("injected: buffer allocation failed")
        if sum(send_cnt) != T * K:
            raise MemoryError("pair counts do not add up")
    except MemoryError as exc:
        local_error = str(exc)
    agree(local_error is None)
    # dispatch rows (bf16 bits) and their local expert ids, run by run
    rows = x_local[sp["token"]].astype(np.int32)
    local_e = (sp["expert"] % El).astype(np.int64)
    rrows = a2a(rows, send_cnt, recv_cnt)
    re = a2a(local_e, send_cnt, recv_cnt)
    # the owner computes its experts on the rows it holds
    if rrows.shape[0]:
        first = rank * El
        # every slot names the row's expert; only slot 0 has weight
        force = np.repeat((first + re).astype(np.uint32)[:, None], K, axis=1)
        wt = np.zeros((rrows.shape[0], K), np.float32)
        wt[:, 0] = 1.0
        out, _, _ = layer.block(rrows.astype(np.uint16), force, wt)
    else:
        out = np.zeros((0, D), np.float32)
    # outputs back to the tokens' ranks, into their sorted positions
    ret = a2a(out, recv_cnt, send_cnt)
    pos = np.empty(T * K, np.int64)
    pos[sp["token"] * K + sp["rank"]] = np.arange(T * K)
    y = np.zeros((T, D), np.float64)
    for k in range(K):
        y += w[:, k:k + 1].astype(np.float64) * ret[pos[np.arange(T) * K + k]]
    return y.astype(np.float32)


def ep_forward_peer(layer, x_local: np.ndarray, rank: int, world: int, all_gather, a2a,
                    caps: dict, fail_at: str | None = None) -> np.ndarray:
    """One rank of the peer-memory transport (tsg_ep_moe_block_forward with
    ep_transport 1).  One all-gather carries every rank's per-expert counts,
    its token rows per owner, T and a status word; from it every rank
    computes the same plan for all ranks (pair runs, row and map offsets in
    each owner's buffers, every buffer's need), so a growth is decided alike
    everywhere and its handle exchange carries a status word.  The peer
    stores are emulated by an all-to-all whose pieces land at the offsets the
    plan gives.  `fail_at`: "route" (before the counts go out) or "grow" (an
    allocation of a growth)."""
    from oracle import oracle as O

    h = layer.h
    E, K, D = h.num_experts, h.top_k, h.d
    El = E // world
    T = x_local.shape[0]
    ok = True
    counts = np.zeros(E, np.int64)
    tok = np.zeros(world, np.int64)
    try:
        if fail_at == "route":
            raise MemoryError("injected: routing launch failed")
        ids, w, _, _ = layer.router(x_local)
        pairs = O.make_pairs(ids)
        g = O.group_pairs(pairs, T, K, E, 16)
        sp = g["sorted_pairs"]
        counts = g["counts"].astype(np.int64)
        owner_of = ids.astype(np.int64) // El  # [T, K]
        on = np.stack([(owner_of == o).any(axis=1) for o in range(world)])  # [world, T]
        slots = np.where(on, np.cumsum(on, axis=1) - 1, -1)
        tok = on.sum(axis=1)
    except MemoryError as exc:
        ok, local_error = False, str(exc)
    # agreement: every rank's words
    words = np.concatenate([counts, tok, [T, 1 if ok else 0]])
    M = all_gather(words).reshape(world, -1)
    if not ok:
        raise EPError(local_error)
    bad = [q for q in range(world) if M[q, E + world + 1] != 1]
    if bad:
        raise EPError(f"rank {bad[0]} failed before the row exchange")
    # the plan, the same on every rank
    Tq = M[:, E + world]
    snd = np.array([[M[q, o * El:(o + 1) * El].sum() for o in range(world)] for q in range(world)])
    soff = np.concatenate([np.zeros((world, 1), np.int64), np.cumsum(snd, axis=1)[:, :-1]], axis=1)
    tokm = M[:, E:E + world]
    assert (snd.sum(axis=1) == Tq * K).all()
    rpo = np.concatenate([np.zeros((1, world), np.int64), np.cumsum(snd, axis=0)[:-1]], axis=0)  # [q, o]
    rro = np.concatenate([np.zeros((1, world), np.int64), np.cumsum(tokm, axis=0)[:-1]], axis=0)
    need = {"rows": tokm.sum(axis=0) * D, "map": snd.sum(axis=0), "ret": Tq * K * D}
    grow = any((need[k] > caps[k]).any() for k in need)
    if grow:
        st = all_gather(np.array([0 if fail_at == "grow" else 1]))
        bad = [q for q in range(world) if st[q] != 1]
        if bad:
            raise EPError(f"rank {bad[0]} could not allocate its exchange buffers")
        for k in need:
            caps[k] = np.maximum(caps[k], need[k] + need[k] // 4)
    # dispatch: a token row once per owner, and each pair's row index
    send_rows, send_map, rs, ms = [], [], [], []
    for o in range(world):
        toks = np.nonzero(slots[o] >= 0)[0]
        send_rows.append(x_local[toks].astype(np.int32))
        run = sp[soff[rank, o]:soff[rank, o] + snd[rank, o]]
        assert (run["expert"] // El == o).all()
        send_map.append(rro[rank, o] + slots[o][run["token"]])
        rs.append(len(toks))
        ms.append(len(run))
    rr = [int(tokm[q, rank]) for q in range(world)]
    rm = [int(snd[q, rank]) for q in range(world)]
    rows_in = a2a(np.concatenate(send_rows).reshape(-1, D), rs, rr)
    map_in = a2a(np.concatenate(send_map), ms, rm)
    # the pieces land where the plan says: source q's rows at rro[q, me],
    # its map entries at rpo[q, me]
    assert rows_in.shape[0] == tokm[:, rank].sum() and map_in.shape[0] == snd[:, rank].sum()
    xp = rows_in[map_in]  # the owner's expansion
    # the owner computes its experts, one run per (source rank, local expert)
    out = np.zeros((xp.shape[0], D), np.float32)
    for q in range(world):
        row = rpo[q, rank]
        for j in range(El):
            c = int(M[q, rank * El + j])
            if c:
                force = np.full((c, K), rank * El + j, np.uint32)
                wt = np.zeros((c, K), np.float32)
                wt[:, 0] = 1.0
                out[row:row + c], _, _ = layer.block(xp[row:row + c].astype(np.uint16), force, wt)
            row += c
    # returned to each source rank at soff[q, me] of its sorted order
    ret = a2a(out, rm, ms)
    pos = np.empty(T * K, np.int64)
    pos[sp["token"] * K + sp["rank"]] = np.arange(T * K)
    y = np.zeros((T, D), np.float64)
    for k in range(K):
        y += w[:, k:k + 1].astype(np.float64) * ret[pos[np.arange(T) * K + k]]
    return y.astype(np.float32)


def _rank_main(rank: int, port: int, q, fail_rank: int = -1, fail_at: str | None = None):
    try:
        sys.path.insert(0, str(ROOT))
        import torch.distributed as dist
        from oracle import oracle as O
        from tsugumi_b200.synthetic import host_layer, host_tokens

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)

        def a2a(arr, send_splits, recv_splits):
            arr = np.ascontiguousarray(arr)
            tail = arr.shape[1:]
            src = torch.from_numpy(arr.reshape(arr.shape[0], -1) if tail else arr)
            out = torch.empty((sum(recv_splits),) + tuple(src.shape[1:]), dtype=src.dtype)
            dist.all_to_all_single(out, src, recv_splits, send_splits)
            return out.numpy().reshape((sum(recv_splits),) + tail)

        def all_gather(arr):
            src = torch.from_numpy(np.ascontiguousarray(arr, np.int64))
            out = [torch.empty_like(src) for _ in range(WORLD)]
            dist.all_gather(out, src)
            return torch.cat(out).numpy()

        layer = O.OracleLayer(host_layer("tiny", 11))
        T = 24
        x_all = host_tokens(WORLD * T, layer.h.d, 5)
        x = np.ascontiguousarray(x_all[rank * T:(rank + 1) * T])
        my_fail = fail_at if rank == fail_rank else None
        try:
            if fail_at in (None, "route_peer", "grow"):
                caps = {"rows": np.zeros(WORLD, np.int64), "map": np.zeros(WORLD, np.int64),
                        "ret": np.zeros(WORLD, np.int64)}
                peer_fail = "route" if my_fail == "route_peer" else my_fail
                got = ep_forward_peer(layer, x, rank, WORLD, all_gather, a2a, caps, peer_fail)
                if fail_at is None:  # a second call: no growth, the same result
                    got2 = ep_forward_peer(layer, x, rank, WORLD, all_gather, a2a, caps)
                    assert np.array_equal(got, got2)
                    got1 = ep_forward(layer, x, rank, WORLD, a2a)
                    assert np.allclose(got, got1, rtol=0, atol=1e-6)
            else:
                got = ep_forward(layer, x, rank, WORLD, a2a, my_fail)
        except EPError as exc:
            dist.destroy_process_group()
            q.put((rank, "ep_error", str(exc)))
            return
        want, _, _ = layer.block(x)
        rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
        dist.destroy_process_group()
        q.put((rank, "ok", rel))
    except Exception as exc:
        q.put((rank, "error", repr(exc)))


def _run_ranks(fail_rank=-1, fail_at=None):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q, fail_rank, fail_at))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(WORLD):
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()  # this test's own child, by handle
    return sorted(results)


def test_expert_parallel_protocol_on_two_gloo_ranks():
    for rank, status, payload in _run_ranks():
        assert status == "ok", f"rank {rank}: {payload}"
        assert payload < 1e-6, f"rank {rank}: rel L2 {payload}"


@pytest.mark.parametrize("fail_rank,fail_at", [(1, "route"), (0, "plan"), (0, "route_peer"),
                                               (1, "grow")])
def test_a_rank_failure_ends_the_call_on_every_rank(fail_rank, fail_at):
    """A host-side failure on one rank (before its counts go out, or while it
    sizes its buffers after them) ends the call with an error on every rank
    at the next agreement point; no rank is left in an exchange (the queue
    read would time out)."""
    results = _run_ranks(fail_rank, fail_at)
    assert len(results) == WORLD
    for rank, status, payload in results:
        assert status == "ep_error", f"rank {rank}: {status} {payload}"
        if fail_at == "grow":
            assert f"rank {fail_rank} could not allocate" in payload
        elif rank == fail_rank:
            assert "injected" in payload
        else:
            assert f"rank {fail_rank} failed" in payload
