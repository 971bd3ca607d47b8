"""The expert-parallel protocol on two CPU ranks (gloo), with the oracle
doing the arithmetic: route, sort the pairs by expert (so each owner's pairs
form one run), exchange per-expert counts with a status word, plan and size
the buffers, agree on a second status word, send each row to its expert's
owner, compute the owned experts on the received rows, return the outputs,
combine in rank order.  Each rank's result must equal the oracle's whole
block for its tokens; and a failure injected on one rank's host side (in its
routing, or in its plan and buffers) must end the call on every rank with an
error at the next agreement point -- no rank left waiting in an exchange.
The steps are those of tsg_ep_moe_block_forward."""

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

        layer = O.OracleLayer(host_layer("tiny", 11))
        T = 24
        x_all = host_tokens(WORLD * T, layer.h.d, 5)
        x = np.ascontiguousarray(x_all[rank * T:(rank + 1) * T])
        try:
            got = ep_forward(layer, x, rank, WORLD, a2a, fail_at if rank == fail_rank else None)
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


@pytest.mark.parametrize("fail_rank,fail_at", [(1, "route"), (0, "plan")])
def test_a_rank_failure_ends_the_call_on_every_rank(fail_rank, fail_at):
    """A host-side failure on one rank (before its counts go out, or while it
    sizes its buffers after them) ends the call with an error on every rank
    at the next agreement point; no rank is left in an exchange (the queue
    read would time out)."""
    results = _run_ranks(fail_rank, fail_at)
    assert len(results) == WORLD
    for rank, status, payload in results:
        assert status == "ep_error", f"rank {rank}: {status} {payload}"
        if rank == fail_rank:
            assert "injected" in payload
        else:
            assert f"rank {fail_rank} failed" in payload
