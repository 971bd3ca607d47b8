"""Expert parallelism on 2 GPUs: each rank's output equals the single-GPU
block's output for the same tokens, bit for bit (same kernels, same rows,
same combine order).  Skipped with fewer than two GPUs."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
WORLD = int(os.environ.get("TSG_EP_TEST_WORLD", "2"))
CASES = [
    # config, tokens of rank 0 (rank r has 3r more), skew
    ("tiny", 16, None),
    ("gemma", 700, 1.1),
    ("qwen", 300, None),
    ("gemma_dense", 200, 1.1),
    ("tiny", 0, None),  # rank 0 has no tokens; rank 1 three
]
# (transport, return, dispatch): peer memory as by default (rows stored by
# the dispatch kernel, outputs returned by the copy engines); peer memory
# with both moved by the copy engines; with both stored by kernels (GEMM2's
# epilogue for the outputs); NCCL all-to-all
TRANSPORTS = ((1, 1, 0), (1, 1, 1), (1, 0, 0), (0, 1, 0))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, port: int, q):
    try:
        sys.path.insert(0, str(ROOT))
        import torch.distributed as dist
        import tsugumi_b200 as tb
        from tsugumi_b200 import ep
        from tsugumi_b200.synthetic import device_layer_tensors

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        ctx = tb.Context(rank)
        ctx.set_stream(torch.cuda.current_stream())
        # the expert-parallel path runs the tensor-core contraction for every
        # batch; the single-GPU reference must too (not the batched GEMVs nor
        # the decode kernels, which a rank with a few tokens would reach)
        ctx.set_option("gemv_max_tokens", 0)
        ctx.set_decode_max_tokens(0)
        group = ep.ExpertParallelGroup.from_torch_distributed(ctx)
        msgs = []
        for transport, ret, disp in TRANSPORTS:
            ctx.set_option("ep_transport", transport)
            ctx.set_option("ep_return", ret)
            ctx.set_option("ep_dispatch", disp)
            for name, T0, skew in CASES:
                t = device_layer_tensors(name, 4242, skew, dev)
                full = tb.MoELayer(ctx, t)
                shard = ep.EPMoELayer(group, t)
                g = torch.Generator(device=dev)
                g.manual_seed(77)
                Ts = [T0 + 3 * r for r in range(WORLD)]
                x_all = torch.randn((sum(Ts), t["d"]), generator=g, device=dev).to(torch.bfloat16)
                x = x_all[sum(Ts[:rank]):sum(Ts[:rank + 1])].contiguous()
                want = full.forward(x, out_dtype=torch.float32)
                got = shard.forward(x, out_dtype=torch.float32)
                got2 = shard.forward(x, out_dtype=torch.float32)  # second call, warm buffers
                ctx.sync()
                same = torch.equal(got, want) and torch.equal(got2, want)
                diff = float((got - want).abs().max()) if got.numel() else 0.0
                msgs.append((f"{name} transport {transport} return {ret} dispatch {disp}", same,
                             diff))
                if transport == 1:
                    ph = shard.phase_ms()
                    msgs.append((f"{name} phases", all(v >= 0 for v in ph.values()), 0.0))
                shard.close()
                full.close()
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, "ok", msgs))
    except Exception as exc:  # reported to the parent
        q.put((rank, "error", repr(exc)))


def test_expert_parallel_matches_single_gpu_bit_for_bit():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(WORLD):
            results.append(q.get(timeout=300))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()  # this test's own child, by handle
    for rank, status, payload in results:
        assert status == "ok", f"rank {rank}: {payload}"
        for name, same, diff in payload:
            assert same, f"rank {rank} {name}: max |diff| {diff}"
