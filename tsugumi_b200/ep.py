"""Expert parallelism across the GPUs of one node (one process per GPU).

The experts of a layer are split contiguously over R ranks; each rank routes
its own tokens and the library moves token rows to the experts' owners and
the expert outputs back over NCCL (``tsg_ep_moe_block_forward``).  The
reference runs on one device, so there is no reference counterpart; each
rank's arithmetic is the single-GPU block's, and the outputs are bit-equal to
it.
"""

from __future__ import annotations

import ctypes as C

from . import _abi
from ._abi import check
from .moe import Context, MoELayer, _ptr

UNIQUE_ID_BYTES = 128


def new_unique_id() -> bytes:
    """A fresh NCCL unique id (made on one rank, handed to all)."""
    lib = _abi.load()
    buf = (C.c_uint8 * UNIQUE_ID_BYTES)()
    check(lib.tsg_ep_unique_id(C.cast(buf, C.c_void_p)))
    return bytes(buf)


class ExpertParallelGroup:
    """This process's context joined to an expert-parallel group."""

    def __init__(self, ctx: Context, rank: int, world: int, unique_id: bytes):
        if len(unique_id) != UNIQUE_ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        buf = (C.c_uint8 * UNIQUE_ID_BYTES).from_buffer_copy(unique_id)
        check(ctx.lib.tsg_ep_init(ctx.h, C.cast(buf, C.c_void_p), rank, world), ctx.h)
        self.ctx, self.rank, self.world = ctx, rank, world

    @classmethod
    def from_torch_distributed(cls, ctx: Context) -> "ExpertParallelGroup":
        """Uses an initialised torch.distributed process group (any backend)
        only to hand rank 0's NCCL unique id to every rank."""
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [new_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(ctx, rank, world, obj[0])

    def expert_range(self, num_experts: int) -> tuple[int, int]:
        """[first, first + count) experts owned by this rank."""
        if num_experts % self.world:
            raise ValueError("numExperts must be a multiple of the group size")
        n = num_experts // self.world
        return self.rank * n, n


def shard_tensors(t: dict, group: ExpertParallelGroup) -> dict:
    """This rank's view of a layer's tensors (as made by
    synthetic.device_layer_tensors): all router rows and the shared expert,
    and the blobs of the rank's own experts."""
    first, count = group.expert_range(t["num_experts"])
    s = dict(t)
    stride = t["expert_stride"]
    s["experts"] = t["experts"][first * stride:(first + count) * stride]
    return s


class EPMoELayer(MoELayer):
    """One rank's shard of a MoE layer."""

    def __init__(self, group: ExpertParallelGroup, t: dict, **kw):
        self.group = group
        self.expert_first, self.expert_count = group.expert_range(t["num_experts"])
        super().__init__(group.ctx, shard_tensors(t, group), **kw)

    def forward(self, hidden, y=None, residual=None, out_dtype=None):
        """tsg_ep_moe_block_forward: collective over the group; each rank
        passes its own tokens."""
        import torch

        T = hidden.shape[0]
        if y is None:
            y = torch.empty((T, self.d), dtype=out_dtype or torch.bfloat16, device=hidden.device)
        dt = _abi.DTYPE_F32 if y.dtype == torch.float32 else _abi.DTYPE_BF16
        check(self.ctx.lib.tsg_ep_moe_block_forward(
            self.ctx.h, self.h, self.expert_first, _ptr(hidden), hidden.stride(0), T,
            _ptr(residual), _ptr(y), y.stride(0), dt), self.ctx.h)
        return y

    PHASES = ("route", "exchange_plan", "dispatch", "expand", "gate_up", "down_return", "barrier",
              "combine")

    def phase_ms(self) -> dict:
        """Device time of each phase of the context's last peer-transport
        call (tsg_ep_phase_ms); waits for it."""
        buf = (C.c_float * len(self.PHASES))()
        check(self.ctx.lib.tsg_ep_phase_ms(self.ctx.h, C.cast(buf, C.c_void_p), len(self.PHASES)),
              self.ctx.h)
        return {k: float(v) for k, v in zip(self.PHASES, buf)}
