"""Expert-parallel MoeVerify and MoeDecode over torch.distributed: one process per GPU.

The reference runs both ops on one GPU (MoeVerify src/bolt_ops.cu:1178-1257, MoeDecode
:589-619).  Here rank g of G owns experts [g*E//G, (g+1)*E//G) and holds only their weights.
Every rank sees the same routing (MoeRoute is replicated), computes the fp32 partial output of
the (token, expert) pairs whose expert is local (``bolt_moe_verify_shard`` /
``bolt_moe_decode_shard``), and the partials are summed with one all-reduce (NCCL over NVLink on
GPUs) before the bf16 cast.  Summing in fp32 keeps the result within fp32 reassociation of the
single-GPU op; a bf16 reduction would add a second rounding.

The per-shard compute and the cast are the CUDA ops; both can be replaced by callables, which
the CPU tests use to run the distributed logic on ``gloo`` ranks with the oracle as the shard
computation.
"""
from __future__ import annotations

import os
from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["expert_range", "ShardedMoeVerify", "ShardedMoeDecode", "PeerReducer"]


def expert_range(num_experts: int, rank: int, world: int):
    """[e_begin, e_end) of the experts owned by ``rank``: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("expert_range: need 0 <= rank < world")
    return rank * num_experts // world, (rank + 1) * num_experts // world


class PeerReducer:
    """Peer-visible buffers of ``bolt_moe_verify_shard_allreduce`` for the ranks of ``group``
    (CUDA, one process per GPU): torch symmetric memory maps every rank's buffer -- two halves of
    ``world`` slots of ``max_rows * 1024`` fp32 partials (slot q receives rank q's partial), then the
    flag words, zeroed here -- into every peer; the call counters are this rank's.  Only plain peer loads and stores touch it, so torch's NVLink
    multicast binding is switched off (unless the caller set TORCH_SYMM_MEM_DISABLE_MULTICAST).
    Create it on every rank (a collective) before stream capture, and make the same sequence of
    calls on every rank."""

    CTAS = 16  # kPeerReduceCtas of the kernel

    def __init__(self, group=None, max_rows: int = 8, device=None):
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        group = group if group is not None else dist.group.WORLD
        world = dist.get_world_size(group)
        self.half = int(max_rows) * 1024
        self.buf = symm_mem.empty(2 * world * self.half + self.CTAS * world, dtype=torch.float32, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.rank, self.world = self.handle.rank, self.handle.world_size
        self.bufs_dev = self.handle.buffer_ptrs_dev
        self.counters = torch.zeros(self.CTAS, dtype=torch.int32, device=device)


class ShardedMoeVerify:
    """MoeVerify with experts sharded over the ranks of ``group`` (``iq2`` as the op's attribute).

    ``weights`` are this rank's slices ``(fc1_w, fc1_s, fc2_w, fc2_s)`` of experts
    [e_begin, e_end) (use :meth:`local_slice` to cut them from full-size tensors).
    """

    def __init__(self, num_experts: int, topk: int, iq2: int = 0, group=None,
                 shard_fn: Optional[Callable] = None, cast_fn: Optional[Callable] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.num_experts = int(num_experts)
        self.topk = int(topk)
        self.iq2 = int(iq2)
        self.e_begin, self.e_end = expert_range(self.num_experts, self.rank, self.world)
        self.shard_fn = shard_fn if shard_fn is not None else self._cuda_shard
        self.cast_fn = cast_fn if cast_fn is not None else self._cuda_cast

    def local_slice(self, t: torch.Tensor) -> torch.Tensor:
        """This rank's experts of a full [E, ...] weight or scale tensor (contiguous copy)."""
        return t[self.e_begin:self.e_end].contiguous()

    def _cuda_shard(self, z, idx, w, weights, e_begin, e_end):
        from . import ops
        out_partial, _h, _part, _meta = ops.moe_verify_shard(z, idx, w, *weights, topk=self.topk, iq2=self.iq2,
                                                             e_begin=e_begin, e_end=e_end,
                                                             num_experts=self.num_experts)
        return out_partial

    @staticmethod
    def _cuda_cast(t):
        from . import ops
        return ops.f32_to_bf16(t)

    def partial(self, z, idx, w, weights) -> torch.Tensor:
        """fp32 [R, 1024]: sum over this rank's pairs of w * part."""
        return self.shard_fn(z, idx, w, weights, self.e_begin, self.e_end)

    def fused(self, z, idx, w, weights, reducer: "PeerReducer", out=None, outputs=None) -> torch.Tensor:
        """As ``__call__``, with the partials summed through peer memory inside the op's last
        kernel (``bolt_moe_verify_shard_allreduce``) instead of an NCCL all-reduce and a cast."""
        from . import ops
        return ops.moe_verify_shard_allreduce(z, idx, w, *weights, topk=self.topk, iq2=self.iq2, e_begin=self.e_begin,
                                              e_end=self.e_end, reducer=reducer, num_experts=self.num_experts,
                                              out=out, outputs=outputs)

    def __call__(self, z, idx, w, weights) -> torch.Tensor:
        """bf16 [R, 1024] MoeVerify output, identical on every rank."""
        p = self.partial(z, idx, w, weights)
        if self.world > 1:
            dist.all_reduce(p, op=dist.ReduceOp.SUM, group=self.group)
        return self.cast_fn(p)


class ShardedMoeDecode(ShardedMoeVerify):
    """MoeDecode (int4, exact fp32 weight contract) with experts sharded over ``group``."""

    def __init__(self, num_experts: int, topk: int, group=None, shard_fn: Optional[Callable] = None,
                 cast_fn: Optional[Callable] = None):
        super().__init__(num_experts, topk, 0, group, shard_fn, cast_fn)

    def _cuda_shard(self, z, idx, w, weights, e_begin, e_end):
        from . import ops
        out_partial, _h, _part = ops.moe_decode_shard(z, idx, w, *weights, topk=self.topk, e_begin=e_begin,
                                                      e_end=e_end, num_experts=self.num_experts)
        return out_partial
