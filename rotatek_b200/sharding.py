"""Sharding of the RotateK decode across GPUs (one process per GPU).

A decode call's work splits into independent (batch row, KV head) units: each
unit reads only its own K̃ / V / K_full / V_full rows and writes the outputs of
its own GQA group of query heads, so no partial result crosses GPUs.  Two plans:

* ``batch``: rank r holds batch rows [r*B/N, (r+1)*B/N) for every KV head.  No
  collective at all; each rank's output is its own batch slice.
* ``heads``: rank r holds KV heads [r*H/N, (r+1)*H/N) (and their G query heads
  each) for the whole batch.  The outputs [B, 1, H_q/N, D] are gathered along
  the head axis with one NCCL all_gather per layer when the caller needs every
  head on every rank (the next layer's output projection does).

``auto`` follows the multi-GPU configuration of the benchmark: one KV head per
GPU when N equals the number of KV heads, batch sharding otherwise.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ShardPlan:
    mode: str            # "batch" | "heads"
    rank: int
    world: int
    batch: int           # global batch
    kv_heads: int        # global KV heads
    groups: int          # query heads per KV head
    b0: int              # this rank's batch rows [b0, b1)
    b1: int
    h0: int              # this rank's KV heads [h0, h1)
    h1: int

    @property
    def local_batch(self) -> int:
        return self.b1 - self.b0

    @property
    def local_kv_heads(self) -> int:
        return self.h1 - self.h0

    @property
    def local_q_heads(self) -> int:
        return self.local_kv_heads * self.groups

    @property
    def needs_gather(self) -> bool:
        return self.mode == "heads" and self.world > 1


def plan(rank: int, world: int, batch: int, kv_heads: int, groups: int, mode: str = "auto") -> ShardPlan:
    """This rank's share of a [batch, kv_heads * groups] decode."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if mode == "auto":
        mode = "heads" if world == kv_heads else "batch"
    if mode == "heads":
        if kv_heads % world:
            raise ValueError(f"{kv_heads} KV heads do not split over {world} ranks")
        step = kv_heads // world
        return ShardPlan("heads", rank, world, batch, kv_heads, groups, 0, batch, rank * step, (rank + 1) * step)
    if mode == "batch":
        if batch % world:
            raise ValueError(f"batch {batch} does not split over {world} ranks")
        step = batch // world
        return ShardPlan("batch", rank, world, batch, kv_heads, groups, rank * step, (rank + 1) * step, 0, kv_heads)
    raise ValueError(f"unknown sharding mode {mode!r}")


def shard_inputs(p: ShardPlan, q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse, v_sparse):
    """This rank's slices of full-size decode inputs (views, no copies):
    q [B, H_q, D], per-KV-head tensors [B, H_kv, ...], mask [B, S_f]."""
    bs = slice(p.b0, p.b1)
    hs = slice(p.h0, p.h1)
    qs = slice(p.h0 * p.groups, p.h1 * p.groups)
    return dict(
        q_full=q_full[bs, qs], R_partial=R_partial[bs, hs],
        delta_mu=None if delta_mu is None else delta_mu[bs, hs],
        k_full=k_full[bs, hs], v_full=v_full[bs, hs],
        mask_full=None if mask_full is None else mask_full[bs],
        k_sparse=k_sparse[bs, hs], v_sparse=v_sparse[bs, hs], num_kv_groups=p.groups)


def gather_output(p: ShardPlan, out_local: torch.Tensor, group=None, out: torch.Tensor = None,
                  async_op: bool = False):
    """Every rank's [B_loc, 1, H_q_loc, D] output assembled into [B, 1, H_q, D]
    (one all_gather; along heads for the ``heads`` plan, along the batch for
    ``batch``).  With ``async_op`` returns (out, work)."""
    import torch.distributed as dist

    b, _, hq, d = out_local.shape
    if p.mode == "heads":
        # all_gather along dim 0 needs the head axis outermost: [H_q_loc, B, D]
        src = out_local.reshape(b, hq, d).transpose(0, 1).contiguous()
        buf = torch.empty((p.world * hq, b, d), dtype=out_local.dtype, device=out_local.device)
        work = dist.all_gather_into_tensor(buf, src, group=group, async_op=async_op)

        def finish():
            full = buf.transpose(0, 1).reshape(b, 1, p.world * hq, d)
            if out is not None:
                out.copy_(full)
                return out
            return full
    else:
        src = out_local.contiguous()
        buf = torch.empty((p.world * b, 1, hq, d), dtype=out_local.dtype, device=out_local.device)
        work = dist.all_gather_into_tensor(buf, src, group=group, async_op=async_op)

        def finish():
            if out is not None:
                out.copy_(buf)
                return out
            return buf
    if async_op:
        return finish, work
    return finish()


__all__ = ["ShardPlan", "plan", "shard_inputs", "gather_output"]
