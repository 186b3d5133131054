"""Multi-GPU causal attention: batch x head sharding with an NCCL all-gather of the results.

The reference is single-GPU; this layer is the B200 build's scale-out path (one process per
GPU, torch.distributed over NCCL/NVLink).  Work units are (batch, K/V head) pairs: the view
q.view(B * H_kv, group, S, D) puts each unit's query heads next to each other, so the units a
rank owns form ONE contiguous slab of every tensor.  Consequences:
  * a rank's shard is itself a valid kernel input (B' = units, H = group, H_kv = 1), so GQA
    groups stay whole and dK/dV need no cross-rank reduction (no reduce, no all-to-all);
  * all_gather_into_tensor of the per-rank slabs rebuilds the full [B, H, S, D] tensor in place,
    with no permutation copy.
The only collectives are the all-gathers of O (forward) and of dQ, dK, dV (backward).  Each rank
holds the full inputs (replicated) and receives the full outputs, which is the drop-in
semantics of the single-GPU functions.  Requires (B * H_kv) % world_size == 0.
"""
import importlib.util
import os
import sys

import torch
import torch.distributed as dist


def _backward_module():
    """attention/backward/fused_backward.py, loaded by path under one shared module name."""
    if __package__:
        from .backward import fused_backward
        return fused_backward
    name = "_fa_b200_fused_backward"
    mod = sys.modules.get(name)
    if mod is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "backward", "fused_backward.py")
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return mod


def shard_units(B, H_kv, world, rank):
    """[u0, u1): the (batch, K/V head) units of `rank`; units are numbered b * H_kv + g."""
    units = B * H_kv
    if units % world:
        raise ValueError(f"B * H_kv = {units} units cannot be split evenly over {world} ranks")
    per = units // world
    return rank * per, (rank + 1) * per


def _unit_view(t, H_kv):
    B, H, S, D = t.shape
    return t.view(B * H_kv, H // H_kv, S, D)


class ShardedFusedAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, tile_m, tile_n, group):
        fb = _backward_module()
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        fb._check(q, k, v, tile_m, tile_n)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        H_kv = k.shape[1]
        u0, u1 = shard_units(q.shape[0], H_kv, world, rank)
        ql = _unit_view(q, H_kv)[u0:u1]
        kl = _unit_view(k, H_kv)[u0:u1]
        vl = _unit_view(v, H_kv)[u0:u1]
        ol, lse = fb._forward(ql, kl, vl, tile_m, tile_n)
        o = torch.empty_like(q)
        dist.all_gather_into_tensor(_unit_view(o, H_kv), ol, group=group)
        ctx.save_for_backward(ql, kl, vl, ol, lse)
        ctx.meta = (tile_m, tile_n, group, H_kv, u0, u1, q.shape, k.shape)
        return o

    @staticmethod
    def backward(ctx, do):
        fb = _backward_module()
        ql, kl, vl, ol, lse = ctx.saved_tensors
        tile_m, tile_n, group, H_kv, u0, u1, qshape, kshape = ctx.meta
        do = do.contiguous()
        if do.dtype != ql.dtype:
            do = do.to(ql.dtype)
        dol = _unit_view(do, H_kv)[u0:u1]
        dql, dkl, dvl = fb._backward(ql, kl, vl, ol, lse, dol, tile_m, tile_n)
        dq = torch.empty(qshape, device=do.device, dtype=do.dtype)
        dk = torch.empty(kshape, device=do.device, dtype=do.dtype)
        dv = torch.empty(kshape, device=do.device, dtype=do.dtype)
        dist.all_gather_into_tensor(_unit_view(dq, H_kv), dql, group=group)
        dist.all_gather_into_tensor(_unit_view(dk, H_kv), dkl, group=group)
        dist.all_gather_into_tensor(_unit_view(dv, H_kv), dvl, group=group)
        return dq, dk, dv, None, None, None


def sharded_attention_autograd(q, k, v, tile_m=64, tile_n=64, group=None):
    """Causal (GQA) attention with autograd, sharded over the ranks of `group`.

    q [B, H, S, D], k and v [B, H_kv, S, D] are replicated on every rank; every rank returns the
    full output (and, in backward, the full dQ, dK, dV)."""
    return ShardedFusedAttentionFn.apply(q, k, v, tile_m, tile_n, group)


def sharded_attention(q, k, v, tile_m=64, tile_n=64, group=None):
    """Forward only (no autograd graph): shard, compute, all-gather O."""
    with torch.no_grad():
        return ShardedFusedAttentionFn.apply(q, k, v, tile_m, tile_n, group)
