"""Multi-GPU causal attention: batch x head sharding with an NCCL all-gather of the results.

The reference is single-GPU; this layer is the B200 build's scale-out path (one process per
GPU, torch.distributed over NCCL/NVLink).  Work units are (batch, K/V head) pairs: the view
q.view(B * H_kv, group, S, D) puts each unit's query heads next to each other, so any run of
consecutive units is ONE contiguous slab of every tensor.  Consequences:
  * a run of units is itself a valid kernel input (B' = units, H = group, H_kv = 1), so GQA
    groups stay whole and dK/dV need no cross-rank reduction (no reduce, no all-to-all);
  * all_gather_into_tensor of equal per-rank runs that sit side by side in rank order rebuilds a
    contiguous slab of the full [B, H, S, D] tensor in place, with no permutation copy.

Pipelining.  A rank's units are split into C chunks, and chunk c of rank r is the run of units
[(c * W + r) * cs, (c * W + r + 1) * cs) (W ranks, cs units per chunk).  Chunk c of all ranks
together is then the contiguous slab [c * W * cs, (c + 1) * W * cs), so its all-gather can be
issued as soon as chunk c is computed and runs on a side stream while chunk c + 1 computes.
With C = 1 this is the plain contiguous split.  Only the last chunk's gathers are exposed.

The only collectives are the all-gathers of O (forward) and of dQ, dK, dV (backward), and every
rank issues them in the same order.  They overlap the kernels only if NCCL's blocks get SMs while
the attention kernels (one CTA per SM) are queued: create the process group with
ProcessGroupNCCL.Options(is_high_priority_stream=True), as bench.py does.  Each rank holds the
full inputs (replicated) and receives the full outputs, which is the drop-in semantics of the
single-GPU functions.  Requires (B * H_kv) % world_size == 0.
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
    """[u0, u1): the contiguous run of (batch, K/V head) units of `rank` when the work is not
    chunked; units are numbered b * H_kv + g."""
    units = B * H_kv
    if units % world:
        raise ValueError(f"B * H_kv = {units} units cannot be split evenly over {world} ranks")
    per = units // world
    return rank * per, (rank + 1) * per


# Fewer units than this per chunk would leave too few CTAs per launch to fill 148 SMs.
MIN_UNITS_PER_CHUNK = 8
MAX_CHUNKS = 4


def plan_chunks(units, world):
    """Number of chunks C per rank: the largest of MAX_CHUNKS, ..., 2 that divides the rank's
    units with at least MIN_UNITS_PER_CHUNK units per chunk, else 1."""
    if units % world:
        raise ValueError(f"B * H_kv = {units} units cannot be split evenly over {world} ranks")
    per = units // world
    for c in range(MAX_CHUNKS, 1, -1):
        if per % c == 0 and per // c >= MIN_UNITS_PER_CHUNK:
            return c
    return 1


def chunk_ranges(units, world, rank, chunks):
    """[(u0, u1)] for each chunk of `rank`: chunk c is units [(c W + r) cs, (c W + r + 1) cs)."""
    per = units // world
    cs = per // chunks
    return [((c * world + rank) * cs, (c * world + rank + 1) * cs) for c in range(chunks)]


def _unit_view(t, H_kv):
    B, H, S, D = t.shape
    return t.view(B * H_kv, H // H_kv, S, D)


_COMM_STREAMS = {}


def _comm_stream(device):
    """One high-priority side stream per device for the all-gathers."""
    s = _COMM_STREAMS.get(device)
    if s is None:
        s = torch.cuda.Stream(device=device, priority=-1)
        _COMM_STREAMS[device] = s
    return s


class _Gathers:
    """Issues all-gathers of finished chunks on a side stream (CUDA) or inline (CPU/gloo).

    Tensors handed to a gather stay referenced until finish(), after which the caller's stream
    is ordered after every gather: no buffer is reused while NCCL may still read or write it."""

    def __init__(self, device, group):
        self.group = group
        self.cuda = device.type == "cuda"
        self.keep = []
        if self.cuda:
            self.compute = torch.cuda.current_stream(device)
            self.comm = _comm_stream(device)

    def gather(self, pairs):
        if not self.cuda:
            for out, inp in pairs:
                dist.all_gather_into_tensor(out, inp, group=self.group)
            return
        ready = torch.cuda.Event()
        ready.record(self.compute)
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            for out, inp in pairs:
                dist.all_gather_into_tensor(out, inp, group=self.group)
        self.keep.extend(t for pair in pairs for t in pair)

    def finish(self):
        if self.cuda:
            self.compute.wait_stream(self.comm)
        self.keep.clear()


class ShardedFusedAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, tile_m, tile_n, group):
        fb = _backward_module()
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        fb._check(q, k, v, tile_m, tile_n)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        H_kv = k.shape[1]
        units = q.shape[0] * H_kv
        chunks = plan_chunks(units, world)
        ranges = chunk_ranges(units, world, rank, chunks)
        qu, ku, vu = _unit_view(q, H_kv), _unit_view(k, H_kv), _unit_view(v, H_kv)
        o = torch.empty_like(q)
        ou = _unit_view(o, H_kv)
        span = (units // world // chunks) * world  # units per gathered slab
        gathers = _Gathers(q.device, group)
        saved = []
        for c, (a, b) in enumerate(ranges):
            ol, lse = fb._forward(qu[a:b], ku[a:b], vu[a:b], tile_m, tile_n)
            gathers.gather([(ou[c * span:(c + 1) * span], ol)])
            saved += [ol, lse]
        gathers.finish()
        ctx.save_for_backward(q, k, v, *saved)
        ctx.meta = (tile_m, tile_n, group, H_kv, ranges, span)
        return o

    @staticmethod
    def backward(ctx, do):
        fb = _backward_module()
        q, k, v, *saved = ctx.saved_tensors
        tile_m, tile_n, group, H_kv, ranges, span = ctx.meta
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        qu, ku, vu, dou = (_unit_view(t, H_kv) for t in (q, k, v, do))
        dq = torch.empty(q.shape, device=do.device, dtype=do.dtype)
        dk = torch.empty(k.shape, device=do.device, dtype=do.dtype)
        dv = torch.empty(k.shape, device=do.device, dtype=do.dtype)
        dqu, dku, dvu = (_unit_view(t, H_kv) for t in (dq, dk, dv))
        gathers = _Gathers(do.device, group)
        for c, (a, b) in enumerate(ranges):
            ol, lse = saved[2 * c], saved[2 * c + 1]
            sl = slice(c * span, (c + 1) * span)
            # dK, dV of this chunk travel while its dQ kernel runs
            delta, dkl, dvl = fb._backward_kv(qu[a:b], ku[a:b], vu[a:b], ol, lse, dou[a:b], tile_m, tile_n)
            gathers.gather([(dku[sl], dkl), (dvu[sl], dvl)])
            dql = fb._backward_q(qu[a:b], ku[a:b], vu[a:b], dou[a:b], lse, delta, tile_m, tile_n)
            gathers.gather([(dqu[sl], dql)])
        gathers.finish()
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
