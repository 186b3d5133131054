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
together is then the contiguous slab [c * W * cs, (c + 1) * W * cs), so it can be gathered as soon
as chunk c is computed, on a side stream, while chunk c + 1 computes.  With C = 1 this is the plain
contiguous split.  The kernels write a rank's own chunk straight into the full output tensor.

Gathering a chunk (CUDA, the default "pull" mode): each rank copies its chunk into a staging area
of symmetric memory (every rank's staging area is mapped into every other rank), a one-element
NCCL all-reduce on the side stream acts as the barrier "every rank has staged chunk c", and each
rank then pulls the W - 1 other chunks from the peers' staging areas with plain device-to-device
copies, which run on the copy engines and take no SMs away from the attention kernels.  A final
barrier keeps the staging area from being overwritten before every peer has read it.  With
FA_GATHER=nccl (and always on CPU / gloo) a chunk is gathered with all_gather_into_tensor
instead; the NCCL kernels then compete with the attention kernels for SMs.

Every rank issues the same collectives in the same order.  Each rank holds the full inputs
(replicated) and receives the full outputs, which is the drop-in semantics of the single-GPU
functions.  Requires (B * H_kv) % world_size == 0.
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


def max_chunks(world):
    """The copy engines sit idle while a pass computes its first chunk and the last chunk's
    copies run after the kernels: finer chunks shorten both, at the price of more, smaller
    launches.  Four is the measured choice: at 16 heads per launch (eight chunks of the bench's
    128 units) the forward runs at about 64 % of its full-grid rate, which costs more than the
    shorter exposed copies save."""
    return 4


def plan_chunks(units, world):
    """Number of chunks C per rank: the largest of max_chunks(world), ..., 2 that divides the
    rank's units with at least MIN_UNITS_PER_CHUNK units per chunk, else 1."""
    if units % world:
        raise ValueError(f"B * H_kv = {units} units cannot be split evenly over {world} ranks")
    per = units // world
    for c in range(max_chunks(world), 1, -1):
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
_WORKSPACES = {}
_FLAGS = {}


def _comm_stream(device):
    """One high-priority side stream per device for the gathers."""
    s = _COMM_STREAMS.get(device)
    if s is None:
        s = torch.cuda.Stream(device=device, priority=-1)
        _COMM_STREAMS[device] = s
    return s


def _group_name(group):
    return (group if group is not None else dist.group.WORLD).group_name


def _workspace(device, group, nbytes):
    """Symmetric staging memory of at least `nbytes` on every rank of `group` (collective when it
    has to grow: every rank asks for the same size at the same point)."""
    key = (device, _group_name(group))
    ws = _WORKSPACES.get(key)
    if ws is None or ws[0].numel() < nbytes:
        import torch.distributed._symmetric_memory as symm_mem
        size = max(nbytes, ws[0].numel() if ws is not None else 0)
        buf = symm_mem.empty(size, dtype=torch.uint8, device=device)
        handle = symm_mem.rendezvous(buf, _group_name(group))
        old = ws
        ws = (buf, handle, old)  # a replaced area stays mapped: peers may still hold its address
        _WORKSPACES[key] = ws
    return ws[1]


def _flag(device):
    f = _FLAGS.get(device)
    if f is None:
        f = torch.zeros(1, dtype=torch.int32, device=device)
        _FLAGS[device] = f
    return f


def gather_mode(device):
    if device.type != "cuda":
        return "nccl"
    mode = os.environ.get("FA_GATHER", "pull")
    if mode not in ("pull", "nccl"):
        raise ValueError(f"FA_GATHER must be 'pull' or 'nccl', not {mode!r}")
    return mode


class _Gathers:
    """The gathers of one forward or backward pass.

    gather(items) takes (slab, local, stage_offset) triples: `slab` is the output slab of one
    chunk (W * cs units), `local` is this rank's cs units, which the kernels already wrote into
    the rank's slot of the slab, and `stage_offset` is where the chunk goes in the staging area
    (the same on every rank).  Tensors handed over stay referenced until finish(), after which
    the caller's stream is ordered after every copy: no buffer is reused while a peer or NCCL may
    still read or write it."""

    def __init__(self, device, group, stage_bytes):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cuda = device.type == "cuda"
        self.mode = gather_mode(device)
        self.keep = []
        if self.cuda:
            self.compute = torch.cuda.current_stream(device)
            self.comm = _comm_stream(device)
        if self.mode == "pull":
            self.handle = _workspace(device, group, stage_bytes)
            self.flag = _flag(device)

    def _barrier(self):
        dist.all_reduce(self.flag, group=self.group)

    def gather(self, items):
        if not self.cuda:
            for slab, local, _ in items:
                dist.all_gather_into_tensor(slab, local, group=self.group)
            return
        ready = torch.cuda.Event()
        ready.record(self.compute)
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            if self.mode == "nccl":
                for slab, local, _ in items:
                    dist.all_gather_into_tensor(slab, local, group=self.group)
            else:
                for _, local, off in items:
                    self.handle.get_buffer(self.rank, tuple(local.shape), local.dtype,
                                           off // local.element_size()).copy_(local)
                self._barrier()
                for slab, local, off in items:
                    cs = local.shape[0]
                    for step in range(1, self.world):
                        peer = (self.rank + step) % self.world
                        src = self.handle.get_buffer(peer, tuple(local.shape), local.dtype,
                                                     off // local.element_size())
                        slab[peer * cs:(peer + 1) * cs].copy_(src)
        self.keep.extend(t for slab, local, _ in items for t in (slab, local))

    def finish(self):
        if self.cuda:
            if self.mode == "pull":
                with torch.cuda.stream(self.comm):
                    self._barrier()
            self.compute.wait_stream(self.comm)
        self.keep.clear()


def _nbytes(t):
    return t.numel() * t.element_size()


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
        span = (units // world // chunks) * world  # units per gathered slab
        qu, ku, vu = _unit_view(q, H_kv), _unit_view(k, H_kv), _unit_view(v, H_kv)
        o = torch.empty_like(q)
        ou = _unit_view(o, H_kv)
        chunk_bytes = _nbytes(ou[:span // world])
        gathers = _Gathers(q.device, group, chunks * chunk_bytes)
        lses = []
        for c, (a, b) in enumerate(ranges):
            _, lse = fb._forward(qu[a:b], ku[a:b], vu[a:b], tile_m, tile_n, out=ou[a:b])
            gathers.gather([(ou[c * span:(c + 1) * span], ou[a:b], c * chunk_bytes)])
            lses.append(lse)
        gathers.finish()
        ctx.save_for_backward(q, k, v, o, *lses)
        ctx.meta = (tile_m, tile_n, group, H_kv, ranges, span)
        return o

    @staticmethod
    def backward(ctx, do):
        fb = _backward_module()
        q, k, v, o, *lses = ctx.saved_tensors
        tile_m, tile_n, group, H_kv, ranges, span = ctx.meta
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        qu, ku, vu, ou, dou = (_unit_view(t, H_kv) for t in (q, k, v, o, do))
        dq = torch.empty(q.shape, device=do.device, dtype=do.dtype)
        dk = torch.empty(k.shape, device=do.device, dtype=do.dtype)
        dv = torch.empty(k.shape, device=do.device, dtype=do.dtype)
        dqu, dku, dvu = (_unit_view(t, H_kv) for t in (dq, dk, dv))
        chunks = len(ranges)
        cq = _nbytes(dqu[ranges[0][0]:ranges[0][1]])
        ckv = _nbytes(dku[ranges[0][0]:ranges[0][1]])
        off_k, off_v, off_q = 0, chunks * ckv, 2 * chunks * ckv  # staging: dK chunks | dV | dQ
        gathers = _Gathers(do.device, group, 2 * chunks * ckv + chunks * cq)
        for c, (a, b) in enumerate(ranges):
            sl = slice(c * span, (c + 1) * span)
            # dK, dV of this chunk travel while its dQ kernel runs
            delta, _, _ = fb._backward_kv(qu[a:b], ku[a:b], vu[a:b], ou[a:b], lses[c], dou[a:b],
                                          tile_m, tile_n, dk=dku[a:b], dv=dvu[a:b])
            gathers.gather([(dku[sl], dku[a:b], off_k + c * ckv), (dvu[sl], dvu[a:b], off_v + c * ckv)])
            fb._backward_q(qu[a:b], ku[a:b], vu[a:b], dou[a:b], lses[c], delta, tile_m, tile_n, dq=dqu[a:b])
            gathers.gather([(dqu[sl], dqu[a:b], off_q + c * cq)])
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
