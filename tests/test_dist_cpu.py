"""Multi-rank host logic of attention.dist on CPU (gloo, world size 2).

The sm_100a kernels cannot run here, so the spawned ranks swap the kernel module for a CPU test
double (fp32 torch math); what is under test is the sharding (which (batch, K/V head) units a
rank computes), the all-gathers that rebuild O, dQ, dK, dV, and failure handling on the host.
"""
import math
import os
import socket
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cpu_kernels():
    """Test double for attention.backward.fused_backward: same _check/_forward/_backward
    signatures, fp32 torch math on the CPU."""
    import sys
    sys.path.insert(0, os.path.join(REPO, "fused-attention_b200"))
    from attention.backward import fused_backward as real

    def attn32(q, k, v):
        H, H_kv = q.shape[1], k.shape[1]
        k = k.repeat_interleave(H // H_kv, 1)
        v = v.repeat_interleave(H // H_kv, 1)
        n, d = q.shape[-2], q.shape[-1]
        s = (q @ k.transpose(-1, -2)) / math.sqrt(d)
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
        return torch.softmax(s, -1) @ v, torch.logsumexp(s, -1) * 1.4426950408889634

    def _forward(q, k, v, tm, tn, out=None):
        o, lse = attn32(q.float(), k.float(), v.float())
        if out is not None:
            out.copy_(o)
            return out, lse
        return o.to(q.dtype), lse

    def _backward(q, k, v, o, lse, do, tm, tn):
        with torch.enable_grad():  # called from inside an autograd backward
            qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
            attn32(qf, kf, vf)[0].backward(do.float())
        return qf.grad.to(q.dtype), kf.grad.to(k.dtype), vf.grad.to(v.dtype)

    def _backward_kv(q, k, v, o, lse, do, tm, tn, dk=None, dv=None):
        dq_, dk_, dv_ = _backward(q, k, v, o, lse, do, tm, tn)
        if dk is not None:
            dk.copy_(dk_), dv.copy_(dv_)
            dk_, dv_ = dk, dv
        return dq_, dk_, dv_  # the dQ of the double stands in for delta

    def _backward_q(q, k, v, do, lse, delta, tm, tn, dq=None):
        if dq is not None:
            return dq.copy_(delta)
        return delta

    return types.SimpleNamespace(_check=real._check, _forward=_forward, _backward=_backward,
                                 _backward_kv=_backward_kv, _backward_q=_backward_q)


def _inputs(B, H, H_kv, S, D):
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, H_kv, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H_kv, S, D, generator=g).to(torch.bfloat16)
    do = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    return q, k, v, do


def _worker(rank, world, port, shape, result_path, min_units=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    sys.path.insert(0, os.path.join(REPO, "fused-attention_b200"))
    from attention import dist as adist
    fake = _cpu_kernels()
    adist._backward_module = lambda: fake
    if min_units is not None:
        adist.MIN_UNITS_PER_CHUNK = min_units
    q, k, v, do = _inputs(*shape)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = adist.sharded_attention_autograd(qg, kg, vg, 64, 64)
    o.backward(do)
    if rank == 0:
        torch.save({"o": o.detach(), "dq": qg.grad, "dk": kg.grad, "dv": vg.grad}, result_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("shape,min_units", [
    ((2, 4, 4, 128, 64), None), ((1, 8, 2, 128, 64), None), ((2, 4, 1, 64, 64), None),
    ((4, 4, 4, 64, 64), 1), ((4, 8, 2, 64, 64), 2)],
    ids=["mha_batch_split", "gqa_head_split", "mqa", "mha_4_chunks", "gqa_2_chunks"])
def test_sharded_matches_single_process(shape, min_units, tmp_path):
    world = 2
    out = str(tmp_path / "r0.pt")
    mp.start_processes(_worker, args=(world, _free_port(), shape, out, min_units), nprocs=world,
                       start_method="spawn")
    got = torch.load(out)
    fake = _cpu_kernels()
    q, k, v, do = _inputs(*shape)
    o_ref, lse = fake._forward(q, k, v, 64, 64)
    dq, dk, dv = fake._backward(q, k, v, o_ref, lse, do, 64, 64)
    for name, ref in (("o", o_ref), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert torch.equal(got[name], ref), name


def test_shard_units():
    import sys
    sys.path.insert(0, os.path.join(REPO, "fused-attention_b200"))
    from attention.dist import shard_units
    assert [shard_units(8, 8, 8, r) for r in (0, 7)] == [(0, 8), (56, 64)]
    assert shard_units(1, 8, 2, 1) == (4, 8)
    with pytest.raises(ValueError):
        shard_units(1, 3, 2, 0)


def test_chunk_layout():
    """Chunk c of all ranks, in rank order, is one contiguous slab; all chunks cover every unit
    exactly once."""
    import sys
    sys.path.insert(0, os.path.join(REPO, "fused-attention_b200"))
    from attention.dist import chunk_ranges, plan_chunks
    assert plan_chunks(128 * 8, 8) == 4 and plan_chunks(128 * 2, 2) == 4
    assert plan_chunks(16, 2) == 1 and plan_chunks(32, 2) == 2
    with pytest.raises(ValueError):
        plan_chunks(10, 4)
    for units, world in ((1024, 8), (96, 2), (64, 4), (8, 8)):
        chunks = plan_chunks(units, world)
        per_rank = [chunk_ranges(units, world, r, chunks) for r in range(world)]
        span = units // world // chunks * world
        seen = []
        for c in range(chunks):
            runs = [per_rank[r][c] for r in range(world)]
            assert runs[0][0] == c * span and runs[-1][1] == (c + 1) * span
            assert all(runs[r][1] == runs[r + 1][0] for r in range(world - 1))
            seen += [u for a, b in runs for u in range(a, b)]
        assert sorted(seen) == list(range(units))


def _failing_worker(rank, world, port, flag_path):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        # this rank dies between steps, before joining the collective
        os._exit(3)
    t = torch.zeros(4)
    try:
        dist.all_reduce(t)
        with open(flag_path, "w") as f:
            f.write("completed")
    except Exception as e:  # the survivor must see an error, not hang
        with open(flag_path, "w") as f:
            f.write("error:" + type(e).__name__)
    os._exit(0)


def test_dead_rank_is_detected_by_timeout(tmp_path):
    flag = str(tmp_path / "flag.txt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, flag)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung instead of timing out")
    assert open(flag).read().startswith("error:")
