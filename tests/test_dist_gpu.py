"""Multi-GPU sharded attention (attention.dist) on real GPUs with NCCL: 2 ranks, one per GPU.

The sharded forward + backward must reproduce the single-GPU result exactly: every rank runs the
same kernels on whole (batch, K/V head) units and the all-gathers only move bytes.  Skipped when
fewer than two GPUs are visible.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, shape, out_path, min_units=None, mode="pull"):
    import sys
    from datetime import timedelta
    sys.path.insert(0, os.path.join(REPO, "fused-attention_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", FA_GATHER=mode)
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev,
                            pg_options=opts)
    from attention import dist as adist
    from attention.dist import sharded_attention_autograd
    if min_units is not None:
        adist.MIN_UNITS_PER_CHUNK = min_units
    from attention.backward.fused_backward import fused_attention_autograd
    B, H, H_kv, S, D = shape
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(B, H, S, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(B, H_kv, S, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(B, H_kv, S, D, device=dev, generator=g).to(torch.bfloat16)
    do = torch.randn(B, H, S, D, device=dev, generator=g).to(torch.bfloat16)
    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = sharded_attention_autograd(qs, ks, vs, 64, 128)
    o.backward(do)
    q1, k1, v1 = (t.clone().requires_grad_(True) for t in (q, k, v))
    o1 = fused_attention_autograd(q1, k1, v1, 64, 128)
    o1.backward(do)
    torch.cuda.synchronize()
    same = all(torch.equal(a, b) for a, b in ((o, o1), (qs.grad, q1.grad), (ks.grad, k1.grad), (vs.grad, v1.grad)))
    flags = torch.tensor([1 if same else 0], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        with open(out_path, "w") as f:
            f.write("same" if int(flags.item()) == 1 else "different")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["pull", "nccl"])
@pytest.mark.parametrize("shape,min_units", [((2, 8, 8, 1024, 128), None), ((1, 8, 2, 2048, 64), None),
                                              ((4, 8, 8, 1024, 128), 2), ((4, 8, 4, 1024, 64), 1)],
                         ids=["mha_batch", "gqa_heads", "mha_4_chunks", "gqa_4_chunks"])
def test_sharded_matches_single_gpu(shape, min_units, mode, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "result.txt")
    mp.start_processes(_worker, args=(2, _free_port(), shape, out, min_units, mode), nprocs=2,
                       start_method="spawn")
    assert open(out).read() == "same"
