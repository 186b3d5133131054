"""fa_bwd_noalloc: the backward entry point that allocates no device memory.

Who needs it: callers that cannot call cudaMalloc, such as a plugin running inside a framework
whose memory pool has already reserved nearly all of HBM (a raw cudaMalloc from the plugin then
fails), or a latency-critical path where cudaMalloc is off limits because it can synchronise the
device.  The regular backward asks such a caller for a float32 `delta` scratch buffer; this entry
point keeps that scratch in a fixed-size static device array inside the library instead
(FA_NOALLOC_MAX_ROWS rows of B*H*S) and takes only the inputs and outputs.

The GPU test calls it through the C ABI twice in a row, with different shapes and dtypes (so a
stale scratch from the first call would show), and compares dQ, dK, dV with the regular
three-call backward (fa_bwd_preprocess, fa_bwd_dkdv, fa_bwd_dq) that uses a caller-allocated
delta.  A second GPU test captures the entry point into a CUDA graph on a side stream (after one
uncaptured call, as the header requires) and checks that replays write the same bits as uncaptured
calls, also after the inputs change in place.  This file is named to be collected last.
"""
import ctypes

import pytest
import torch

FA_OK = 0
FA_ERR_TOO_LARGE = 7
FA_NOALLOC_MAX_ROWS = 1 << 22
ATOL = RTOL = 2e-2  # the elementwise rule the other parity tests use


def _nat():
    from attention.fused.fused import _native
    return _native()


def _call_noalloc(lib, q, k, v, o, do, lse, dq, dk, dv, tile_m, tile_n, status, stream):
    B, H, S, D = q.shape
    H_kv = k.shape[1]
    P = ctypes.c_void_p
    return lib.fa_bwd_noalloc(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(o.data_ptr()),
                              P(do.data_ptr()), P(lse.data_ptr()), P(dq.data_ptr()), P(dk.data_ptr()),
                              P(dv.data_ptr()), B, H, H_kv, S, D,
                              1 if q.dtype == torch.bfloat16 else 0, tile_m, tile_n,
                              P(status.data_ptr()), P(stream))


@pytest.mark.gpu
def test_noalloc_backward_matches_regular_backward_twice(cuda_device):
    nat = _nat()
    lib = nat.load()
    cases = [((2, 4, 2, 512, 128), torch.float16, (64, 128)),
             ((1, 8, 8, 1024, 64), torch.bfloat16, (64, 64))]
    for call, ((B, H, H_kv, S, D), dtype, (tm, tn)) in enumerate(cases):
        g = torch.Generator(device=cuda_device).manual_seed(100 + call)
        q = torch.randn(B, H, S, D, device=cuda_device, generator=g).to(dtype)
        k = torch.randn(B, H_kv, S, D, device=cuda_device, generator=g).to(dtype)
        v = torch.randn(B, H_kv, S, D, device=cuda_device, generator=g).to(dtype)
        do = torch.randn(B, H, S, D, device=cuda_device, generator=g).to(dtype)
        o = torch.empty_like(q)
        lse = torch.empty(B, H, S, device=cuda_device, dtype=torch.float32)
        nat.fwd(q, k, v, o, lse, tm, tn)

        # regular path: caller-allocated delta
        delta = torch.empty(B, H, S, device=cuda_device, dtype=torch.float32)
        dq_r, dk_r, dv_r = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        nat.bwd_preprocess(o, do, delta)
        nat.bwd_dkdv(q, k, v, do, lse, delta, dk_r, dv_r, tm, tn)
        nat.bwd_dq(q, k, v, do, lse, delta, dq_r, tm, tn)

        # allocation-free path, through the C ABI
        dq_n, dk_n, dv_n = torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0)
        status = nat.status_tensor(cuda_device)
        rc = _call_noalloc(lib, q, k, v, o, do, lse, dq_n, dk_n, dv_n, tm, tn, status,
                           torch.cuda.current_stream(cuda_device).cuda_stream)
        assert rc == FA_OK, lib.fa_strerror(rc).decode()
        nat.check_status(cuda_device)
        for name, got, ref in (("dQ", dq_n, dq_r), ("dK", dk_n, dk_r), ("dV", dv_n, dv_r)):
            assert torch.isfinite(got).all(), (call, name)
            err = ((got.float() - ref.float()).abs() / (ATOL + RTOL * ref.float().abs())).max().item()
            assert err <= 1.0, (call, name, err)
            assert torch.equal(got, ref), (call, name)  # same kernels, same inputs: identical bits


@pytest.mark.gpu
def test_noalloc_backward_replays_from_a_cuda_graph(cuda_device):
    nat = _nat()
    lib = nat.load()
    B, H, H_kv, S, D, tm, tn = 2, 4, 2, 512, 128, 64, 128
    g = torch.Generator(device=cuda_device).manual_seed(7)
    q, do = (torch.randn(B, H, S, D, device=cuda_device, generator=g).half() for _ in range(2))
    k, v = (torch.randn(B, H_kv, S, D, device=cuda_device, generator=g).half() for _ in range(2))
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device=cuda_device, dtype=torch.float32)
    nat.fwd(q, k, v, o, lse, tm, tn)
    status = nat.status_tensor(cuda_device)
    main = torch.cuda.current_stream(cuda_device)

    def eager():
        outs = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
        rc = _call_noalloc(lib, q, k, v, o, do, lse, *outs, tm, tn, status, main.cuda_stream)
        assert rc == FA_OK, lib.fa_strerror(rc).decode()
        nat.check_status(cuda_device)
        return outs

    ref = eager()  # the uncaptured call that must precede capture in this context
    dq, dk, dv = torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(main)
    graph = torch.cuda.CUDAGraph()
    rcs = []
    with torch.cuda.graph(graph, stream=side):
        rcs.append(_call_noalloc(lib, q, k, v, o, do, lse, dq, dk, dv, tm, tn, status, side.cuda_stream))
    assert rcs == [FA_OK], lib.fa_strerror(rcs[0]).decode()
    torch.cuda.synchronize(cuda_device)
    assert bool((dq == 7.0).all())  # capture records the launches without running them
    for replay in range(2):
        if replay == 1:  # new inputs in the same buffers: the graph reads them, the scratch is reused
            do.copy_(torch.randn(do.shape, device=cuda_device, generator=g).half())
            o.mul_(-1.0)
            ref = eager()
        graph.replay()
        torch.cuda.synchronize(cuda_device)
        nat.check_status(cuda_device)
        for name, got, r in zip(("dQ", "dK", "dV"), (dq, dk, dv), ref):
            assert torch.equal(got, r), (replay, name)
    del graph


def test_noalloc_rejects_problems_beyond_its_scratch():
    """Checked on the host before anything touches a device (runs without a GPU)."""
    lib = _nat().load()
    P = ctypes.c_void_p
    ptr = P(256)
    B, H, S = 16, 32, 16384  # 8M rows > FA_NOALLOC_MAX_ROWS
    assert B * H * S > FA_NOALLOC_MAX_ROWS
    rc = lib.fa_bwd_noalloc(ptr, ptr, ptr, ptr, ptr, ptr, ptr, ptr, ptr, B, H, H, S, 128, 0, 64, 64, ptr, None)
    assert rc == FA_ERR_TOO_LARGE
    assert "exceeds" in lib.fa_strerror(rc).decode()
