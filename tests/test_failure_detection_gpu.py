"""Device-side failure detection, tested without faulting, trapping or hanging the GPU.

Every pipeline wait in the kernels is bounded: when one runs out, the kernel writes an error code
into the caller's int32[4] status word, drains its own copies and UMMAs, frees its TMEM and
returns; CTAs that start (or wait) after that see the non-zero status word and stop at once.

(a) A status word that is already non-zero makes every CTA of the forward, dK/dV and dQ kernels
    return before it writes anything: outputs pre-filled with a sentinel stay untouched.
(b) The failure-detection test library (fused-attention_b200/build.py: build_stall_test, the same
    sources with a 20 ms pipeline-wait limit and, at pipeline step 1, a wait on an mbarrier that
    nothing arrives at) runs each kernel on an ordinary input: the launch returns within a
    fraction of a second, the status word holds a pipeline-timeout code, the binding raises
    KernelError, and the product kernels then run correctly on the same device.
"""
import ctypes
import os
import time

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.gpu_util import seeded

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STALL_LIB = os.path.join(REPO, "fused-attention_b200", "_build", "libfa_sm100_stalltest.so")
PIPELINE_TIMEOUT_CODES = set(range(101, 109)) | {110}  # fa_sm100.cuh DeviceError
SENTINEL = 1234.0
SHAPE = (2, 4, 512, 128)


def _nat():
    from attention.fused.fused import _native
    return _native()


def _inputs():
    q, k, v, do = (seeded(f"fd_{n}", SHAPE, torch.float16) for n in "qkvd")
    nat = _nat()
    o = torch.empty_like(q)
    lse = torch.empty(SHAPE[:3], device=q.device, dtype=torch.float32)
    delta = torch.empty_like(lse)
    nat.fwd(q, k, v, o, lse, 64, 128)
    nat.bwd_preprocess(o, do, delta)
    nat.check_status(q.device)
    return q, k, v, do, o, lse, delta


def _check_against_oracle(q, k, v, do, o, dq, dk, dv):
    ref = ora.causal_attention_grads(*(t.float().cpu().numpy() for t in (q, k, v, do)))
    for name, got, r in zip(("O", "dQ", "dK", "dV"), (o, dq, dk, dv), ref):
        g = got.float().cpu().numpy()
        assert np.isfinite(g).all(), name
        assert ora.max_abs(g, r) <= 2e-2, (name, ora.max_abs(g, r))


def test_nonzero_status_word_stops_every_cta_before_it_writes(cuda_device):
    nat = _nat()
    q, k, v, do, o_ok, lse, delta = _inputs()
    outs = [torch.full_like(t, SENTINEL) for t in (q, q, k, v)]  # o, dq, dk, dv
    o, dq, dk, dv = outs
    status = nat.status_tensor(cuda_device)
    status.copy_(torch.tensor([199, 7, 0, 0], dtype=torch.int32))
    try:
        nat.fwd(q, k, v, o, None, 64, 128)
        nat.bwd_dkdv(q, k, v, do, lse, delta, dk, dv, 64, 128)
        nat.bwd_dq(q, k, v, do, lse, delta, dq, 64, 128)
        torch.cuda.synchronize()
        for name, t in zip(("O", "dQ", "dK", "dV"), outs):
            assert bool((t == SENTINEL).all()), name
        assert status.tolist() == [199, 7, 0, 0]  # nothing overwrote the first error
        with pytest.raises(nat.KernelError, match="code 199"):
            nat.check_status(cuda_device)  # raises and resets the word
    finally:
        status.zero_()
    # after the reset the same launches write every output
    nat.fwd(q, k, v, o, None, 64, 128)
    nat.bwd_dkdv(q, k, v, do, lse, delta, dk, dv, 64, 128)
    nat.bwd_dq(q, k, v, do, lse, delta, dq, 64, 128)
    nat.check_status(cuda_device)
    assert torch.equal(o, o_ok)
    _check_against_oracle(q, k, v, do, o, dq, dk, dv)


def _stall_lib():
    assert os.path.exists(STALL_LIB), f"{STALL_LIB} is not built (fused-attention_b200/build.py)"
    lib = ctypes.CDLL(STALL_LIB)
    for name, args in _nat().SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_char_p if name in ("fa_strerror", "fa_last_cuda_error") else ctypes.c_int
    return lib


@pytest.mark.parametrize("kernel", ["forward", "forward64", "dkdv", "dq"])
def test_pipeline_wait_runs_out_and_the_device_stays_usable(kernel, cuda_device):
    nat = _nat()
    lib = _stall_lib()
    q, k, v, do, o_ok, lse, delta = _inputs()
    B, H, S, D = SHAPE
    out = torch.full_like(q, SENTINEL)
    out_k, out_v = torch.full_like(k, SENTINEL), torch.full_like(v, SENTINEL)
    status = nat.status_tensor(cuda_device)
    P = ctypes.c_void_p
    ptr = lambda t: P(t.data_ptr())  # noqa: E731
    stream = P(torch.cuda.current_stream(cuda_device).cuda_stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if kernel in ("forward", "forward64"):  # 128-key tiles, and 64-key tiles (two S buffers per tile)
        tile_n = 128 if kernel == "forward" else 64
        rc = lib.fa_fwd(ptr(q), ptr(k), ptr(v), ptr(out), ptr(lse), B, H, H, S, D, 0, 64, tile_n, ptr(status), stream)
    elif kernel == "dkdv":
        rc = lib.fa_bwd_dkdv(ptr(q), ptr(k), ptr(v), ptr(do), ptr(lse), ptr(delta), ptr(out_k), ptr(out_v),
                             B, H, H, S, D, 0, 64, 128, ptr(status), stream)
    else:
        rc = lib.fa_bwd_dq(ptr(q), ptr(k), ptr(v), ptr(do), ptr(lse), ptr(delta), ptr(out),
                           B, H, H, S, D, 0, 64, 128, ptr(status), stream)
    assert rc == 0, lib.fa_strerror(rc)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    code = status.tolist()[0]
    assert code in PIPELINE_TIMEOUT_CODES, status.tolist()
    assert elapsed < 10.0, elapsed
    with pytest.raises(nat.KernelError, match=f"code {code}"):
        nat.check_status(cuda_device)
    assert status.tolist()[0] == 0
    # The context is intact: the product kernels run on the same device and are correct.
    from attention.backward.fused_backward import fused_attention_autograd
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = fused_attention_autograd(qa, ka, va, 64, 128)
    o.backward(do)
    nat.check_status(cuda_device)
    assert torch.equal(o.detach(), o_ok)
    _check_against_oracle(q, k, v, do, o.detach(), qa.grad, ka.grad, va.grad)
