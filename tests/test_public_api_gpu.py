"""The reference-facing entry points on the GPU: the public forward wrappers (the launch without
an LSE buffer that `fused_attention` / `fused_gqa_attention` make) and both command-line drivers
end to end (.npz in, .npy out, exit status 0), each against the CPU oracle.

Tolerances (written here, as in the other forward tests): elementwise |out - ref| <= 2e-2 +
2e-2 |ref| (the reference's rule, tests/fused/run_correctness.py:33-35 in the reference) and
max |out - ref| <= 2e-2 on O.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.gpu_util import to_dev

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "fused-attention_b200")
O_MAX_ABS = 2e-2


def _check(out, q, k, v):
    ref = ora.causal_attention(*(t.float().cpu().numpy() for t in (q, k, v)))
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert ora.elementwise_ratio(got, ref) <= 1.0
    assert ora.max_abs(got, ref) <= O_MAX_ABS


@pytest.mark.parametrize("tiles", [(64, 64), (64, 128), (128, 128)])
@pytest.mark.parametrize("case", [ora.Case(2, 4, 512, 64, "large"), ora.Case(1, 3, 1024, 128, "tiny"),
                                  ora.Case(2, 2, 256, 32, "large")], ids=lambda c: c.id)
def test_fused_attention_public_wrapper(case, tiles, cuda_device):
    from attention.fused.fused import fused_attention, _native
    q, k, v = (to_dev(x) for x in ora.make_inputs(case))
    o = fused_attention(q, k, v, *tiles)
    _native().check_status(cuda_device)
    assert o.shape == q.shape and o.dtype == q.dtype
    _check(o, q, k, v)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,H_kv", [(8, 2), (8, 1), (6, 3)])
def test_fused_gqa_attention_public_wrapper(H, H_kv, dtype, cuda_device):
    from attention.gqa.fused_gqa import fused_gqa_attention, _native
    B, N, D = 2, 512, 128
    q = to_dev(ora.seeded_normal(f"pq{H}{H_kv}", (B, H, N, D), 1.0, np.float32), dtype)
    k = to_dev(ora.seeded_normal(f"pk{H}{H_kv}", (B, H_kv, N, D), 1.0, np.float32), dtype)
    v = to_dev(ora.seeded_normal(f"pv{H}{H_kv}", (B, H_kv, N, D), 1.0, np.float32), dtype)
    for tiles in ((64, 64), (64, 128)):
        o = fused_gqa_attention(q, k, v, *tiles)
        _native().check_status(cuda_device)
        _check(o, q, k, v)


def test_wrapper_output_equals_the_lse_saving_launch(cuda_device):
    """The forward without an LSE buffer computes the same bits as the LSE-saving forward."""
    from attention.fused.fused import fused_attention, _native
    from attention.backward.fused_backward import _forward
    case = ora.Case(2, 4, 1024, 128, "large")
    q, k, v = (to_dev(x) for x in ora.make_inputs(case))
    for tiles in ((64, 64), (64, 128)):
        o_plain = fused_attention(q, k, v, *tiles)
        o_lse, lse = _forward(q, k, v, *tiles)
        _native().check_status(cuda_device)
        assert torch.equal(o_plain, o_lse)
        assert torch.isfinite(lse).all()


def _run_cli(script, npz, out, *extra):
    cmd = [sys.executable, os.path.join(PKG, script), "--input", npz, "--output", out, *extra]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=REPO)


@pytest.mark.parametrize("backend", ["cutile", "fused", "reference"])
def test_run_attention_cli_end_to_end(backend, tmp_path, cuda_device):
    """run_attention.py: .npz Q, K, V -> .npy float16 O of the same shape, exit 0, matching the
    oracle (the reference's CLI path, run_attention.py:76-130 in the reference)."""
    case = ora.Case(2, 4, 512, 64, "tiny")
    q, k, v = ora.make_inputs(case)
    npz, out = str(tmp_path / "in.npz"), str(tmp_path / "out.npy")
    np.savez(npz, Q=q, K=k, V=v)
    r = _run_cli("run_attention.py", npz, out, "--backend", backend, "--block-m", "64", "--block-n", "128")
    assert r.returncode == 0, r.stderr
    o = np.load(out)
    assert o.dtype == np.float16 and o.shape == q.shape
    ref = ora.causal_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    assert ora.elementwise_ratio(o.astype(np.float32), ref) <= 1.0
    assert ora.max_abs(o.astype(np.float32), ref) <= O_MAX_ABS


def test_run_attention_gqa_cli_end_to_end(tmp_path, cuda_device):
    B, H, H_kv, N, D = 1, 8, 2, 256, 128
    q = ora.seeded_normal("cliq", (B, H, N, D))
    k = ora.seeded_normal("clik", (B, H_kv, N, D))
    v = ora.seeded_normal("cliv", (B, H_kv, N, D))
    npz, out = str(tmp_path / "in.npz"), str(tmp_path / "out.npy")
    np.savez(npz, Q=q, K=k, V=v)
    r = _run_cli("run_attention_gqa.py", npz, out, "--backend", "cutile", "--verbose")
    assert r.returncode == 0, r.stderr
    assert "wrote" in r.stderr
    o = np.load(out)
    assert o.dtype == np.float16 and o.shape == q.shape
    ref = ora.causal_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    assert ora.elementwise_ratio(o.astype(np.float32), ref) <= 1.0
    assert ora.max_abs(o.astype(np.float32), ref) <= O_MAX_ABS
