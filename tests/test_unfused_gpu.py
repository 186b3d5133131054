"""The unfused three-kernel baseline (attention/fused/unfused.py, attention/gqa/unfused_gqa.py)
on the GPU: O against the CPU oracle, and the materialised S and P against an fp32 computation of
the same matrices (the reference's `return_intermediates=True` contract: tiles on or below the
diagonal hold the masked scores / probabilities, everything above the diagonal stays -inf / 0).

Tolerances (written here): O as in the other forward tests, |out - ref| <= 2e-2 + 2e-2 |ref| and
max |out - ref| <= 2e-2; S (fp32 from fp32 tensor-core accumulation) |S - ref| <= 1e-3 (1 + |ref|);
P (16-bit) |P - ref| <= 2e-3 + 1e-2 ref.
"""
import math
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


def _check_o(o, q, k, v):
    ref = ora.causal_attention(*(t.float().cpu().numpy() for t in (q, k, v)))
    got = o.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert ora.elementwise_ratio(got, ref) <= 1.0
    assert ora.max_abs(got, ref) <= 2e-2


@pytest.mark.parametrize("case", [ora.Case(2, 3, 512, 64, "large"), ora.Case(1, 2, 1024, 128, "tiny"),
                                  ora.Case(2, 2, 256, 32, "large"), ora.Case(1, 2, 192, 64, "tiny")],
                         ids=lambda c: c.id)
def test_unfused_attention_matches_oracle(case, cuda_device):
    from attention.fused.unfused import unfused_attention, _native
    q, k, v = (to_dev(x) for x in ora.make_inputs(case))
    o = unfused_attention(q, k, v, 64, 64)
    _native().check_status(cuda_device)
    _check_o(o, q, k, v)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,H_kv", [(8, 2), (4, 1), (6, 3)])
def test_unfused_gqa_attention_matches_oracle(H, H_kv, dtype, cuda_device):
    from attention.gqa.unfused_gqa import unfused_gqa_attention
    from attention.fused.unfused import _native
    B, N, D = 2, 384, 128
    q = to_dev(ora.seeded_normal(f"uq{H}{H_kv}", (B, H, N, D), 1.0, np.float32), dtype)
    k = to_dev(ora.seeded_normal(f"uk{H}{H_kv}", (B, H_kv, N, D), 1.0, np.float32), dtype)
    v = to_dev(ora.seeded_normal(f"uv{H}{H_kv}", (B, H_kv, N, D), 1.0, np.float32), dtype)
    o = unfused_gqa_attention(q, k, v, 64, 128)
    _native().check_status(cuda_device)
    _check_o(o, q, k, v)


@pytest.mark.parametrize("N,D", [(256, 64), (384, 128)])
def test_unfused_intermediates(N, D, cuda_device):
    from attention.fused.unfused import unfused_attention, _native
    B, H = 1, 2
    q, k, v = (to_dev(ora.seeded_normal(f"ui{n}{N}", (B, H, N, D), 1.0, np.float32)) for n in "qkv")
    o, S, P = unfused_attention(q, k, v, 64, 64, return_intermediates=True)
    _native().check_status(cuda_device)
    s_ref = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(D)
    mask = torch.ones(N, N, dtype=torch.bool, device=q.device).triu(1)
    s_ref = s_ref.masked_fill(mask, float("-inf"))
    p_ref = torch.softmax(s_ref, dim=-1)
    # every entry on or below the diagonal, plus -inf / 0 everywhere above it
    below = ~mask
    assert bool(torch.isneginf(S[..., mask]).all())
    assert bool((P[..., mask] == 0).all())
    ds = (S[..., below] - s_ref[..., below]).abs()
    assert float((ds / (1 + s_ref[..., below].abs())).max()) <= 1e-3
    dp = (P.float() - p_ref).abs()
    assert float((dp - (2e-3 + 1e-2 * p_ref)).max()) <= 0
    _check_o(o, q, k, v)


def test_unfused_cli_backend(tmp_path, cuda_device):
    case = ora.Case(1, 4, 256, 64, "tiny")
    q, k, v = ora.make_inputs(case)
    npz, out = str(tmp_path / "in.npz"), str(tmp_path / "out.npy")
    np.savez(npz, Q=q, K=k, V=v)
    r = subprocess.run([sys.executable, os.path.join(REPO, "fused-attention_b200", "run_attention.py"),
                        "--input", npz, "--output", out, "--backend", "unfused"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    o = np.load(out).astype(np.float32)
    ref = ora.causal_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    assert ora.elementwise_ratio(o, ref) <= 1.0 and ora.max_abs(o, ref) <= 2e-2
