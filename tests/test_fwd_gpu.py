"""Forward (MHA, GQA, LSE) parity of the sm_100a kernel against the CPU oracle and golden vectors.

Tolerances (written here, from the reference and BASELINE):
  * elementwise |out - ref| <= 2e-2 + 2e-2 |ref|  (tests/fused/run_correctness.py:33-35 in the
    reference) and max |out - ref| <= 2e-2 on O;
  * relative LSE error <= 1e-3 (|ref| floored at 1, i.e. absolute below 1).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.gpu_util import elementwise_ratio, reference_rows, sampled_heads, seeded, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
O_MAX_ABS = 2e-2
LSE_REL = 1e-3


def _nat():
    from attention.fused.fused import _native
    return _native()


def fwd(q, k, v, tile_m=64, tile_n=64, with_lse=False):
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device=q.device, dtype=torch.float32) if with_lse else None
    _nat().fwd(q.contiguous(), k.contiguous(), v.contiguous(), o, lse, tile_m, tile_n)
    _nat().check_status(q.device)
    return (o, lse) if with_lse else o


def _check_case(q_np, k_np, v_np, dtype=torch.float16, tiles=(64, 64), lse=True):
    q, k, v = (to_dev(x, dtype) for x in (q_np, k_np, v_np))
    o, l = fwd(q, k, v, *tiles, with_lse=True)
    qf, kf, vf = (t.float().cpu().numpy() for t in (q, k, v))
    ref = ora.causal_attention(qf, kf, vf)
    out = o.float().cpu().numpy()
    assert np.isfinite(out).all()
    assert ora.elementwise_ratio(out, ref) <= 1.0
    assert ora.max_abs(out, ref) <= O_MAX_ABS
    if lse:
        assert ora.lse_rel_err(l.cpu().numpy(), ora.lse_log2(qf, kf)) <= LSE_REL


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "mha_*.npz")) +
                                        glob.glob(os.path.join(GOLDEN, "gqa_*.npz"))), ids=os.path.basename)
def test_golden_vectors(path, cuda_device):
    g = np.load(path)
    cid = str(g["case_id"])
    parts = cid.split("_")
    D = int([p for p in parts if p.startswith("D")][0][1:])
    case = next(c for c in (ora.mha_cases() + ora.gqa_cases()) if c.id == cid)
    q, k, v = (to_dev(x) for x in ora.make_inputs(case))
    o, l = fwd(q, k, v, with_lse=True)
    s = int(g["row_stride"])
    out = o.float().cpu().numpy()[:, :, ::s]
    assert ora.elementwise_ratio(out, g["o"]) <= 1.0
    assert ora.max_abs(out, g["o"]) <= O_MAX_ABS
    assert ora.lse_rel_err(l.cpu().numpy()[:, :, ::s], g["lse"]) <= LSE_REL


def test_config1_b1_h8_s1024_d64(cuda_device):
    """B=1, H=8, S=1024, D=64, fp16, i.i.d. N(0,1), against the CPU oracle."""
    shape = (1, 8, 1024, 64)
    q, k, v = (ora.seeded_normal(f"C1_{n}", shape) for n in "QKV")
    _check_case(q, k, v)


REF_GRID = [c for c in ora.mha_cases() if c.N <= 2048]


@pytest.mark.parametrize("case", REF_GRID, ids=lambda c: c.id)
def test_reference_mha_grid(case, cuda_device):
    """The reference's own MHA case grid (tests/fused/cases.py), N <= 2048, against the oracle."""
    _check_case(*ora.make_inputs(case), lse=case.N <= 512)


GQA_GRID = [c for c in ora.gqa_cases() if c.N <= 512]


@pytest.mark.parametrize("case", GQA_GRID, ids=lambda c: c.id)
def test_reference_gqa_grid(case, cuda_device):
    _check_case(*ora.make_inputs(case))


@pytest.mark.parametrize("tiles", [(64, 64), (64, 128), (128, 128), (128, 64)])
@pytest.mark.parametrize("D", [64, 128])
def test_tile_shapes(tiles, D, cuda_device):
    case = ora.Case(2, 3, 512, D, "large")
    _check_case(*ora.make_inputs(case), tiles=tiles)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,H_kv", [(8, 8), (8, 2), (8, 1), (6, 2), (5, 1), (4, 4)])
def test_gqa_and_dtypes(dtype, H, H_kv, cuda_device):
    shape_q, shape_kv = (2, H, 384, 128), (2, H_kv, 384, 128)
    q = ora.seeded_normal(f"gq{H}{H_kv}", shape_q, 1.0, np.float32)
    k = ora.seeded_normal(f"gk{H}{H_kv}", shape_kv, 1.0, np.float32)
    v = ora.seeded_normal(f"gv{H}{H_kv}", shape_kv, 1.0, np.float32)
    _check_case(q, k, v, dtype=dtype)


@pytest.mark.parametrize("S", [64, 128, 192, 320])
def test_short_and_odd_tile_counts(S, cuda_device):
    """S that is not a multiple of the 2 x 128-row CTA unit (single or partial query tiles)."""
    case = ora.Case(1, 3, S, 64, "large")
    _check_case(*ora.make_inputs(case))


def test_deterministic(cuda_device):
    q, k, v = (seeded(f"det{n}", (2, 4, 1024, 128), torch.float16) for n in "qkv")
    a = fwd(q, k, v)
    b = fwd(q, k, v)
    assert torch.equal(a, b)


@pytest.mark.parametrize("S,dtype,H_kv", [(8192, torch.float16, 32), (16384, torch.float16, 32),
                                          (8192, torch.bfloat16, 2), (8192, torch.bfloat16, 1)])
def test_baseline_sizes_sampled(S, dtype, H_kv, cuda_device):
    """BASELINE configs 2/3 sizes (B=4, H=32, D=128): full kernel run, fp32 device reference on
    sampled heads and query-row windows, plus size-independent properties on every output."""
    B, H, D = 4, 32, 128
    q = seeded(f"bq{S}", (B, H, S, D), dtype)
    k = seeded(f"bk{S}{H_kv}", (B, H_kv, S, D), dtype)
    v = seeded(f"bv{S}{H_kv}", (B, H_kv, S, D), dtype)
    o, lse = fwd(q, k, v, 64, 128, with_lse=True)
    assert torch.isfinite(o).all()
    # every output row is a convex combination of V rows
    vmax = v.float().abs().amax(dim=(2, 3))  # [B, H_kv]
    omax = o.float().abs().amax(dim=(2, 3)).view(B, H_kv, H // H_kv).amax(-1)
    assert bool((omax <= vmax * (1 + 1e-2) + 1e-3).all())
    for b, h in sampled_heads(B, H, n=3):
        for r0 in (0, S // 2 - 128, S - 256):
            rows = slice(r0, r0 + 256)
            ref, ref_lse = reference_rows(q, k, v, b, h, rows, with_lse=True)
            got = o[b, h, rows]
            assert elementwise_ratio(got, ref) <= 1.0
            assert float((got.float() - ref).abs().max()) <= O_MAX_ABS
            rel = ((lse[b, h, rows] - ref_lse).abs() / ref_lse.abs().clamp_min(1.0)).max()
            assert float(rel) <= LSE_REL


def test_status_clean(cuda_device):
    _nat().check_status(cuda_device)
