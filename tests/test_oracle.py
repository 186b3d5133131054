"""The CPU oracle against the golden fixtures made by the reference's own PyTorch code."""
import glob
import os

import numpy as np
import pytest

from oracle import attention_oracle as ora

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _fixtures(prefix):
    files = sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))
    assert files, f"no {prefix} fixtures"
    return files


def _case_from_id(cid):
    parts = cid.split("_")
    vals = {p[0]: p[1:] for p in parts[:-1] if p[0] in "BHND"}
    hkv = [p for p in parts if p.startswith("Hkv")]
    return ora.Case(int(vals["B"]), int(parts[1][1:]), int(vals["N"]), int(vals["D"]), parts[-1],
                    int(hkv[0][3:]) if hkv else 0)


@pytest.mark.parametrize("path", _fixtures("mha_") + _fixtures("gqa_"), ids=os.path.basename)
def test_forward_oracle_matches_reference(path):
    g = np.load(path)
    case = _case_from_id(str(g["case_id"]))
    assert case.id == str(g["case_id"]) and case.seed == int(g["seed"])
    q, k, v = ora.make_inputs(case)
    # the seeded generator reproduces the reference's inputs exactly
    np.testing.assert_array_equal(q.reshape(-1)[:64], g["q_head"])
    np.testing.assert_allclose(ora_checksums(q, k, v), g["input_checksums"], rtol=1e-12)
    s = int(g["row_stride"])
    o = ora.causal_attention(q, k, v)
    assert ora.max_abs(o[:, :, ::s], g["o"]) < 2e-5
    lse = ora.lse_log2(q, k)
    assert ora.max_abs(lse[:, :, ::s], g["lse"]) < 1e-4


def ora_checksums(*arrays):
    return np.array([[float(np.asarray(a, np.float64).sum()), float(np.abs(np.asarray(a, np.float64)).sum())]
                     for a in arrays])


@pytest.mark.parametrize("path", _fixtures("bwd_"), ids=os.path.basename)
def test_backward_oracle_matches_reference_autograd(path):
    g = np.load(path)
    o, dq, dk, dv = ora.causal_attention_grads(g["q"], g["k"], g["v"], g["do"])
    for name, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        ref = g[name]
        assert ora.rel_fro(got, ref) < 1e-5, name
        assert ora.max_abs(got, ref) < 1e-3 * max(1.0, float(np.abs(ref).max())), name


@pytest.mark.parametrize("tiles", [(64, 64), (64, 128), (128, 64), (128, 128)])
@pytest.mark.parametrize("mag", ["tiny", "large"])
def test_tiled_algorithm_matches_exact(tiles, mag):
    """The kernel algorithm restatement (online softmax, exp2, fp16 P) agrees with the exact
    fp32 reference within the reference's own tolerance."""
    case = ora.Case(1, 2, 256, 64, mag)
    q, k, v = ora.make_inputs(case)
    out, lse = ora.tiled_forward(q, k, v, *tiles)
    assert ora.elementwise_ratio(out, ora.causal_attention(q, k, v)) < 0.5
    assert ora.lse_rel_err(lse, ora.lse_log2(q, k)) < 1e-5


def test_case_grids_match_reference_counts():
    assert len(ora.mha_cases()) == 84
    assert len(ora.gqa_cases()) == 96
    assert ora.mha_cases()[0].id == "B1_H1_N128_D32_tiny"
    assert ora.gqa_cases()[0].id == "B4_H8_Hkv1_N128_D32_tiny"


def test_tolerance_rules_detect_a_planted_error():
    """A mistake planted in the oracle's output must be caught by every comparison rule."""
    case = ora.Case(1, 1, 128, 64, "large")
    q, k, v = ora.make_inputs(case)
    ref = ora.causal_attention(q, k, v)
    bad = ref.copy()
    bad[0, 0, 77, 5] += 0.1
    assert ora.elementwise_ratio(ref, ref) == 0.0
    assert ora.elementwise_ratio(bad, ref) > 1.0
    assert ora.max_abs(bad, ref) > 2e-2
    lse = ora.lse_log2(q, k)
    bad_lse = lse.copy()
    bad_lse[0, 0, 3] += 0.01
    assert ora.lse_rel_err(bad_lse, lse) > 1e-3
