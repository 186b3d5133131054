"""The correctness runner's harness (tests/runners/run_correctness.py) on CPU: with `--impl reference`
the fp32 ground truth goes through the same case generation, error metrics and CSV writing, and
must pass with the reference's columns."""
import csv
import importlib.util
import os

import pytest

RUNNER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "runners", "run_correctness.py")


def _runner():
    spec = importlib.util.spec_from_file_location("_t_run_correctness", RUNNER)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("suite,case,columns", [
    ("fused", "B1_H1_N128_D32_tiny", "FWD_COLUMNS"),
    ("gqa", "B4_H8_Hkv2_N128_D32_large", "GQA_COLUMNS"),
    ("backward", "B1_H1_N128_D64", "BWD_COLUMNS"),
])
def test_reference_self_check_writes_the_reference_schema(suite, case, columns, tmp_path):
    rc = _runner()
    out = tmp_path / "c.csv"
    assert rc.main(["--suite", suite, "--impl", "reference", "--device", "cpu", "--filter", case,
                    "--csv", str(out)]) == 0
    rows = list(csv.reader(open(out)))
    assert rows[0] == getattr(rc, columns)
    assert len(rows) == 2 and "PASS" in rows[1]


def test_fused_impl_needs_a_gpu(tmp_path):
    rc = _runner()
    assert rc.main(["--suite", "fused", "--device", "cpu", "--csv", str(tmp_path / "x.csv")]) == 2


def test_forward_errors_flag_non_finite_and_tolerance():
    import torch
    rc = _runner()
    ref = torch.tensor([1.0, 0.0, -2.0])
    mx, rel, ratio, finite = rc.forward_errors(torch.tensor([1.01, 0.0, -2.0]), ref)
    assert finite and abs(mx - 0.01) < 1e-6 and ratio < 1.0
    assert not rc.forward_errors(torch.tensor([float("nan"), 0.0, -2.0]), ref)[3]
    assert rc.forward_errors(torch.tensor([1.1, 0.0, -2.0]), ref)[2] > 1.0
