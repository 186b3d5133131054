"""The reference's complete correctness grids on the GPU, through the per-case runner that writes
its CSV schema (tests/runners/run_correctness.py): all 84 MHA forward cases and all 96 GQA forward
cases (every N up to 8192, both magnitudes, D in {32, 64, 128}) and its 7 backward cases, each
(and both forward grids through the unfused three-kernel baseline as well)
against an fp32 ground truth computed on the same device.  A case passes under the reference's
own rules: forward |out - ref| <= 2e-2 + 2e-2 |ref| everywhere (tests/fused/run_correctness.py:
33-35 in the reference), backward relative Frobenius error <= 2e-2 on O, dQ, dK and dV
(tests/backward/run_correctness_backward.py:35-37)."""
import csv

import pytest

from tests.runners.run_correctness import main as run_correctness

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("suite,impl,tiles,n_cases", [("fused", "fused", (64, 64), 84), ("fused", "fused", (64, 128), 84),
                                                      ("gqa", "fused", (64, 64), 96), ("gqa", "fused", (128, 128), 96),
                                                      ("backward", "fused", (64, 64), 7),
                                                      ("fused", "unfused", (64, 64), 84), ("gqa", "unfused", (64, 64), 96)])
def test_reference_grid(suite, impl, tiles, n_cases, tmp_path, cuda_device):
    path = tmp_path / f"{suite}.csv"
    rc = run_correctness(["--suite", suite, "--impl", impl, "--tile-m", str(tiles[0]), "--tile-n", str(tiles[1]),
                          "--csv", str(path)])
    rows = list(csv.DictReader(open(path)))
    assert len(rows) == n_cases
    failed = [r.get("case") or r.get("test") for r in rows if r["result"] != "PASS"]
    assert rc == 0 and not failed, failed
