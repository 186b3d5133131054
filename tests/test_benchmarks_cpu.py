"""The benchmark scripts' row, speedup and aggregate logic (no GPU needed): per-configuration rows
keep the reference's column order, fused speedups are other_ms / fused_ms, failed runs leave empty
cells, and the aggregate table averages per N / per D with geometric-mean speedups."""
import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(REPO, "fused-attention_b200", "benchmarks")


def _load(name):
    spec = importlib.util.spec_from_file_location("_t_" + name, os.path.join(BENCH, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _rows(h_kv=None):
    """D, N, B, H, impl, tile_m, tile_n, median_ms, tflops, first_call_ms [, H_kv]."""
    extra = [] if h_kv is None else [h_kv]
    out = []
    for (D, N, fused_ms, sdpa_ms) in [(64, 128, 2.0, 1.0), (64, 512, 1.0, 2.0), (128, 128, 4.0, 2.0)]:
        out.append([D, N, 2, 8, "fused", 64, 64, f"{fused_ms:.4f}", "10.000", "1.0"] + extra)
        out.append([D, N, 2, 8, "unfused", 64, 64, "", "", ""] + extra)
        out.append([D, N, 2, 8, "sdpa", 64, 64, f"{sdpa_ms:.4f}", "20.000", "1.0"] + extra)
    return out


def test_forward_speedups_and_summary():
    fb = _load("benchmark_forward")
    rows = _rows()
    fb.speedups(rows)
    fused = [r for r in rows if r[4] == "fused"]
    assert [r[-1] for r in fused] == ["0.500", "2.000", "0.500"]  # sdpa_ms / fused_ms
    assert all(r[-2] == "" for r in fused)                         # unfused never ran
    assert all(r[-1] == "" and r[-2] == "" for r in rows if r[4] != "fused")
    header, body = fb.summary_rows(rows)
    assert header[:2] == ["scope", "value"] and header[-2:] == ["fused_speedup_vs_unfused", "fused_speedup_vs_sdpa"]
    by_scope = {(b[0], b[1]): b for b in body}
    assert by_scope[("N", 128)][header.index("fused_avg_median_ms")] == "3.0000"
    assert by_scope[("all", "all")][-1] == f"{(0.5 * 2.0 * 0.5) ** (1 / 3):.2f}"
    assert by_scope[("D", 64)][header.index("unfused_avg_median_ms")] == ""


def test_gqa_rows_keep_the_reference_columns():
    gq = _load("benchmark_forward_gqa")
    fb = gq._forward_bench()
    rows = _rows(h_kv=2)
    fb.speedups(rows)
    for r in rows:
        r += ["NVIDIA B200", "kernel.py", fb.kernel_tiles(64) if r[4] == "fused" else ""]
        assert len(r) == len(gq.SEP_COLUMNS)
        assert r[gq.SEP_COLUMNS.index("H_kv")] == 2
    header, body = fb.summary_rows(rows)
    assert len(body) == 2 + 2 + 1  # two N values, two D values, overall
    sep, agg = gq.output_paths("b200_fused_gqa", 128, 64, 2)
    assert sep == "results/benchmarks/fused_gqa/b200_fused_gqa/128x64/Hkv2/bench_forward_gqa_sep_b200_fused_gqa_128x64_Hkv2.csv"
    assert agg.endswith("/Hkv2/bench_forward_gqa_agg_b200_fused_gqa_128x64_Hkv2.csv")


def test_gqa_cli_rejects_a_head_count_that_does_not_divide():
    gq = _load("benchmark_forward_gqa")
    with pytest.raises(SystemExit):
        gq.main(["--H", "8", "--H-kv", "3"])


def test_csv_kernel_columns_name_no_machine_path():
    """The kernel column is repository-relative and kernel_tiles names the tile shape that ran."""
    fb = _load("benchmark_forward")
    assert fb.kernel_label(fb.DEFAULT_KERNEL) == "fused-attention_b200/attention/fused/fused.py"
    assert fb.kernel_label("/elsewhere/custom_kernel.py") == "custom_kernel.py"
    assert [fb.kernel_tiles(n) for n in (32, 64, 128, 256)] == ["q128_kv64", "q128_kv64", "q128_kv128", "q128_kv128"]
