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


def _bench():
    spec = importlib.util.spec_from_file_location("_t_bench", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("B,H,H_kv,world,cap,expect", [(4, 32, 32, 1, 32, 32), (8, 32, 8, 1, 32, 32),
                                                       (4, 32, 32, 1, 16, 16), (8, 32, 8, 1, 64, 64),
                                                       (32, 32, 32, 8, 32, 4), (8, 32, 8, 8, 32, 1)])
def test_e2e_slices_cover_every_head_once_in_whole_groups(B, H, H_kv, world, cap, expect):
    """bench.py's end-to-end slices: every (batch, query head) and (batch, K/V head) lands in
    exactly one slice, each slice pairs K/V head g with query heads [g*grp, (g+1)*grp), and the
    count respects the cap (one GPU) or is one slice per `world` batch entries (several GPUs)."""
    slices = _bench().e2e_slices(B, H, H_kv, world, cap)
    assert len(slices) == expect
    grp = H // H_kv
    seen_q, seen_kv = set(), set()
    for (bq, hq), (bk, hk) in slices:
        assert bq == bk and bq.stop - bq.start == world
        assert hq.start == hk.start * grp and hq.stop == hk.stop * grp
        seen_q |= {(b, h) for b in range(bq.start, bq.stop) for h in range(hq.start, hq.stop)}
        seen_kv |= {(b, h) for b in range(bk.start, bk.stop) for h in range(hk.start, hk.stop)}
    assert seen_q == {(b, h) for b in range(B) for h in range(H)}
    assert seen_kv == {(b, h) for b in range(B) for h in range(H_kv)}
    assert sum((q[0].stop - q[0].start) * (q[1].stop - q[1].start) for q, _ in slices) == B * H
