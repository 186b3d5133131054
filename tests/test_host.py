"""Host-side logic that runs without a GPU: the C-ABI library loads and exports every declared
symbol, argument validation in C and Python, the input contracts and the CLI exit codes."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "fused-attention_b200")
HEADER = os.path.join(REPO, "include", "fa_sm100.h")


def _native():
    from attention.fused.fused import _native as n
    return n()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FA_API\s+[\w\s\*]*?\b(fa_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert {"fa_fwd", "fa_bwd_preprocess", "fa_bwd_dkdv", "fa_bwd_dq", "fa_strerror",
            "fa_abi_version", "fa_last_cuda_error"} <= set(syms)


def test_library_loads_and_exports_every_declared_symbol():
    lib = ctypes.CDLL(_native().LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(_native().SIGNATURES) >= set(declared_symbols())
    assert _native().load().fa_abi_version() == _native().ABI_VERSION


def test_strerror_covers_codes():
    lib = _native().load()
    for code in range(0, 7):
        assert lib.fa_strerror(code).decode() not in ("", "unknown error code")
    assert lib.fa_strerror(99).decode() == "unknown error code"


def test_error_codes_match_the_header_and_map_to_python_exceptions():
    """The binding's FA_ERR_* values are the header's; argument errors raise ValueError, CUDA /
    driver / device errors RuntimeError, each with the library's message."""
    nat = _native()
    text = open(HEADER).read()
    codes = {m.group(1): int(m.group(2)) for m in re.finditer(r"\b(FA_(?:OK|ERR_\w+))\s*=\s*(\d+)", text)}
    assert codes and all(getattr(nat, name) == value for name, value in codes.items()), codes
    lib = nat.load()
    for name in ("FA_ERR_INVALID_ARG", "FA_ERR_UNSUPPORTED", "FA_ERR_ALIGNMENT", "FA_ERR_TOO_LARGE"):
        with pytest.raises(ValueError, match=re.escape(lib.fa_strerror(codes[name]).decode())):
            nat._raise(codes[name], "call")
    for name in ("FA_ERR_DRIVER", "FA_ERR_DEVICE"):
        with pytest.raises(RuntimeError, match=re.escape(lib.fa_strerror(codes[name]).decode())):
            nat._raise(codes[name], "call")


def _fwd_rc(**kw):
    lib = _native().load()
    args = dict(q=8, k=8, v=8, o=8, lse=None, B=1, H=8, H_kv=8, S=128, D=64, dtype=0, tm=64, tn=64,
                st=16)
    args.update(kw)
    vp = ctypes.c_void_p
    return lib.fa_fwd(vp(args["q"]), vp(args["k"]), vp(args["v"]), vp(args["o"]), args["lse"],
                      args["B"], args["H"], args["H_kv"], args["S"], args["D"], args["dtype"],
                      args["tm"], args["tn"], vp(args["st"]), None)


@pytest.mark.parametrize("kw,code", [
    (dict(B=0), 1), (dict(S=0), 1), (dict(H=6, H_kv=4), 1), (dict(q=0), 1), (dict(st=0), 1),
    (dict(D=48), 2), (dict(D=96), 2), (dict(dtype=2), 2), (dict(tm=32), 2), (dict(tn=256), 2),
])
def test_c_abi_rejects_bad_arguments_before_touching_the_device(kw, code):
    assert _fwd_rc(**kw) == code


def test_alignment_and_shape_rules_are_checked_before_the_device():
    """Misaligned bases answer FA_ERR_ALIGNMENT and a backward S that is not a multiple of 64
    FA_ERR_UNSUPPORTED, with or without a GPU; a well-formed call on a machine without an sm_100
    device answers a CUDA / device error, never FA_OK."""
    lib = _native().load()
    vp = ctypes.c_void_p
    a, m = vp(256), vp(264)  # 16-byte aligned, misaligned
    assert _fwd_rc(q=264, k=256, v=256, o=256) == 3
    assert _fwd_rc(q=256, k=256, v=256, o=256, lse=ctypes.c_void_p(258)) == 3
    assert lib.fa_bwd_preprocess(m, a, a, 1, 8, 128, 64, 0, a, None) == 3
    assert lib.fa_bwd_dkdv(a, a, a, a, a, a, m, a, 1, 8, 8, 128, 64, 0, 64, 64, a, None) == 3
    assert lib.fa_bwd_dq(a, a, a, a, a, a, a, 1, 8, 8, 96, 64, 0, 64, 64, a, None) == 2  # S % 64
    assert lib.fa_bwd_noalloc(a, a, a, a, a, a, a, a, m, 1, 8, 8, 128, 64, 0, 64, 64, a, None) == 3
    if not torch.cuda.is_available():
        assert _fwd_rc(q=256, k=256, v=256, o=256) in (4, 5, 6)  # CUDA, driver or device error


def test_backward_rejects_unsupported_head_dims_before_touching_the_device():
    """Head dims outside {32, 64, 128} answer FA_ERR_UNSUPPORTED from every backward entry point."""
    lib = _native().load()
    vp = ctypes.c_void_p
    p = vp(16)
    for D in (48, 96, 256):
        assert lib.fa_bwd_preprocess(p, p, p, 1, 8, 128, D, 0, p, None) == 2
        assert lib.fa_bwd_dkdv(p, p, p, p, p, p, p, p, 1, 8, 8, 128, D, 0, 64, 64, p, None) == 2
        assert lib.fa_bwd_dq(p, p, p, p, p, p, p, 1, 8, 8, 128, D, 0, 64, 64, p, None) == 2
        assert lib.fa_bwd_noalloc(p, p, p, p, p, p, p, p, p, 1, 8, 8, 128, D, 0, 64, 64, p, None) == 2


def test_wrappers_launch_the_requested_kv_tile(monkeypatch):
    """The drop-in wrappers check the caller's tile_m / tile_n against N (the reference's rule) and
    launch the forward kernel with the K/V tile tile_n selects: 64 keys for tile_n <= 64, else 128."""
    from attention.fused.fused import fused_attention
    from attention.gqa.fused_gqa import fused_gqa_attention
    from attention.backward.fused_backward import _forward
    nat = _native()
    calls = []
    monkeypatch.setattr(nat, "fwd", lambda q, k, v, o, lse, tm, tn: calls.append((tm, tn, lse is None)))
    q = torch.zeros(1, 4, 128, 64, dtype=torch.float16)
    kv = torch.zeros(1, 2, 128, 64, dtype=torch.float16)
    fused_attention(q, q, q)
    fused_attention(q, q, q, 128, 64)
    fused_attention(q, q, q, 64, 128)
    fused_gqa_attention(q, kv, kv, 64, 64)
    fused_gqa_attention(q, kv, kv, 64, 128)
    _forward(q, q, q, 64, 64)
    _forward(q, q, q, 64, 128)
    assert calls == [(64, 64, True), (128, 64, True), (64, 128, True), (64, 64, True), (64, 128, True),
                     (64, 64, False), (64, 128, False)]
    assert [nat.kv_tile(t) for t in (16, 32, 64, 128, 256)] == [64, 64, 64, 128, 128]


def test_python_wrappers_keep_reference_errors():
    from attention.fused.fused import fused_attention
    from attention.gqa.fused_gqa import fused_gqa_attention
    from attention.backward.fused_backward import fused_attention_autograd
    q = torch.zeros(1, 2, 96, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="divisible"):
        fused_attention(q, q, q, 64, 64)
    k = torch.zeros(1, 3, 128, 64, dtype=torch.float16)
    q2 = torch.zeros(1, 4, 128, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="GQA needs"):
        fused_gqa_attention(q2, k, k)
    with pytest.raises(TypeError):
        fused_attention_autograd(q2.float(), q2.float(), q2.float())
    with pytest.raises(ValueError):
        fused_attention_autograd(q2, k, k)


def test_validation_contract():
    from attention.fused.validation import ValidationError, validate_qkv
    from attention.gqa.validation_gqa import validate_qkv as validate_gqa
    ok = np.zeros((2, 4, 128, 64), np.float16)
    validate_qkv(ok, ok, ok, 64, 64)
    with pytest.raises(ValidationError, match="only float16 and bfloat16"):
        validate_qkv(ok.astype(np.float32), ok, ok, 64, 64)
    z = np.zeros((1, 1, 128, 32), np.float16)
    validate_qkv(z, z, z, 64, 64)  # D = 32 is a reference head dim
    with pytest.raises(ValidationError, match="head dim D=96"):
        z = np.zeros((1, 1, 128, 96), np.float16)
        validate_qkv(z, z, z, 64, 64)
    with pytest.raises(ValidationError, match="not divisible"):
        validate_qkv(ok, ok, ok, 128, 48)
    with pytest.raises(ValidationError, match="head count mismatch"):
        validate_qkv(ok, np.ascontiguousarray(ok[:, :2]), np.ascontiguousarray(ok[:, :2]), 64, 64)
    kv = np.zeros((2, 2, 128, 64), np.float16)
    assert validate_gqa(ok, kv, kv, 64, 64) == 2
    with pytest.raises(ValidationError, match="not divisible by KV heads"):
        kv3 = np.zeros((2, 3, 128, 64), np.float16)
        validate_gqa(ok, kv3, kv3, 64, 64)
    t = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16)
    validate_qkv(t, t, t, 64, 64)


def _cli(script, *args):
    r = subprocess.run([sys.executable, os.path.join(PKG, script), *args], capture_output=True, text=True,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": os.environ.get("CUDA_VISIBLE_DEVICES", "")})
    return r.returncode, r.stderr


def test_cli_exit_codes(tmp_path):
    missing = tmp_path / "nope.npz"
    rc, err = _cli("run_attention.py", "--input", str(missing), "--output", str(tmp_path / "o.npy"))
    assert rc == 2 and "not found" in err
    bad = tmp_path / "bad.npz"
    np.savez(bad, Q=np.zeros((1, 1, 128, 64), np.float32), K=np.zeros((1, 1, 128, 64), np.float32),
             V=np.zeros((1, 1, 128, 64), np.float32))
    rc, err = _cli("run_attention.py", "--input", str(bad), "--output", str(tmp_path / "o.npy"))
    assert rc == 2 and "dtype" in err
    miss_v = tmp_path / "mv.npz"
    np.savez(miss_v, Q=np.zeros((1, 1, 128, 64), np.float16), K=np.zeros((1, 1, 128, 64), np.float16))
    rc, err = _cli("run_attention_gqa.py", "--input", str(miss_v), "--output", str(tmp_path / "o.npy"))
    assert rc == 2 and "missing" in err
    good = tmp_path / "good.npz"
    z = np.zeros((1, 2, 128, 64), np.float16)
    np.savez(good, Q=z, K=z[:, :1], V=z[:, :1])
    # a runtime failure (here: no GPU visible to the child process) is exit status 1
    r = subprocess.run([sys.executable, os.path.join(PKG, "run_attention_gqa.py"), "--input", str(good),
                        "--output", str(tmp_path / "o.npy"), "--backend", "unfused"], capture_output=True,
                       text=True, env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 1 and "unfused backend failed" in r.stderr and "no CUDA GPU" in r.stderr


def test_bench_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` (CPU only) prints one JSON line with the keys the driver reads."""
    import json
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--seq", "256", "--dim", "64"], capture_output=True, text=True,
                       timeout=600, env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_bench_reference_arm_prints_only_on_rank_0():
    """Under torchrun the reference arm runs on rank 0 alone; other ranks exit 0 without output."""
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "0", "--seq", "256", "--dim", "64"], capture_output=True,
                       text=True, timeout=600,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": "", "RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
