"""Causal fused attention forward on B200 (sm_100a).

Drop-in for the reference's `attention/fused/fused.py` (`fused_attention`, :68-76): same name,
arguments, return value and errors.  The kernel is a hand-written sm_100a CUDA kernel
(TMA + tcgen05 UMMA + TMEM, warp-specialised, causal tile skipping, heavy-first order) in
libfa_sm100.so, reached through its C ABI (`fa_fwd`).  Work is enqueued on torch's current
stream without a host synchronisation, like the reference's `ct.launch`.

This file can be imported by path (the reference's runners do that), so it locates the
binding module by path too.
"""
import importlib.util
import os
import sys

import torch

LOG2E = 1.4426950408889634  # log2(e): exp(x) = exp2(x * LOG2E); the kernel folds LOG2E / sqrt(D)


def _native():
    """The ctypes binding (attention/_lib.py), loaded by path under one shared module name."""
    mod = sys.modules.get("_fa_b200_native")
    if mod is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib.py")
        spec = importlib.util.spec_from_file_location("_fa_b200_native", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["_fa_b200_native"] = mod
        spec.loader.exec_module(mod)
    return mod


def fused_attention(q, k, v, tile_m=64, tile_n=64):
    """Causal softmax(q k^T / sqrt(D)) v for q, k, v of shape [B, H, N, D] (float16 or bfloat16).

    Raises ValueError if N is not divisible by tile_m and tile_n (as the reference does).
    tile_n selects the kernel's K/V tile (64 keys for tile_n <= 64, else 128, the faster one); the
    query side always runs 128-row tcgen05 tiles, so tile_m only takes part in the divisibility
    rule.
    """
    B, H, N, D = q.shape
    if N % tile_m != 0 or N % tile_n != 0:
        raise ValueError(f"N={N} must be divisible by tile_m={tile_m} and tile_n={tile_n}")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must all be (B, H, N, D); got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    O = torch.empty_like(q)
    nat = _native()
    nat.fwd(q, k, v, O, None, tile_m, nat.kv_tile(tile_n))
    return O
