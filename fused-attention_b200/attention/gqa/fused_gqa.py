"""Causal fused GQA/MQA attention forward on B200 (sm_100a).

Drop-in for the reference's `attention/gqa/fused_gqa.py` (`fused_gqa_attention`, :70-82):
K and V have H_kv heads and query head h reads K/V head h // (H // H_kv) (:18).  On B200 one
CTA computes two query tiles that read the same K/V head, so for even group sizes each K/V
tile is loaded into shared memory once for two query heads of the group.
"""
import importlib.util
import os
import sys

import torch

LOG2E = 1.4426950408889634


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


def fused_gqa_attention(q, k, v, tile_m=64, tile_n=64):
    """Causal GQA attention: q [B, H, N, D], k and v [B, H_kv, N, D] with H_kv dividing H.

    tile_m and tile_n keep the reference's divisibility rule; tile_n also selects the kernel's K/V
    tile (64 keys for tile_n <= 64, else 128) and the query side always runs 128-row tiles."""
    B, H, N, D = q.shape
    H_kv = k.shape[1]
    if tuple(k.shape) != (B, H_kv, N, D) or v.shape != k.shape or H % H_kv != 0:
        raise ValueError(f"GQA needs K, V of shape [B, H_kv, N, D] with H_kv dividing H; got Q {tuple(q.shape)}, K {tuple(k.shape)}, V {tuple(v.shape)}")
    if N % tile_m != 0 or N % tile_n != 0:
        raise ValueError(f"N={N} must be divisible by tile_m={tile_m} and tile_n={tile_n}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    O = torch.empty_like(q)
    nat = _native()
    nat.fwd(q, k, v, O, None, tile_m, nat.kv_tile(tile_n))
    return O
