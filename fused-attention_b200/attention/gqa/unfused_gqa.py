"""Unfused causal GQA/MQA attention baseline on B200 (sm_100a).

Drop-in for the reference's `attention/gqa/unfused_gqa.py` (`unfused_gqa_attention`, :99-128):
K and V have H_kv heads and query head h reads K/V head h // (H // H_kv); S, P and O keep H heads.
The same three kernels as attention/fused/unfused.py (fa_unfused_fwd handles the head mapping).
"""
import importlib.util
import os
import sys


def _unfused_module():
    """attention/fused/unfused.py, loaded by path (this file may itself be imported by path)."""
    name = "_fa_b200_unfused"
    mod = sys.modules.get(name)
    if mod is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fused", "unfused.py")
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return mod


def unfused_gqa_attention(q, k, v, tile_m=64, tile_n=64, return_intermediates=False):
    """Causal GQA attention through materialised S and P: q [B, H, N, D], k and v [B, H_kv, N, D]."""
    B, H, N, D = q.shape
    if N % tile_m != 0 or N % tile_n != 0:
        raise ValueError(f"N={N} must be divisible by tile_m={tile_m} and tile_n={tile_n}")
    H_kv = k.shape[1]
    if tuple(k.shape) != (B, H_kv, N, D) or v.shape != k.shape or H % H_kv != 0:
        raise ValueError(f"GQA needs K, V of shape [B, H_kv, N, D] with H_kv dividing H; got "
                         f"Q {tuple(q.shape)}, K {tuple(k.shape)}, V {tuple(v.shape)}")
    O, S, P = _unfused_module().run_unfused(q, k, v, return_intermediates)
    return (O, S, P) if return_intermediates else O
