"""Unfused causal attention baseline on B200 (sm_100a): the reference's three-kernel path.

Drop-in for the reference's `attention/fused/unfused.py` (`unfused_attention`, :96-116): same
name, arguments, return values and errors.  Three kernels run on torch's current stream through
the C ABI (`fa_unfused_fwd`), with the scores and probabilities materialised in global memory:

  1. S = causal_mask(Q K^T / sqrt(D))   fp32 [B, H, N, N]   (TMA + tcgen05 UMMA)
  2. P = row_softmax(S)                 dtype of q           (two passes per row, HBM-bound)
  3. O = P V                                                (TMA + tcgen05 UMMA)

Only tiles on or below the causal diagonal are computed, read or written; with
return_intermediates=True the buffers start as -inf / 0, so the returned S and P are clean.
S and P are full B*H*N*N buffers, as in the reference.
"""
import importlib.util
import os
import sys

import torch


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


def run_unfused(q, k, v, return_intermediates):
    """Allocate S, P and O, launch the three kernels; (O, S, P)."""
    B, H, N, D = q.shape
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if return_intermediates:
        S = torch.full((B, H, N, N), float("-inf"), device=q.device, dtype=torch.float32)
        P = torch.zeros((B, H, N, N), device=q.device, dtype=q.dtype)
    else:
        S = torch.empty((B, H, N, N), device=q.device, dtype=torch.float32)
        P = torch.empty((B, H, N, N), device=q.device, dtype=q.dtype)
    O = torch.empty_like(q)
    _native().unfused_fwd(q, k, v, O, S, P)
    return O, S, P


def unfused_attention(q, k, v, tile_m=64, tile_n=64, return_intermediates=False):
    """Causal attention (B, H, N, D) through materialised S and P; tile_m / tile_n keep the
    reference's divisibility rule (the kernels run 128 x 128 tiles)."""
    B, H, N, D = q.shape
    if N % tile_m != 0 or N % tile_n != 0:
        raise ValueError(f"N={N} must be divisible by tile_m={tile_m} and tile_n={tile_n}")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must all be (B, H, N, D); got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    O, S, P = run_unfused(q, k, v, return_intermediates)
    return (O, S, P) if return_intermediates else O
