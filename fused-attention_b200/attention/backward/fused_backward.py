"""Causal fused attention with a recompute-based backward pass and autograd, on B200 (sm_100a).

Drop-in for the reference's `attention/backward/fused_backward.py`: `FusedAttentionFn`
(:187-201), `fused_attention_autograd` (:204-206), `_check` (:151-158), `_forward` (:161-170)
and `_backward` (:173-184), with the same argument order, saved tensors and return values.

  forward : the sm_100a forward kernel also writes the log2-domain LSE (fp32 [B, H, N]) that
            the reference assembles on the host as m + log2(l) (:169), directly.
  backward: three launches on the current stream, all atomic-free:
            delta = rowsum(dO * O)              (preprocess kernel; the reference uses torch, :175)
            dK, dV  (one CTA per K/V tile, loops over the query tiles that see it; for GQA it
                     also loops over the query heads of the group, summing in TMEM)
            dQ      (one CTA per query tile pair, loops over visible K/V tiles)

Extensions over the reference (documented gaps it leaves open): bfloat16 as well as float16, and
GQA/MQA (k, v with H_kv heads dividing H) in the backward too.
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


def _check(q, k, v, tile_m, tile_n):
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must be float16 (or all bfloat16)")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"q, k, v must all be (B, H, N, D); got {q.shape}, {k.shape}, {v.shape}")
    B, H, N, D = q.shape
    H_kv = k.shape[1]
    if tuple(k.shape) != (B, H_kv, N, D) or v.shape != k.shape or H % H_kv != 0:
        raise ValueError(f"q, k, v must all be (B, H, N, D) (k, v may have H_kv | H heads); "
                         f"got {q.shape}, {k.shape}, {v.shape}")
    if N % tile_m or N % tile_n:
        raise ValueError(f"N={N} must be divisible by tile_m={tile_m} and tile_n={tile_n}")


def _forward(q, k, v, tile_m, tile_n, out=None):
    B, H, N, D = q.shape
    o = torch.empty_like(q) if out is None else out
    lse = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    nat = _native()
    nat.fwd(q, k, v, o, lse, tile_m, nat.kv_tile(tile_n))  # the backward kernels run 128 x 128 tiles
    return o, lse


def _backward_kv(q, k, v, o, lse, do, tile_m, tile_n, dk=None, dv=None):
    """First half of _backward: delta = rowsum(dO * O), then dK and dV (into dk / dv when given,
    contiguous tensors shaped like k).  Returns (delta, dk, dv)."""
    B, H, N, D = q.shape
    nat = _native()
    delta = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    nat.bwd_preprocess(o, do, delta)
    nat.bwd_dkdv(q, k, v, do, lse, delta, dk, dv, tile_m, tile_n)
    return delta, dk, dv


def _backward_q(q, k, v, do, lse, delta, tile_m, tile_n, dq=None):
    """Second half of _backward: dQ (into dq when given) from the delta of _backward_kv."""
    dq = torch.empty_like(q) if dq is None else dq
    _native().bwd_dq(q, k, v, do, lse, delta, dq, tile_m, tile_n)
    return dq


def _backward(q, k, v, o, lse, do, tile_m, tile_n):
    B, H, N, D = q.shape
    delta = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    _native().bwd(q, k, v, o, do, lse, delta, dq, dk, dv, tile_m, tile_n)  # delta, dK/dV, dQ
    return dq, dk, dv


class FusedAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, tile_m=64, tile_n=64):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        _check(q, k, v, tile_m, tile_n)
        o, lse = _forward(q, k, v, tile_m, tile_n)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.tiles = (tile_m, tile_n)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        dq, dk, dv = _backward(q, k, v, o, lse, do, *ctx.tiles)
        return dq, dk, dv, None, None


def fused_attention_autograd(q, k, v, tile_m=64, tile_n=64):
    """Causal attention (B, H, N, D) float16/bfloat16 with autograd support (k, v may be GQA)."""
    return FusedAttentionFn.apply(q, k, v, tile_m, tile_n)
