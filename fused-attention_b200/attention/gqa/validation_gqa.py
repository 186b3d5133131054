"""Input contract of the GQA/MQA path.

Mirrors the reference's `attention/gqa/validation_gqa.py:39-104` (same function, exception type,
messages and return value: the group size H // H_kv) with the B200 limits of
`attention/fused/validation.py` (float16 or bfloat16, N <= 32768, D in {32, 64, 128}).
  Q: [B, H, N, D]   K, V: [B, H_kv, N, D]   1 <= H_kv <= H, H % H_kv == 0
"""
import importlib.util
import os
import sys


def _mha_validation():
    if __package__:  # imported as attention.gqa.validation_gqa: share the package's class
        from ..fused import validation
        return validation
    name = "_fa_b200_validation"
    mod = sys.modules.get(name)
    if mod is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fused", "validation.py")
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return mod


_v = _mha_validation()
ValidationError = _v.ValidationError
MAX_BATCH, MAX_HEADS, MAX_SEQ_LEN = _v.MAX_BATCH, _v.MAX_HEADS, _v.MAX_SEQ_LEN
SUPPORTED_HEAD_DIMS = _v.SUPPORTED_HEAD_DIMS


def validate_qkv(q, k, v, block_m: int, block_n: int) -> int:
    """Raise ValidationError if Q, K, V are not supported; return the group size H // H_kv."""
    _v.check_tensors({"Q": q, "K": k, "V": v})
    B, H, Nq, D = q.shape
    Bk, Hk, Nk, Dk = k.shape
    Bv, Hv, Nv, Dv = v.shape
    if not (B == Bk == Bv):
        raise ValidationError(f"batch size mismatch: Q={B}, K={Bk}, V={Bv}")
    if Hk != Hv:
        raise ValidationError(f"K/V head count mismatch: K={Hk}, V={Hv}; K and V must have the same H_kv")
    if not (Nq == Nk == Nv):
        raise ValidationError(
            f"sequence length mismatch: Q={Nq}, K={Nk}, V={Nv}; causal self-attention needs Nq == Nk")
    if not (D == Dk == Dv):
        raise ValidationError(
            f"head dim mismatch: Q={D}, K={Dk}, V={Dv}; Q, K and V must share the same head dim D")
    if not 1 <= B <= MAX_BATCH:
        raise ValidationError(f"batch size B={B} out of range [1, {MAX_BATCH}]")
    if not 1 <= H <= MAX_HEADS:
        raise ValidationError(f"head count H={H} out of range [1, {MAX_HEADS}]")
    H_kv = Hk
    if not 1 <= H_kv <= H:
        raise ValidationError(f"KV head count H_kv={H_kv} out of range [1, H={H}]")
    if H % H_kv != 0:
        raise ValidationError(
            f"query heads H={H} not divisible by KV heads H_kv={H_kv}; "
            f"H_kv must divide H (each group of H // H_kv query heads shares one K/V head)")
    _v.check_ranges(B, H, Nq, D, block_m, block_n)
    return H // H_kv
