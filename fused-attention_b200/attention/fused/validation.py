"""Input contract of the MHA path (CLI, kernels, tests).

Mirrors the reference's `attention/fused/validation.py:37-88` (same function, exception type
and message wording) with the limits the B200 kernels support:
  Q, K, V: [B, H, N, D], contiguous, all float16 or all bfloat16 (the reference: float16 only)
  1 <= B <= 16, 1 <= H <= 32, 1 <= N <= 32768 (the reference: 8192), D in {32, 64, 128}
  N divisible by the query tile (block_m) and key tile (block_n)
Works on NumPy arrays and torch tensors (anything with .shape and .dtype).
"""

MAX_BATCH = 16
MAX_HEADS = 32
MAX_SEQ_LEN = 32768
SUPPORTED_HEAD_DIMS = (32, 64, 128)
SUPPORTED_DTYPES = ("float16", "bfloat16")


class ValidationError(ValueError):
    """Raised for inputs outside the supported scope."""


def _dtype_name(x) -> str:
    return str(x.dtype).replace("torch.", "")


def _is_contiguous(x) -> bool:
    if hasattr(x, "is_contiguous"):
        return x.is_contiguous()
    flags = getattr(x, "flags", None)
    return True if flags is None else bool(flags["C_CONTIGUOUS"])


def check_tensors(tensors):
    """dtype / rank / contiguity checks shared by the MHA and GQA contracts."""
    dtypes = set()
    for name, t in tensors.items():
        dt = _dtype_name(t)
        if dt not in SUPPORTED_DTYPES:
            raise ValidationError(f"{name} has dtype {dt}; only float16 and bfloat16 are supported")
        dtypes.add(dt)
        if len(t.shape) != 4:
            raise ValidationError(
                f"{name} must be 4-D [B, H, N, D], got {len(t.shape)}-D shape {tuple(t.shape)}")
        if not _is_contiguous(t):
            raise ValidationError(f"{name} must be contiguous")
    if len(dtypes) > 1:
        raise ValidationError(f"Q, K and V must share one dtype, got {sorted(dtypes)}")


def check_ranges(B, H, Nq, D, block_m, block_n):
    if not 1 <= B <= MAX_BATCH:
        raise ValidationError(f"batch size B={B} out of range [1, {MAX_BATCH}]")
    if not 1 <= H <= MAX_HEADS:
        raise ValidationError(f"head count H={H} out of range [1, {MAX_HEADS}]")
    if not 1 <= Nq <= MAX_SEQ_LEN:
        raise ValidationError(f"sequence length N={Nq} out of range [1, {MAX_SEQ_LEN}]")
    if D not in SUPPORTED_HEAD_DIMS:
        raise ValidationError(f"head dim D={D} not supported; allowed {SUPPORTED_HEAD_DIMS}")
    for label, block in (("query tile block_m", block_m), ("key tile block_n", block_n)):
        if block <= 0:
            raise ValidationError(f"{label}={block} must be positive")
        if Nq % block != 0:
            raise ValidationError(
                f"sequence length N={Nq} is not divisible by the {label}={block}; "
                f"use N that is a multiple of {block} (partial edge tiles are not supported)")


def validate_qkv(q, k, v, block_m: int, block_n: int) -> None:
    """Raise ValidationError if Q, K, V are not supported for the given tile sizes."""
    check_tensors({"Q": q, "K": k, "V": v})
    B, H, Nq, D = q.shape
    Bk, Hk, Nk, Dk = k.shape
    Bv, Hv, Nv, Dv = v.shape
    if not (B == Bk == Bv):
        raise ValidationError(f"batch size mismatch: Q={B}, K={Bk}, V={Bv}")
    if not (H == Hk == Hv):
        raise ValidationError(f"head count mismatch: Q={H}, K={Hk}, V={Hv}")
    if not (Nq == Nk == Nv):
        raise ValidationError(
            f"sequence length mismatch: Q={Nq}, K={Nk}, V={Nv}; causal self-attention needs Nq == Nk")
    if not (D == Dk == Dv):
        raise ValidationError(
            f"head dim mismatch: Q={D}, K={Dk}, V={Dv}; Q, K and V must share the same head dim D")
    check_ranges(B, H, Nq, D, block_m, block_n)
