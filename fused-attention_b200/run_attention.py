"""Command-line interface for causal attention on B200.

    python run_attention.py --input INPUT.npz --output OUTPUT.npy --backend cutile

Input:  .npz with contiguous float16 arrays Q, K, V, each [B, H, N, D];
        1<=B<=16, 1<=H<=32, 1<=N<=32768, D in {32, 64, 128}, N divisible by --block-m and --block-n
Output: .npy, float16, shape [B, H, N, D]
Backends: cutile / fused (sm_100a kernel), unfused (the three-kernel baseline on sm_100a),
reference (PyTorch fp32)
Exit status: 0 success, 2 unsupported input or usage error, 1 runtime failure.
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from attention.cli import EXIT_INVALID, EXIT_OK, EXIT_RUNTIME, OUTPUT_DTYPE, BACKENDS, load_qkv  # noqa: E402,F401
from attention.cli import main as _main  # noqa: E402
from attention.fused.validation import ValidationError, validate_qkv  # noqa: E402


def get_backend(name):
    """Return fn(q, k, v, block_m, block_n) -> torch.Tensor [B, H, N, D]. Imports lazily."""
    if name in ("cutile", "fused"):
        from attention.fused.fused import fused_attention
        return fused_attention
    if name == "unfused":
        from attention.fused.unfused import unfused_attention
        return lambda q, k, v, bm, bn: unfused_attention(q, k, v, bm, bn)
    if name == "reference":
        from attention.fused.reference import causal_attention_reference
        return lambda q, k, v, bm, bn: causal_attention_reference(q, k, v)
    raise NotImplementedError(f"backend '{name}' is not implemented")


def main(argv=None) -> int:
    return _main(argv, "Causal scaled dot-product attention on Q, K, V from an .npz file.",
                 get_backend, validate_qkv, ValidationError)


if __name__ == "__main__":
    sys.exit(main())
