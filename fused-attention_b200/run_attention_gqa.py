"""Command-line interface for causal grouped-query attention (GQA/MQA) on B200.

    python run_attention_gqa.py --input INPUT.npz --output OUTPUT.npy --backend cutile

Input:  .npz with Q [B, H, N, D], K and V [B, H_kv, N, D] (float16), H_kv dividing H;
        query head h reads K/V head h // (H // H_kv)
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
from attention.gqa.validation_gqa import ValidationError, validate_qkv  # noqa: E402


def get_backend(name):
    """Return fn(q, k, v, block_m, block_n) -> torch.Tensor [B, H, N, D]. Imports lazily."""
    if name in ("cutile", "fused"):
        from attention.gqa.fused_gqa import fused_gqa_attention
        return fused_gqa_attention
    if name == "unfused":
        from attention.gqa.unfused_gqa import unfused_gqa_attention
        return lambda q, k, v, bm, bn: unfused_gqa_attention(q, k, v, bm, bn)
    if name == "reference":
        from attention.gqa.reference_gqa import causal_attention_reference_gqa
        return lambda q, k, v, bm, bn: causal_attention_reference_gqa(q, k, v)
    raise NotImplementedError(f"backend '{name}' is not implemented")


def main(argv=None) -> int:
    return _main(argv, "Causal grouped-query attention on Q, K, V from an .npz file.",
                 get_backend, validate_qkv, ValidationError)


if __name__ == "__main__":
    sys.exit(main())
