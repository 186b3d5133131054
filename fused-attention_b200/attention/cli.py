"""Shared implementation of the two command-line drivers (run_attention.py, run_attention_gqa.py).

Behaviour follows the reference's `run_attention.py:33-130` / `run_attention_gqa.py`:
.npz with arrays Q, K, V in, .npy (float16) out; exit status 0 success, 2 unsupported input or
usage error, 1 runtime failure; non-finite or wrongly shaped output is a runtime failure.

Backends: `cutile` (the reference's name for its fused kernel; here the sm_100a kernel),
`fused` (alias of `cutile`), `unfused` (the reference's 3-kernel cuTile baseline: not built on
B200, reported as not implemented, exit 1), `reference` (PyTorch fp32).
"""
import argparse
import sys
import time

import numpy as np

OUTPUT_DTYPE = np.float16
EXIT_OK, EXIT_RUNTIME, EXIT_INVALID = 0, 1, 2
BACKENDS = ("cutile", "fused", "unfused", "reference")


def parse_args(argv, description):
    p = argparse.ArgumentParser(description=description)
    p.add_argument("--input", required=True, help="input .npz containing Q, K, V")
    p.add_argument("--output", required=True, help="output .npy path")
    p.add_argument("--backend", choices=BACKENDS, default="cutile", help="implementation to run (default: cutile)")
    p.add_argument("--block-m", type=int, default=64, help="query tile size (default: 64)")
    p.add_argument("--block-n", type=int, default=64, help="key/value tile size (default: 64)")
    p.add_argument("--verbose", action="store_true", help="print shapes and timing to stderr")
    return p.parse_args(argv)


def load_qkv(path, ValidationError):
    """Load Q, K, V from an .npz file, raising ValidationError for missing or malformed files."""
    try:
        with np.load(path, allow_pickle=False) as data:
            missing = [key for key in ("Q", "K", "V") if key not in data.files]
            if missing:
                raise ValidationError(f"{path} is missing array(s) {', '.join(missing)}; found {sorted(data.files)}")
            return data["Q"], data["K"], data["V"]
    except FileNotFoundError:
        raise ValidationError(f"input file not found: {path}")
    except (OSError, ValueError) as e:
        if isinstance(e, ValidationError):
            raise
        raise ValidationError(f"could not read {path} as .npz: {e}")


def _to_torch(x):
    """NumPy (float16) array -> contiguous torch CUDA tensor."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run(q, k, v, fn, block_m, block_n):
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA GPU visible to PyTorch")
    q_t, k_t, v_t = (_to_torch(x) for x in (q, k, v))
    out = fn(q_t, k_t, v_t, block_m, block_n)
    torch.cuda.synchronize()
    return out.to(torch.float16).cpu().numpy()


def main(argv, description, get_backend, validate_qkv, ValidationError):
    args = parse_args(argv, description)
    try:
        q, k, v = load_qkv(args.input, ValidationError)
        validate_qkv(q, k, v, args.block_m, args.block_n)
    except ValidationError as e:
        print(f"error: {e}", file=sys.stderr)
        return EXIT_INVALID
    if args.verbose:
        print(f"Q{q.shape} K{k.shape} V{v.shape} backend={args.backend} "
              f"block_m={args.block_m} block_n={args.block_n}", file=sys.stderr)
    try:
        fn = get_backend(args.backend)  # resolve first so unimplemented backends fail fast
        t0 = time.perf_counter()
        out = run(q, k, v, fn, args.block_m, args.block_n)
        elapsed = time.perf_counter() - t0
    except NotImplementedError as e:
        print(f"error: {str(e) or f'backend {args.backend!r} is not implemented yet'}", file=sys.stderr)
        return EXIT_RUNTIME
    except ModuleNotFoundError as e:
        print(f"error: missing dependency '{e.name}'", file=sys.stderr)
        return EXIT_RUNTIME
    except Exception as e:  # kernel/driver failures
        print(f"error: {args.backend} backend failed: {type(e).__name__}: {e}", file=sys.stderr)
        return EXIT_RUNTIME
    expected = q.shape[:3] + (v.shape[3],)
    if out.shape != expected:
        print(f"error: backend returned shape {out.shape}, expected {expected}", file=sys.stderr)
        return EXIT_RUNTIME
    if not np.isfinite(out).all():
        print("error: output contains NaN or Inf", file=sys.stderr)
        return EXIT_RUNTIME
    np.save(args.output, out.astype(OUTPUT_DTYPE, copy=False))
    if args.verbose:
        print(f"wrote {args.output} {out.shape} {OUTPUT_DTYPE.__name__} in {elapsed:.3f}s "
              f"(includes transfer)", file=sys.stderr)
    return EXIT_OK
