"""Shared implementation of the two command-line drivers (run_attention.py, run_attention_gqa.py).

Behaviour follows the reference's `run_attention.py:33-130` / `run_attention_gqa.py`:
.npz with arrays Q, K, V in, .npy (float16) out; exit status 0 success, 2 unsupported input or
usage error, 1 runtime failure; non-finite or wrongly shaped output is a runtime failure.

Backends: `cutile` (the reference's name for its fused kernel; here the sm_100a kernel),
`fused` (alias of `cutile`), `unfused` (the reference's three-kernel baseline, as sm_100a
kernels), `reference` (PyTorch fp32).
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


class _Exit(Exception):
    """Ends the CLI with `code` after printing `error: <message>` to stderr."""

    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


_NPZ_KEYS = ("Q", "K", "V")


def load_qkv(path, ValidationError):
    """Q, K, V arrays of an .npz file; ValidationError (with the reference's messages) when the file
    is absent, unreadable or lacks one of the three arrays."""
    try:
        archive = np.load(path, allow_pickle=False)
    except FileNotFoundError:
        raise ValidationError(f"input file not found: {path}") from None
    except (OSError, ValueError) as e:
        raise ValidationError(f"could not read {path} as .npz: {e}") from None
    with archive:
        absent = [name for name in _NPZ_KEYS if name not in archive.files]
        if absent:
            raise ValidationError(f"{path} is missing array(s) {', '.join(absent)}; found {sorted(archive.files)}")
        try:
            return tuple(archive[name] for name in _NPZ_KEYS)
        except (OSError, ValueError) as e:
            raise ValidationError(f"could not read {path} as .npz: {e}") from None


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


def _inputs(args, validate_qkv, ValidationError):
    """Loaded and validated Q, K, V; an invalid input ends the CLI with exit status 2."""
    try:
        q, k, v = load_qkv(args.input, ValidationError)
        validate_qkv(q, k, v, args.block_m, args.block_n)
    except ValidationError as e:
        raise _Exit(EXIT_INVALID, str(e)) from None
    return q, k, v


def _runtime_message(backend, err):
    """The message for a failure while resolving or running a backend (exit status 1)."""
    if isinstance(err, NotImplementedError):
        return str(err) or f"backend {backend!r} is not implemented yet"
    if isinstance(err, ModuleNotFoundError):
        return f"missing dependency '{err.name}'"
    return f"{backend} backend failed: {type(err).__name__}: {err}"


def _compute(args, get_backend, q, k, v):
    """(output array, seconds).  The backend is looked up before any data moves to the GPU, so an
    unavailable backend is reported without touching the device."""
    try:
        fn = get_backend(args.backend)
        t0 = time.perf_counter()
        out = run(q, k, v, fn, args.block_m, args.block_n)
        return out, time.perf_counter() - t0
    except Exception as e:
        raise _Exit(EXIT_RUNTIME, _runtime_message(args.backend, e)) from None


def _check_output(out, q, v):
    """A wrongly shaped or non-finite result is a runtime failure (exit status 1)."""
    expected = q.shape[:3] + (v.shape[3],)
    if out.shape != expected:
        raise _Exit(EXIT_RUNTIME, f"backend returned shape {out.shape}, expected {expected}")
    if not np.isfinite(out).all():
        raise _Exit(EXIT_RUNTIME, "output contains NaN or Inf")


def main(argv, description, get_backend, validate_qkv, ValidationError):
    args = parse_args(argv, description)
    say = (lambda text: print(text, file=sys.stderr)) if args.verbose else (lambda text: None)
    try:
        q, k, v = _inputs(args, validate_qkv, ValidationError)
        say(f"Q{q.shape} K{k.shape} V{v.shape} backend={args.backend} "
            f"block_m={args.block_m} block_n={args.block_n}")
        out, seconds = _compute(args, get_backend, q, k, v)
        _check_output(out, q, v)
    except _Exit as stop:
        print(f"error: {stop}", file=sys.stderr)
        return stop.code
    np.save(args.output, out.astype(OUTPUT_DTYPE, copy=False))
    say(f"wrote {args.output} {out.shape} {OUTPUT_DTYPE.__name__} in {seconds:.3f}s (includes transfer)")
    return EXIT_OK
