"""ctypes binding of libfa_sm100.so, the sm_100a kernels behind a C ABI (include/fa_sm100.h).

This module is self-contained (it imports nothing else from the package) so the public kernel
files can load it by path when they are themselves imported by path, the way the reference's
runners import a kernel file (`tests/fused/run_correctness.py:107-122` in the reference).

There is no fallback: if the shared library is missing or the device is not an sm_100 GPU, the
calls raise.  Tensors cross the boundary as raw device pointers plus sizes; the CUDA stream is
torch's current stream, so the kernels order with surrounding torch work exactly like the
reference's `ct.launch(torch.cuda.current_stream(), ...)` (attention/fused/fused.py:75).
"""
import contextlib
import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfa_sm100.so")
ABI_VERSION = 1



def kv_tile(tile_n):
    """K/V tile (keys per tile) of the forward kernel for the reference's `tile_n` knob: the sm_100a
    forward has 64- and 128-key variants, so tile_n <= 64 runs the 64-key tile and larger tile_n
    the 128-key tile (the faster one on B200: 18-19 % at N = 8192).  The query side always runs
    128-row tcgen05 tiles, so tile_m takes part only in the caller's divisibility rule."""
    return 64 if int(tile_n) <= 64 else 128

FA_OK = 0
FA_ERR_INVALID_ARG = 1
FA_ERR_UNSUPPORTED = 2
FA_ERR_ALIGNMENT = 3
FA_ERR_CUDA = 4
FA_ERR_DRIVER = 5
FA_ERR_DEVICE = 6
FA_ERR_TOO_LARGE = 7

# exported symbol -> (argtypes) ; every entry point returns int
_VP, _I, _FP = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
SIGNATURES = {
    "fa_abi_version": [],
    "fa_strerror": [_I],
    "fa_last_cuda_error": [],
    "fa_fwd": [_VP, _VP, _VP, _VP, _FP, _I, _I, _I, _I, _I, _I, _I, _I, _VP, _VP],
    "fa_bwd_preprocess": [_VP, _VP, _FP, _I, _I, _I, _I, _I, _VP, _VP],
    "fa_bwd_dkdv": [_VP, _VP, _VP, _VP, _FP, _FP, _VP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _VP, _VP],
    "fa_bwd_dq": [_VP, _VP, _VP, _VP, _FP, _FP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _VP, _VP],
    "fa_bwd_noalloc": [_VP, _VP, _VP, _VP, _VP, _FP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _I, _I, _VP, _VP],
    "fa_unfused_fwd": [_VP, _VP, _VP, _VP, _FP, _VP, _I, _I, _I, _I, _I, _I, _VP, _VP],
}
_RESTYPES = {"fa_strerror": ctypes.c_char_p, "fa_last_cuda_error": ctypes.c_char_p}

_lib = None
_lock = threading.Lock()
_status = {}  # device index -> int32[4] status tensor

DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1}


class KernelError(RuntimeError):
    """A device-side pipeline wait timed out (the kernel stopped instead of hanging)."""


def load():
    """Load (once) and return the ctypes handle of libfa_sm100.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python fused-attention_b200/build.py` "
                    "(this library has no non-CUDA fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            if lib.fa_abi_version() != ABI_VERSION:
                raise RuntimeError(f"libfa_sm100.so ABI {lib.fa_abi_version()} != {ABI_VERSION}; rebuild it")
            _lib = lib
    return _lib


def status_tensor(device):
    """Per-device int32[4] status word the kernels report pipeline timeouts into."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    st = _status.get(idx)
    if st is None:
        with _lock:
            st = _status.get(idx)
            if st is None:
                st = torch.zeros(4, dtype=torch.int32, device=f"cuda:{idx}")
                _status[idx] = st
    return st


def check_status(device=None, reset=True):
    """Synchronise `device` and raise KernelError if a kernel recorded a timeout."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    st = status_tensor(device)
    vals = st.tolist()  # synchronises with the device
    if vals[0] != 0:
        if reset:
            st.zero_()
        raise KernelError(f"device pipeline error code {vals[0]} (cta {vals[1]}, thread {vals[2]})")


def _raise(rc, what):
    lib = load()
    msg = lib.fa_strerror(rc).decode()
    if rc == FA_ERR_CUDA:
        msg += ": " + lib.fa_last_cuda_error().decode()
    if rc in (FA_ERR_INVALID_ARG, FA_ERR_UNSUPPORTED, FA_ERR_ALIGNMENT, FA_ERR_TOO_LARGE):
        raise ValueError(f"{what}: {msg}")  # the caller's arguments
    raise RuntimeError(f"{what}: {msg}")  # CUDA, driver or device


# Raw cudaStream_t of a device's current stream without building a torch Stream object (a
# measurable part of a short call's host time); the public query where torch lacks it.
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream(idx):
    if _RAW_STREAM is not None:
        return _RAW_STREAM(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _dtype_code(t):
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise TypeError(f"dtype {t.dtype} is not supported (float16 or bfloat16)")
    return code


def _launch(t, calls):
    """Run the C entry points `calls` [(name, args)] on t's device: each call gets the device's
    status word and the raw handle of its current stream appended (pointers travel as plain ints,
    which the c_void_p argtypes convert).  Raises on the first non-zero return code."""
    lib = load()
    idx = t.get_device()
    status = status_tensor(t.device).data_ptr()
    stream = _current_stream(idx)
    ctx = contextlib.nullcontext() if idx == torch.cuda.current_device() else torch.cuda.device(idx)
    with ctx:
        for name, args in calls:
            rc = getattr(lib, name)(*args, status, stream)
            if rc != FA_OK:
                _raise(rc, name)


def _p(t):
    return t.data_ptr() if t is not None else None


def fwd(q, k, v, o, lse, tile_m, tile_n):
    """Enqueue the forward kernel: o (and lse if not None) from q, k, v (all contiguous CUDA)."""
    B, H, S, D = q.shape
    _launch(q, [("fa_fwd", (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _p(lse), B, H, k.shape[1],
                            S, D, _dtype_code(q), int(tile_m), int(tile_n)))])


def bwd_preprocess(o, do, delta):
    B, H, S, D = o.shape
    _launch(o, [("fa_bwd_preprocess", (o.data_ptr(), do.data_ptr(), delta.data_ptr(), B, H, S, D, _dtype_code(o)))])


def _dkdv_args(q, k, v, do, lse, delta, dk, dv, tile_m, tile_n):
    B, H, S, D = q.shape
    return (q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), B, H, k.shape[1], S, D, _dtype_code(q), int(tile_m), int(tile_n))


def _dq_args(q, k, v, do, lse, delta, dq, tile_m, tile_n):
    B, H, S, D = q.shape
    return (q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr(),
            dq.data_ptr(), B, H, k.shape[1], S, D, _dtype_code(q), int(tile_m), int(tile_n))


def bwd_dkdv(q, k, v, do, lse, delta, dk, dv, tile_m, tile_n):
    _launch(q, [("fa_bwd_dkdv", _dkdv_args(q, k, v, do, lse, delta, dk, dv, tile_m, tile_n))])


def bwd_dq(q, k, v, do, lse, delta, dq, tile_m, tile_n):
    _launch(q, [("fa_bwd_dq", _dq_args(q, k, v, do, lse, delta, dq, tile_m, tile_n))])


def bwd(q, k, v, o, do, lse, delta, dq, dk, dv, tile_m, tile_n):
    """The whole backward: delta, then dK/dV, then dQ, enqueued in one go."""
    B, H, S, D = o.shape
    _launch(q, [("fa_bwd_preprocess", (o.data_ptr(), do.data_ptr(), delta.data_ptr(), B, H, S, D, _dtype_code(o))),
                ("fa_bwd_dkdv", _dkdv_args(q, k, v, do, lse, delta, dk, dv, tile_m, tile_n)),
                ("fa_bwd_dq", _dq_args(q, k, v, do, lse, delta, dq, tile_m, tile_n))])


def unfused_fwd(q, k, v, o, s, p):
    """Enqueue the unfused three-kernel forward: s (fp32 [B, H, N, N]) = masked scaled scores,
    p (dtype of q, [B, H, N, N]) = row softmax, o = p v."""
    B, H, S, D = q.shape
    _launch(q, [("fa_unfused_fwd", (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), s.data_ptr(),
                                    p.data_ptr(), B, H, k.shape[1], S, D, _dtype_code(q)))])


def load_by_path():
    """Return this module (used by files that are imported by path)."""
    import sys
    return sys.modules[__name__]
