"""CPU oracle for causal (GQA) attention forward, LSE and backward.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (fused-attention_b200/) imports this file;
only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as the checker.

What it restates (reference = nvidiacutile/fused-attention, paths inside that project):
  * causal_attention        the fp32 ground truth, attention/fused/reference.py:16-23 and the
                            GQA head mapping of attention/gqa/reference_gqa.py:15-43
  * lse_log2                the statistic the LSE-saving forward stores,
                            attention/backward/fused_backward.py:60-62,166-169
                            (m in log2 units of the scaled scores, lse = m + log2(l))
  * causal_attention_grads  dQ, dK, dV of the fp32 reference (the backward check of
                            tests/backward/run_correctness_backward.py:25-44), written out
                            analytically: dV = P^T dO, dP = dO V^T, dS = P (dP - delta),
                            dQ = dS K / sqrt(D), dK = dS^T Q / sqrt(D), delta = rowsum(dO O)
                            (attention/backward/fused_backward.py:1-12,175)
  * tiled_forward           the fused kernel's own algorithm, attention/fused/fused.py:34-64:
                            online softmax over K/V tiles in exp2 with the folded constant
                            log2(e)/sqrt(D), P rounded to the 16-bit input type before P V
  * make_inputs / case grids  the reference's seeded input generation
                            (tests/fused/cases.py:27-86, tests/gqa/cases_gqa.py:28-90)
  * tolerance rules         tests/fused/run_correctness.py:33-35,70-80 (elementwise),
                            tests/backward/run_correctness_backward.py:35-37 (relative norm)

Parity is pinned by tests/golden/*.npz, produced by running the reference's own PyTorch code
(see tests/golden/make_golden.py) and checked in tests/test_oracle.py.
"""
import math
import zlib
from dataclasses import dataclass

import numpy as np

LOG2E = 1.4426950408889634
ATOL = 2e-2
RTOL = 2e-2
REL_FLOOR = 1e-3


# ----------------------------------------------------------------------------- inputs
HEAD_DIMS = (32, 64, 128)
SEQ_LENS = (128, 512, 2048, 8192)
BATCH_HEADS = ((1, 1), (2, 8), (3, 5))
MAX_BATCH_HEADS = (16, 32)
MAX_SHAPE_SEQ_LENS = (128, 512)
MAGNITUDES = {"tiny": 0.03, "large": 7.0}
GQA_BATCH, GQA_HEADS, GQA_KV_HEADS = 4, 8, (1, 2, 4, 8)


@dataclass(frozen=True)
class Case:
    """One correctness case; `id` and `seed` follow tests/fused/cases.py:35-53 and
    tests/gqa/cases_gqa.py:38-64 (H_kv is part of the id only for GQA cases)."""
    B: int
    H: int
    N: int
    D: int
    magnitude: str
    H_kv: int = 0  # 0: MHA case (K/V have H heads)

    @property
    def kv_heads(self):
        return self.H_kv or self.H

    @property
    def id(self):
        if self.H_kv:
            return f"B{self.B}_H{self.H}_Hkv{self.H_kv}_N{self.N}_D{self.D}_{self.magnitude}"
        return f"B{self.B}_H{self.H}_N{self.N}_D{self.D}_{self.magnitude}"

    @property
    def sigma(self):
        return MAGNITUDES[self.magnitude]

    @property
    def seed(self):
        return zlib.crc32(self.id.encode())


def mha_cases():
    """The reference's 84 MHA forward cases, in its order (tests/fused/cases.py:56-72)."""
    cases = [Case(B, H, N, D, mag) for D in HEAD_DIMS for N in SEQ_LENS for mag in MAGNITUDES
             for B, H in BATCH_HEADS]
    B, H = MAX_BATCH_HEADS
    cases += [Case(B, H, N, D, mag) for N in MAX_SHAPE_SEQ_LENS for D in HEAD_DIMS for mag in MAGNITUDES]
    return cases


def gqa_cases():
    """The reference's 96 GQA forward cases, in its order (tests/gqa/cases_gqa.py:67-75)."""
    return [Case(GQA_BATCH, GQA_HEADS, N, D, mag, H_kv) for D in HEAD_DIMS for N in SEQ_LENS
            for mag in MAGNITUDES for H_kv in GQA_KV_HEADS]


def make_inputs(case):
    """float16 Q [B,H,N,D], K, V [B,H_kv,N,D]: standard normal, Q and K scaled by sigma, drawn in
    the order Q, K, V from default_rng(crc32(case id)) (tests/fused/cases.py:75-86)."""
    rng = np.random.default_rng(case.seed)
    qs = (case.B, case.H, case.N, case.D)
    kvs = (case.B, case.kv_heads, case.N, case.D)
    q = (rng.standard_normal(qs, dtype=np.float32) * case.sigma).astype(np.float16)
    k = (rng.standard_normal(kvs, dtype=np.float32) * case.sigma).astype(np.float16)
    v = rng.standard_normal(kvs, dtype=np.float32).astype(np.float16)
    return q, k, v


def seeded_normal(name, shape, sigma=1.0, dtype=np.float16):
    """i.i.d. N(0, sigma^2) array seeded by crc32(name): the reproducibility rule of the
    reference's case generators, applied to the BASELINE configurations."""
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    return (rng.standard_normal(shape, dtype=np.float32) * sigma).astype(dtype)


# ----------------------------------------------------------------------------- forward
def _expand(kv, H):
    """[B, H_kv, N, D] -> [B, H, N, D]: query head h uses K/V head h // (H // H_kv)."""
    H_kv = kv.shape[1]
    if H % H_kv:
        raise ValueError(f"H={H} not divisible by H_kv={H_kv}")
    return kv if H_kv == H else np.repeat(kv, H // H_kv, axis=1)


def _scores(q, k):
    """Masked fp32 scores q k^T / sqrt(D) (strict upper triangle = -inf)."""
    q32 = q.astype(np.float32)
    k32 = _expand(k, q.shape[1]).astype(np.float32)
    n, d = q.shape[-2], q.shape[-1]
    s = np.matmul(q32, np.swapaxes(k32, -1, -2)) / np.float32(math.sqrt(d))
    s[..., np.triu(np.ones((n, n), dtype=bool), 1)] = -np.inf
    return s


def _softmax(s):
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    return p / p.sum(axis=-1, keepdims=True)


def causal_attention(q, k, v):
    """fp32 causal (GQA) attention [B, H, N, D] (attention/fused/reference.py:16-23)."""
    p = _softmax(_scores(q, k))
    return np.matmul(p, _expand(v, q.shape[1]).astype(np.float32))


def lse_log2(q, k):
    """log2-domain LSE of the scaled, masked scores, float32 [B, H, N]
    (attention/backward/fused_backward.py:60-62,169: lse = m + log2(l), m in log2 units)."""
    s = _scores(q, k).astype(np.float64) * LOG2E
    m = s.max(axis=-1, keepdims=True)
    return (m[..., 0] + np.log2(np.exp2(s - m).sum(axis=-1))).astype(np.float32)


def causal_attention_grads(q, k, v, do):
    """(O, dQ, dK, dV) in fp32 for the fp32 reference; dK/dV of a K/V head sum its group."""
    B, H, N, D = q.shape
    H_kv = k.shape[1]
    p = _softmax(_scores(q, k))
    q32 = q.astype(np.float32)
    k32 = _expand(k, H).astype(np.float32)
    v32 = _expand(v, H).astype(np.float32)
    do32 = do.astype(np.float32)
    o = np.matmul(p, v32)
    dv_full = np.matmul(np.swapaxes(p, -1, -2), do32)
    dp = np.matmul(do32, np.swapaxes(v32, -1, -2))
    delta = (do32 * o).sum(-1, keepdims=True)
    ds = p * (dp - delta)
    sm = np.float32(1.0 / math.sqrt(D))
    dq = np.matmul(ds, k32) * sm
    dk_full = np.matmul(np.swapaxes(ds, -1, -2), q32) * sm
    g = H // H_kv
    dk = dk_full.reshape(B, H_kv, g, N, D).sum(2)
    dv = dv_full.reshape(B, H_kv, g, N, D).sum(2)
    return o, dq, dk, dv


def delta_rowsum(o, do):
    """delta = rowsum(dO * O) in fp32 (attention/backward/fused_backward.py:175)."""
    return (do.astype(np.float32) * o.astype(np.float32)).sum(-1)


def tiled_forward(q, k, v, tile_m=64, tile_n=64, p_dtype=np.float16):
    """The fused kernel's algorithm (attention/fused/fused.py:34-64), vectorised over a query tile.

    Returns (O fp32 before the final cast, lse log2).  Small cases only (pure NumPy loops over
    tiles)."""
    B, H, N, D = q.shape
    kx = _expand(k, H).astype(np.float32)
    vx = _expand(v, H).astype(np.float32)
    q32 = q.astype(np.float32)
    scale = np.float32(LOG2E / math.sqrt(D))
    out = np.zeros((B, H, N, D), np.float32)
    lse = np.zeros((B, H, N), np.float32)
    for b in range(B):
        for h in range(H):
            for i in range(N // tile_m):
                rows = i * tile_m + np.arange(tile_m)[:, None]
                qt = q32[b, h, i * tile_m:(i + 1) * tile_m]
                m = np.full((tile_m, 1), -np.inf, np.float32)
                l = np.zeros((tile_m, 1), np.float32)
                acc = np.zeros((tile_m, D), np.float32)
                n_kv = ((i + 1) * tile_m + tile_n - 1) // tile_n
                mask_start = (i * tile_m) // tile_n
                for j in range(n_kv):
                    kt = kx[b, h, j * tile_n:(j + 1) * tile_n]
                    vt = vx[b, h, j * tile_n:(j + 1) * tile_n]
                    s = qt @ kt.T
                    if j >= mask_start:
                        cols = j * tile_n + np.arange(tile_n)[None, :]
                        s = np.where(cols > rows, -np.inf, s)
                    m_new = np.maximum(m, s.max(-1, keepdims=True) * scale)
                    alpha = np.exp2(m - m_new)
                    p = np.exp2(s * scale - m_new)
                    l = l * alpha + p.sum(-1, keepdims=True)
                    acc = acc * alpha + p.astype(p_dtype).astype(np.float32) @ vt
                    m = m_new
                out[b, h, i * tile_m:(i + 1) * tile_m] = acc / l
                lse[b, h, i * tile_m:(i + 1) * tile_m] = (m + np.log2(l))[:, 0]
    return out, lse


# ----------------------------------------------------------------------------- comparisons
def elementwise_ratio(out, ref):
    """max |out-ref| / (ATOL + RTOL |ref|); pass iff <= 1 (tests/fused/run_correctness.py:70-80)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    if not np.isfinite(out).all():
        return float("inf")
    return float((np.abs(out - ref) / (ATOL + RTOL * np.abs(ref))).max())


def max_abs(out, ref):
    return float(np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64)).max())


def rel_fro(out, ref):
    """||out - ref|| / ||ref|| (tests/backward/run_correctness_backward.py:35-37)."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-12))


def lse_rel_err(out, ref):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), 1.0)).max())
