"""BASELINE config 5 at long context: causal GQA forward + backward, bf16, B=8, H=32, H_kv=8,
D=128, S in {16384, 32768}, through the public autograd API, against an fp32 reference computed on
the device in query-row chunks (a full S x S fp32 matrix per head would be 4 GiB at S=32768).

Every batch entry is sampled once (one K/V head per entry, its whole query-head group), so every
rank's shard of the batch-sharded multi-GPU layout is covered.  Per sample: O and the LSE on three
query-row windows (start, middle, end), dQ on the same windows, dK and dV on three key-row windows
(which sum over every query row at or after them, in all four query heads of the group).

Tolerances (written here): bf16 outputs use the elementwise rule |x - ref| <= 2e-2 + 2e-2 |ref|
(the reference's rule, tests/fused/run_correctness.py:33-35 in the reference) plus a relative
Frobenius error <= 2e-2 (tests/backward/run_correctness_backward.py:35-37); LSE relative error
<= 1e-3 (|ref| floored at 1).
"""
import math

import pytest
import torch

from tests.gpu_util import seeded

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634
CHUNK = 2048
REL = 2e-2


def _masked_scores(Qc, Kc, r0, c0, scale):
    s = (Qc @ Kc.T) * scale
    rows = torch.arange(r0, r0 + Qc.shape[0], device=Qc.device)[:, None]
    cols = torch.arange(c0, c0 + Kc.shape[0], device=Qc.device)[None, :]
    return s.masked_fill(cols > rows, float("-inf"))


def reference_group(q, k, v, do, b, g, q_windows, k_windows):
    """fp32 reference for batch b, K/V head g and its query-head group, on the device.
    Returns {"O": [per head, per window], "LSE2": ..., "dQ": ..., "dK": [per window], "dV": ...}."""
    H, H_kv, S, D = q.shape[1], k.shape[1], q.shape[2], q.shape[3]
    grp = H // H_kv
    scale = 1.0 / math.sqrt(D)
    K, V = k[b, g].float(), v[b, g].float()
    out = {"O": [], "LSE2": [], "dQ": [], "dK": [torch.zeros(c1 - c0, D, device=q.device) for c0, c1 in k_windows],
           "dV": [torch.zeros(c1 - c0, D, device=q.device) for c0, c1 in k_windows]}
    for h in range(g * grp, (g + 1) * grp):
        Q, dO = q[b, h].float(), do[b, h].float()
        lse = torch.empty(S, device=q.device)
        O = torch.empty(S, D, device=q.device)
        for r0 in range(0, S, CHUNK):
            r1 = r0 + CHUNK
            s = _masked_scores(Q[r0:r1], K[:r1], r0, 0, scale)
            lse[r0:r1] = torch.logsumexp(s, dim=-1)
            O[r0:r1] = torch.exp(s - lse[r0:r1, None]) @ V[:r1]
        delta = (dO * O).sum(-1)
        out["O"].append([O[r0:r1] for r0, r1 in q_windows])
        out["LSE2"].append([lse[r0:r1] * LOG2E for r0, r1 in q_windows])
        dqs = []
        for r0, r1 in q_windows:
            s = _masked_scores(Q[r0:r1], K[:r1], r0, 0, scale)
            p = torch.exp(s - lse[r0:r1, None])
            ds = p * (dO[r0:r1] @ V[:r1].T - delta[r0:r1, None])
            dqs.append(ds @ K[:r1] * scale)
        out["dQ"].append(dqs)
        for w, (c0, c1) in enumerate(k_windows):
            for r0 in range(c0 - c0 % CHUNK, S, CHUNK):
                r1 = r0 + CHUNK
                s = _masked_scores(Q[r0:r1], K[c0:c1], r0, c0, scale)
                p = torch.exp(s - lse[r0:r1, None])
                out["dV"][w] += p.T @ dO[r0:r1]
                ds = p * (dO[r0:r1] @ V[c0:c1].T - delta[r0:r1, None])
                out["dK"][w] += ds.T @ Q[r0:r1] * scale
    return out


def _close(name, got, ref):
    got = got.float()
    assert torch.isfinite(got).all(), name
    ratio = float(((got - ref).abs() / (2e-2 + 2e-2 * ref.abs())).max())
    rel = float((got - ref).norm() / ref.norm().clamp_min(1e-30))
    assert ratio <= 1.0 and rel <= REL, (name, ratio, rel)


@pytest.mark.parametrize("S", [16384, 32768])
def test_config5_long_context_fwd_bwd(S, cuda_device):
    from attention.backward.fused_backward import fused_attention_autograd, _forward, _native
    B, H, H_kv, D = 8, 32, 8, 128
    q = seeded(f"L5q{S}", (B, H, S, D), torch.bfloat16)
    k = seeded(f"L5k{S}", (B, H_kv, S, D), torch.bfloat16)
    v = seeded(f"L5v{S}", (B, H_kv, S, D), torch.bfloat16)
    do = seeded(f"L5d{S}", (B, H, S, D), torch.bfloat16)
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = fused_attention_autograd(qa, ka, va, 64, 128)
    o.backward(do)
    _, lse = _forward(q, k, v, 64, 128)
    _native().check_status(cuda_device)
    grp = H // H_kv
    q_windows = [(0, 128), (S // 2 - 64, S // 2 + 64), (S - 256, S)]
    k_windows = [(0, 128), (S // 2, S // 2 + 128), (S - 128, S)]
    for b in range(B):
        g = (3 * b + 1) % H_kv
        ref = reference_group(q, k, v, do, b, g, q_windows, k_windows)
        for i, h in enumerate(range(g * grp, (g + 1) * grp)):
            for w, (r0, r1) in enumerate(q_windows):
                _close(f"O b{b} h{h} w{w}", o[b, h, r0:r1], ref["O"][i][w])
                _close(f"dQ b{b} h{h} w{w}", qa.grad[b, h, r0:r1], ref["dQ"][i][w])
                r = ref["LSE2"][i][w]
                rel = float(((lse[b, h, r0:r1] - r).abs() / r.abs().clamp_min(1.0)).max())
                assert rel <= 1e-3, ("LSE", b, h, w, rel)
        for w, (c0, c1) in enumerate(k_windows):
            _close(f"dK b{b} g{g} w{w}", ka.grad[b, g, c0:c1], ref["dK"][w])
            _close(f"dV b{b} g{g} w{w}", va.grad[b, g, c0:c1], ref["dV"][w])
