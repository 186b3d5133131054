"""Helpers shared by the GPU parity tests (device-side fp32 reference for large shapes)."""
import math

import numpy as np
import torch

LOG2E = 1.4426950408889634


def to_dev(x, dtype=torch.float16, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=dtype)


def seeded(name, shape, dtype, sigma=1.0, device="cuda"):
    """i.i.d. N(0, sigma^2) drawn on the device from a generator seeded by crc32(name)."""
    import zlib
    g = torch.Generator(device=device).manual_seed(zlib.crc32(name.encode()))
    return (torch.randn(shape, device=device, generator=g, dtype=torch.float32) * sigma).to(dtype)


def reference_rows(q, k, v, b, h, rows, with_lse=False):
    """fp32 causal attention for query rows `rows` (a slice) of head (b, h), on the device.
    K/V head = h // (H // H_kv)  (the reference's GQA mapping)."""
    H, H_kv = q.shape[1], k.shape[1]
    kv = h // (H // H_kv)
    D = q.shape[-1]
    r0, r1 = rows.start, rows.stop
    qf = q[b, h, r0:r1].float()
    kf = k[b, kv, :r1].float()
    vf = v[b, kv, :r1].float()
    s = (qf @ kf.T) / math.sqrt(D)
    qi = torch.arange(r0, r1, device=q.device)[:, None]
    ki = torch.arange(0, r1, device=q.device)[None, :]
    s = s.masked_fill(ki > qi, float("-inf"))
    o = torch.softmax(s, dim=-1) @ vf
    if with_lse:
        return o, torch.logsumexp(s.double(), dim=-1).float() * LOG2E
    return o


def sampled_heads(B, H, n=4, seed=0):
    rng = np.random.default_rng(seed)
    pairs = {(0, 0), (B - 1, H - 1)}
    while len(pairs) < min(n, B * H):
        pairs.add((int(rng.integers(B)), int(rng.integers(H))))
    return sorted(pairs)


def elementwise_ratio(out, ref, atol=2e-2, rtol=2e-2):
    out = out.float()
    if not torch.isfinite(out).all():
        return float("inf")
    return float(((out - ref).abs() / (atol + rtol * ref.abs())).max())


def reference_grads(q, k, v, do, b, g):
    """fp32 autograd of causal attention for batch b, K/V head g and its whole query-head group,
    on the device.  Returns (o, dq) for the group's query heads and (dk, dv) for head g."""
    H, H_kv = q.shape[1], k.shape[1]
    grp = H // H_kv
    hs = slice(g * grp, (g + 1) * grp)
    qf = q[b, hs].float().requires_grad_(True)
    kf = k[b, g].float().requires_grad_(True)
    vf = v[b, g].float().requires_grad_(True)
    N, D = q.shape[-2], q.shape[-1]
    s = (qf @ kf.T) / math.sqrt(D)
    mask = torch.ones(N, N, dtype=torch.bool, device=q.device).triu(1)
    o = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1) @ vf
    o.backward(do[b, hs].float())
    return o.detach(), qf.grad, kf.grad, vf.grad


def reference_backward_inputs(B, H, N, D, sigma, seed):
    """The reference's backward case inputs: a CUDA generator seeded N + D, q, k, v scaled by
    sigma then dO, all cast to fp16 (tests/backward/cases_backward.py:58-62 in the reference)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(B, H, N, D, device="cuda", generator=gen) * sigma for _ in range(3))
    do = torch.randn(B, H, N, D, device="cuda", generator=gen)
    return [t.half() for t in (q, k, v)], do.half()
