"""PyTorch fp32 causal GQA attention: the `reference` backend of run_attention_gqa.py.

Same definition as the reference project's `attention/gqa/reference_gqa.py:15-47`: K/V head
g serves query heads [g * group, (g + 1) * group), realised with repeat_interleave.
"""
import math

import torch
import torch.nn.functional as F


def _expand_kv(k32, v32, num_q_heads):
    h_kv = k32.shape[1]
    if v32.shape[1] != h_kv:
        raise ValueError(f"K/V head count mismatch: K={h_kv}, V={v32.shape[1]}")
    if h_kv < 1 or num_q_heads % h_kv != 0:
        raise ValueError(f"H={num_q_heads} not divisible by H_kv={h_kv}")
    group = num_q_heads // h_kv
    if group == 1:
        return k32, v32
    return k32.repeat_interleave(group, dim=1), v32.repeat_interleave(group, dim=1)


def reference_gqa_attention(q, k, v):
    q32, k32, v32 = q.float(), k.float(), v.float()
    k32, v32 = _expand_kv(k32, v32, q32.shape[1])
    return F.scaled_dot_product_attention(q32, k32, v32, is_causal=True)


def reference_gqa_attention_explicit(q, k, v):
    q32, k32, v32 = q.float(), k.float(), v.float()
    k32, v32 = _expand_kv(k32, v32, q32.shape[1])
    n, d = q32.shape[-2], q32.shape[-1]
    scores = (q32 @ k32.transpose(-1, -2)) / math.sqrt(d)
    future = torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1)
    probs = torch.softmax(scores.masked_fill(future, float("-inf")), dim=-1)
    return probs @ v32


causal_attention_reference_gqa = reference_gqa_attention_explicit
