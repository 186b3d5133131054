"""PyTorch fp32 causal attention: the `reference` backend of run_attention.py.

Same definition as the reference project's `attention/fused/reference.py:16-27` (upcast to
fp32, explicit scores / softmax / PV with the strictly-upper triangle masked).  It is a
user-selected backend of the CLI, not a fallback of the fused path.
"""
import math

import torch
import torch.nn.functional as F


def reference_attention(q, k, v):
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)


def reference_attention_explicit(q, k, v):
    q32, k32, v32 = q.float(), k.float(), v.float()
    n, d = q32.shape[-2], q32.shape[-1]
    scores = (q32 @ k32.transpose(-1, -2)) / math.sqrt(d)
    future = torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1)
    probs = torch.softmax(scores.masked_fill(future, float("-inf")), dim=-1)
    return probs @ v32


causal_attention_reference = reference_attention_explicit
