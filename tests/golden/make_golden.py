"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own PyTorch code.

    python tests/golden/make_golden.py [--reference /path/to/fused-attention]

Needs a checkout of the reference project (nvidiacutile/fused-attention); it is only run in the
build container, never on the GPU box.  What it calls, all from the reference checkout:
  tests/fused/cases.py        Case, make_inputs            (seeded fp16 inputs)
  tests/gqa/cases_gqa.py      Case, make_inputs
  attention/fused/reference.py        reference_attention_explicit   (fp32 ground truth)
  attention/gqa/reference_gqa.py      reference_gqa_attention_explicit
  tests/backward/run_correctness_backward.py reference + torch autograd (fp32 gradients)
The LSE fixture is logsumexp of the reference's masked, scaled scores times log2(e), the
quantity attention/backward/fused_backward.py:169 stores.

Each fixture keeps input checksums (to pin the seeded generator), and the outputs with every
`ROW_STRIDE`-th query row to keep the files small.
"""
import argparse
import importlib.util
import math
import os
import sys
import zlib

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROW_STRIDE = 4
LOG2E = 1.4426950408889634

MHA_CASES = ["B1_H1_N128_D64_tiny", "B1_H1_N128_D64_large", "B1_H1_N128_D128_large",
             "B1_H1_N512_D64_large", "B1_H1_N128_D32_tiny", "B2_H8_N128_D128_tiny"]
GQA_CASES = [(2, 128, 64, "large"), (1, 128, 128, "tiny"), (4, 128, 64, "large")]  # (H_kv, N, D, mag)
BWD_CASES = [(1, 2, 2, 128, 64, 1.0), (1, 2, 2, 128, 64, 7.0), (1, 4, 2, 128, 64, 1.0),
             (1, 1, 1, 256, 128, 3.0)]  # (B, H, H_kv, N, D, sigma)


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def checksums(*arrays):
    return np.array([[float(np.asarray(a, np.float64).sum()), float(np.abs(np.asarray(a, np.float64)).sum())]
                     for a in arrays])


def lse_from_reference_scores(q, k, group):
    q32, k32 = q.float(), k.float()
    if group > 1:
        k32 = k32.repeat_interleave(group, dim=1)
    n, d = q32.shape[-2], q32.shape[-1]
    s = (q32 @ k32.transpose(-1, -2)) / math.sqrt(d)
    s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
    return (torch.logsumexp(s.double(), dim=-1) * LOG2E).float()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FA_REFERENCE_ROOT"),
                    help="root of a checkout of the reference project (or set FA_REFERENCE_ROOT)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference PATH (a checkout of the reference project) or set FA_REFERENCE_ROOT")
    ref = a.reference
    sys.path.insert(0, ref)
    cases = _load(os.path.join(ref, "tests/fused/cases.py"), "ref_cases")
    cases_gqa = _load(os.path.join(ref, "tests/gqa/cases_gqa.py"), "ref_cases_gqa")
    reference = _load(os.path.join(ref, "attention/fused/reference.py"), "ref_reference")
    reference_gqa = _load(os.path.join(ref, "attention/gqa/reference_gqa.py"), "ref_reference_gqa")
    bwd_src = open(os.path.join(ref, "tests/backward/run_correctness_backward.py")).read()
    # The backward runner imports the cuTile kernel module at top level; take only its
    # `reference` function (fp32 autograd ground truth) by executing that definition.
    start = bwd_src.index("def reference(")
    end = bwd_src.index("\ndef rel_err(")
    ns = {"torch": torch, "math": math}
    exec(bwd_src[start:end], ns)
    bwd_reference = ns["reference"]
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    by_id = {c.id: c for c in cases.all_cases()}
    for cid in MHA_CASES:
        c = by_id[cid]
        q, k, v = cases.make_inputs(c)
        qt, kt, vt = (torch.from_numpy(x) for x in (q, k, v))
        o = reference.reference_attention_explicit(qt, kt, vt).numpy()
        lse = lse_from_reference_scores(qt, kt, 1).numpy()
        np.savez_compressed(os.path.join(HERE, f"mha_{cid}.npz"), case_id=cid, seed=c.seed,
                            input_checksums=checksums(q, k, v), q_head=q.reshape(-1)[:64],
                            o=o[:, :, ::ROW_STRIDE], lse=lse[:, :, ::ROW_STRIDE], row_stride=ROW_STRIDE)
        print("mha", cid, o.shape)

    by_id = {c.id: c for c in cases_gqa.all_cases()}
    for H_kv, N, D, mag in GQA_CASES:
        cid = f"B4_H8_Hkv{H_kv}_N{N}_D{D}_{mag}"
        c = by_id[cid]
        q, k, v = cases_gqa.make_inputs(c)
        qt, kt, vt = (torch.from_numpy(x) for x in (q, k, v))
        o = reference_gqa.reference_gqa_attention_explicit(qt, kt, vt).numpy()
        lse = lse_from_reference_scores(qt, kt, 8 // H_kv).numpy()
        np.savez_compressed(os.path.join(HERE, f"gqa_{cid}.npz"), case_id=cid, seed=c.seed,
                            input_checksums=checksums(q, k, v), q_head=q.reshape(-1)[:64],
                            o=o[:, :, ::ROW_STRIDE], lse=lse[:, :, ::ROW_STRIDE], row_stride=ROW_STRIDE)
        print("gqa", cid, o.shape)

    for B, H, H_kv, N, D, sigma in BWD_CASES:
        cid = f"bwd_B{B}_H{H}_Hkv{H_kv}_N{N}_D{D}_s{sigma:g}"
        rng = np.random.default_rng(zlib.crc32(cid.encode()))
        q = (rng.standard_normal((B, H, N, D), dtype=np.float32) * sigma).astype(np.float16)
        k = (rng.standard_normal((B, H_kv, N, D), dtype=np.float32) * sigma).astype(np.float16)
        v = (rng.standard_normal((B, H_kv, N, D), dtype=np.float32) * sigma).astype(np.float16)
        do = rng.standard_normal((B, H, N, D), dtype=np.float32).astype(np.float16)
        # fp32 leaves holding the fp16 values: the reference upcasts inside, and fp32 leaves keep
        # the gradients unrounded (fp16 leaves would round them to fp16).
        qt, kt, vt = (torch.from_numpy(x.astype(np.float32)).requires_grad_(True) for x in (q, k, v))
        if H_kv == H:
            o = bwd_reference(qt, kt, vt)
        else:
            o = reference_gqa.reference_gqa_attention_explicit(qt, kt, vt)
        o.backward(torch.from_numpy(do).float())
        grads = [t.grad.float().numpy() for t in (qt, kt, vt)]
        np.savez_compressed(os.path.join(HERE, f"{cid}.npz"), case_id=cid, shape=np.array([B, H, H_kv, N, D]),
                            sigma=sigma, input_checksums=checksums(q, k, v, do), q=q, k=k, v=v, do=do,
                            o=o.detach().numpy(), dq=grads[0], dk=grads[1], dv=grads[2])
        print("bwd", cid)


if __name__ == "__main__":
    main()
