"""Shared helpers of the test-suite: seeded inputs, golden fixtures, per-head oracle."""
from __future__ import annotations

import glob
import math
import os

import numpy as np
import torch

from oracle.attention_oracle import attention_bwd, attention_fwd

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances of the path (max-abs against the fp32/fp64 oracle)
TOL_O = 2e-3
TOL_LSE = 2e-3
TOL_GRAD = 5e-3


def make_inputs(B, S, H, D, amp=1.0, seed=0, n=4):
    """q, k, v, dO (in that order) ~ N(0,1)*amp from a seeded CPU generator, fp16."""
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn((B, S, H, D), generator=g) * amp).to(torch.float16) for _ in range(n)]


def golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(path):
    z = np.load(path)
    out = {k: z[k] for k in z.files}
    for k in ("q", "k", "v", "do", "o_ref", "dq_ref", "dk_ref", "dv_ref"):
        out[k] = torch.from_numpy(out[k])
    out["lse_ref"] = torch.from_numpy(out["lse_ref"])
    out["o_eager"] = torch.from_numpy(out["o_eager"])
    out["causal"] = bool(out["causal"])
    out["scale"] = float(out["scale"])
    return out


def oracle_heads(q, k, v, do, causal, scale, heads=None, grads=True):
    """Exact oracle evaluated one (b, h) at a time (bounded memory).

    Returns dict of CPU tensors restricted to `heads` (list of (b, h)), each
    stacked along a new leading axis: o (n,S,D), lse (n,S), dq/dk/dv (n,S,D).
    """
    B, S, H, D = q.shape
    if heads is None:
        heads = [(b, h) for b in range(B) for h in range(H)]
    res = {"o": [], "lse": [], "dq": [], "dk": [], "dv": []}
    for b, h in heads:
        sl = lambda t: t[b:b + 1, :, h:h + 1, :]
        o, lse = attention_fwd(sl(q), sl(k), sl(v), causal, scale, dtype=torch.float64)
        res["o"].append(o[0, :, 0])
        res["lse"].append(lse[0, 0])
        if grads:
            dq, dk, dv = attention_bwd(sl(do), sl(q), sl(k), sl(v), causal, scale)
            res["dq"].append(dq[0, :, 0])
            res["dk"].append(dk[0, :, 0])
            res["dv"].append(dv[0, :, 0])
    return {k: torch.stack(v_) for k, v_ in res.items() if v_}


def pick_heads(t, heads):
    """(B,S,H,D) tensor -> (n,S,D) for the listed (b, h); (B,H,S) -> (n,S)."""
    if t.dim() == 4:
        return torch.stack([t[b, :, h] for b, h in heads])
    return torch.stack([t[b, h] for b, h in heads])


def maxdiff(a, b):
    return float((a.double() - b.double()).abs().max())
