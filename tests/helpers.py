"""Shared checks: the per-token parity metrics of the north star (max relative L2 error per output
token <= 2e-2, cosine similarity per token >= 0.999) and golden-fixture loading."""
import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOK_REL = 2e-2
TOK_COS = 0.999


def rel(a, b):
    """Relative L2 error ||a - b|| / ||b|| over the whole tensor (both moved to the CPU)."""
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def token_metrics(out, ref):
    """(max over tokens of ||out - ref|| / ||ref||, min over tokens of cos(out, ref)); last dim = features."""
    o = torch.as_tensor(out).double().reshape(-1, out.shape[-1])
    r = torch.as_tensor(ref).double().reshape(-1, ref.shape[-1])
    rel = (o - r).norm(dim=-1) / r.norm(dim=-1).clamp_min(1e-30)
    cos = torch.nn.functional.cosine_similarity(o, r, dim=-1)
    return float(rel.max()), float(cos.min())


def assert_tokens_close(out, ref, rel=TOK_REL, cos=TOK_COS, what=""):
    r, c = token_metrics(out, ref)
    assert r <= rel and c >= cos, f"{what}: max per-token rel {r:.3e} (<= {rel}), min cos {c:.6f} (>= {cos})"
    return r, c


def load_golden(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    out = {k: d[k] for k in d.files if k != "meta"}
    out["meta"] = json.loads(str(d["meta"]))
    return out


def token_probe(dim):
    """Same fixed directions as tests/golden/make_golden.py."""
    return np.random.default_rng(np.random.SeedSequence([9, dim])).standard_normal((dim, 8))


def golden_rel(out, g):
    """Compare a full output [T, D] against a golden fixture: (max rel over the stored rows,
    max over tokens of ||R^T (out - ref)|| / (sqrt(8) ||ref||), which estimates the per-token relative
    error since E ||R^T v||^2 = 8 ||v||^2 for the 8 N(0,1) probe directions R, and max per-token
    |sum(out) - sum(ref)| / ||ref||)."""
    out = np.asarray(torch.as_tensor(out).double().cpu())
    rows = g["rows"]
    rr = np.linalg.norm(out[rows] - g["out_rows"], axis=-1) / np.linalg.norm(g["out_rows"], axis=-1)
    proj = out @ token_probe(out.shape[-1])
    pr = np.linalg.norm(proj - g["tok_proj"], axis=-1) / (np.sqrt(8.0) * g["tok_norm"])
    sr = np.abs(out.sum(-1) - g["tok_sum"]) / g["tok_norm"]
    return float(rr.max()), float(pr.max()), float(sr.max())


def rglru_case():
    """The 12-head RG-LRU fixture (tests/golden/make_golden_ssm.py): the reference's ssm_ref with identity conv
    taps, i.e. the RG-LRU of x with block-diagonal gates.  Returns (W, frames) with W in oracle.tapnext_ref's
    dense-gate convention ([out, in] matrices, 768 x 768, block-diagonal) and frames = [(x, h), ...] in order."""
    g = np.load(os.path.join(GOLDEN, "rglru_ref_cases.npz"))

    def dense(w):  # [heads, 64 in, 64 out] (BlockDiagonalLinear) -> [768 out, 768 in]
        H, C, _ = w.shape
        d = np.zeros((H * C, H * C), np.float32)
        for q in range(H):
            d[q * C:(q + 1) * C, q * C:(q + 1) * C] = w[q].T
        return d

    W = {"gx_w": dense(g["wx"]), "gx_b": g["bx"].reshape(-1), "ga_w": dense(g["wa"]), "ga_b": g["ba"].reshape(-1),
         "a_param": g["a_param"].reshape(-1)}
    return W, [(g["first.x"], g["first.h"]), (g["next.x"], g["next.h"])]


RGLRU_TOL = 1e-2  # per row; ssm_ref rounds every intermediate to bf16, the restatement computes in fp32
