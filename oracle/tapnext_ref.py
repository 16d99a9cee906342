"""CPU fp32 restatement of the TAPNext-style per-frame step -- TEST INFRASTRUCTURE; RG-LRU pinned, the
composition unpinned.

Token layout: 8x8 patch conv of a 256x256 frame (1024 tokens) + image position embedding, then the
256 point-query tokens (tapnext/npu/step8.py:251-267).  Each of the 12 blocks is a pre-LN ViT block
(LN -> MHA -> +, LN -> MLP GELU -> +, the vit_block part of step8.py:482-485) followed by a residual
temporal block in the reference's shape (step8.py:474-480: pre-norm, recurrence, + x): t = RMSNorm(x)
(gamma folded, eps 1e-6), then the per-token RG-LRU of tapnext/npu/r9/cpuemu.py:33-47 on t with exact
transcendentals:
    gx = sigmoid(Wx t + bx), ga = sigmoid(Wa t + ba), log_a = -c * ga * softplus(a_param), a = exp(log_a)
    h = t * gx                                  (first frame, h0 is None)
    h = a * h0 + (t * gx) * sqrt(1 - a^2)        (later frames)
    x <- x + h, state <- h (float32)
then the encoder LayerNorm (step8.py:488).

Pinning: rglru() is checked against the reference's own ssm_ref (tapnext/npu/pack8.py:252-279) run with
12 heads of block-diagonal gates and identity conv taps, where ssm_ref's h is exactly this RG-LRU
(tests/golden/make_golden_ssm.py -> rglru_ref_cases.npz, tests/test_oracle_golden.py, within 1e-2 per row:
ssm_ref rounds its intermediates to bf16).  The ViT block is built from tower_ref's operations, which are
pinned to FastMD2._vision.  The composition (a ViT block then the temporal block, dense gates, no conv1d /
gated MLP) is the BASELINE config's simplification of the reference block; with the vendored model not in
the repository, nothing pins the composed step against the reference's outputs.
"""
import torch
import torch.nn.functional as F

from .tower_ref import _t, im2col, layer_norm, gelu, linear


def rglru(x, W, p, h0, c):
    """cpuemu.py:33-47 with exact sigmoid / exp / sqrt, in float32."""
    gx = torch.sigmoid(linear(x, W[p + "gx_w"], W[p + "gx_b"]))
    ga = torch.sigmoid(linear(x, W[p + "ga_w"], W[p + "ga_b"]))
    log_a = -c * ga * F.softplus(_t(W[p + "a_param"]))
    gated = x * gx
    if h0 is None:
        return gated
    a = torch.exp(log_a)
    return a * h0 + gated * torch.sqrt(-torch.expm1(2.0 * log_a))


def rms_norm(x, w, eps):
    """x * rsqrt(mean(x^2) + eps) * w (the temporal pre-norm, step8.py:474)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * _t(w)


def step(frame, queries, W, cfg, state=None, n_blocks=None):
    """frame [3, 256, 256] in [-1, 1], queries [256, 768] -> (features [1280, 768], new state list)."""
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    with torch.no_grad():
        x = linear(im2col(_t(frame).float()[None], cfg.patch)[0], W["patch_w"], W["patch_b"]) + _t(W["pos_emb"])
        x = torch.cat([x, _t(queries).float()], dim=0)[None]
        T = x.shape[1]
        new_state = []
        for i in range(nb):
            p = f"blocks.{i}."
            h = layer_norm(x, W[p + "ln1_w"], W[p + "ln1_b"], cfg.eps)
            q, k, v = [t.view(1, T, cfg.heads, -1).transpose(1, 2) for t in linear(h, W[p + "qkv_w"], W[p + "qkv_b"]).chunk(3, dim=-1)]
            a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(1, T, -1)
            x = x + linear(a, W[p + "proj_w"], W[p + "proj_b"])
            h = layer_norm(x, W[p + "ln2_w"], W[p + "ln2_b"], cfg.eps)
            x = x + linear(gelu(linear(h, W[p + "fc1_w"], W[p + "fc1_b"])), W[p + "fc2_w"], W[p + "fc2_b"])
            t = rms_norm(x, W[p + "rms_w"], cfg.eps)
            hs = rglru(t, W, p, None if state is None else state[i], cfg.lru_c)
            new_state.append(hs)
            x = x + hs
        out = layer_norm(x, W["final_ln_w"], W["final_ln_b"], cfg.eps)[0]
        return out, new_state
