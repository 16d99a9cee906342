"""CPU restatement of the full TAPNext++ block step -- TEST INFRASTRUCTURE (only tests/ and bench.py import it).

Op order of one block (tapnext/npu/step8.py:469-486, the reference's own CPU check of block 0):
    t0 = RMSNorm(x)                                  temporal_pre_norm, x * rsqrt(mean x^2 + eps) * (1 + scale)
    y, xx = linear_yx(t0).chunk(2)                   768 -> 1536
    yg = gelu_tanh(y)
    xc = conv_1d(xx)                                 4 taps over frames, oldest .. current, + bias
    h  = rg_lru(xc)                                  block-diagonal gates (12 heads x 64 x 64)
    res = linear_out(h * yg) + x
    x1 = ffw_down(gelu_tanh(gate) * up) + res        gate, up = ffw_up(RMSNorm(res)) halves (3072 each)
    x2 = x1 + MHA(LN_1(x1))                          12 heads x 64
    x3 = x2 + mlp_3(gelu_erf(mlp_0(LN_2(x2))))       the ViT MLP uses the exact GELU
and the encoder LayerNorm after the last block.  Weight names and shapes follow the reference's state-dict
keys (step8.py:161-183, 205-215); the RMSNorm "scale + 1" convention is pack8.py:108-121 (norm_params);
the gated MLP's [gate | up] split of ffw_up is pack8.py:96-101 (interleave_gated) and its GELU is the tanh
form applied to the bf16 gate (tapnext/npu/mm8.cc:6, 937-960).

Two arithmetic levels:
  * step(): exact float32 math (the parity reference for the bf16 GPU path, per-token tolerance);
  * ssm_bf16(): the recurrent block's element-wise part with the reference's bf16 rounding points, restated
    from pack8.py:249-279 (ssm_ref) and pinned against fixtures that ssm_ref itself produced
    (tests/golden/make_golden_ssm.py).

The vendored TAPNext model (model.py) is not in the repository, so the block as a whole is parity
unpinned: only its recurrent element-wise part is pinned, by ssm_ref.  heads() restates the host tracking
heads (step8.py:327-362, heads_np) and is pinned to fixtures heads_np itself produced
(tests/golden/make_golden_heads.py).
"""
import math

import torch
import torch.nn.functional as F

from .tower_ref import _t, im2col, layer_norm, linear

HEADS, HD = 12, 64


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def gelu_erf(x):
    return 0.5 * x * (1.0 + torch.erf(x / math.sqrt(2.0)))


def rms_norm1(x, scale, eps):
    """Griffin-style RMSNorm: x * rsqrt(mean(x^2) + eps) * (1 + scale) (pack8.py:118)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + _t(scale))


def conv4(xx, hist, w, b):
    """xc = sum_i w[i] * x_(t-3+i) + b, taps oldest .. current; hist = [x_(t-3), x_(t-2), x_(t-1)]."""
    taps = list(hist) + [xx]
    return sum(_t(w)[i] * taps[i] for i in range(4)) + _t(b)


def block_diag(xc, w, b):
    """Per head q: xc[:, q*64:(q+1)*64] @ w[q] (+ b), w [12, 64 in, 64 out] (BlockDiagonalLinear)."""
    R = xc.shape[0]
    return torch.einsum("rqi,qio->rqo", xc.view(R, HEADS, HD), _t(w)).reshape(R, -1) + _t(b).reshape(-1)


def rg_lru(xc, W, p, h0):
    """step8.py:479 / r9/cpuemu.py:33-47 with the block-diagonal gates, exact transcendentals."""
    gx = torch.sigmoid(block_diag(xc, W[p + "gx_w"], W[p + "gx_b"]))
    ga = torch.sigmoid(block_diag(xc, W[p + "ga_w"], W[p + "ga_b"]))
    log_a = -8.0 * ga * F.softplus(_t(W[p + "a_param"]))
    gated = xc * gx
    if h0 is None:
        return gated
    return torch.exp(log_a) * h0 + gated * torch.sqrt(-torch.expm1(2.0 * log_a))


def step(frame, queries, W, cfg, state=None, n_blocks=None):
    """frame [3, 256, 256] in [-1, 1], queries [Q, 768] -> (features [1024 + Q, 768], new state).
    state = None (first frame) or the previous call's: per block (h [T, 768], conv history [x_(t-3), x_(t-2),
    x_(t-1)]); the first frame has zero history and no h0 (step8.py:478-479 with caches None)."""
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    with torch.no_grad():
        x = linear(im2col(_t(frame).float()[None], cfg.patch)[0], W["patch_w"], W["patch_b"]) + _t(W["pos_emb"])
        x = torch.cat([x, _t(queries).float()], dim=0)
        T, Wd = x.shape
        new_state = []
        for i in range(nb):
            p = f"blocks.{i}."
            h0, hist = (None, [torch.zeros(T, Wd)] * 3) if state is None else state[i]
            t0 = rms_norm1(x, W[p + "rms0_scale"], cfg.eps)
            y, xx = linear(t0, W[p + "yx_w"], W[p + "yx_b"]).chunk(2, dim=-1)
            xc = conv4(xx, hist, W[p + "conv_w"], W[p + "conv_b"])
            h = rg_lru(xc, W, p, h0)
            res = linear(h * gelu_tanh(y), W[p + "out_w"], W[p + "out_b"]) + x
            gate, up = linear(rms_norm1(res, W[p + "rms1_scale"], cfg.eps), W[p + "up_w"], W[p + "up_b"]).chunk(2, dim=-1)
            x = linear(gelu_tanh(gate) * up, W[p + "down_w"], W[p + "down_b"]) + res
            new_state.append((h, [hist[1], hist[2], xx]))
            a_in = layer_norm(x[None], W[p + "ln1_w"], W[p + "ln1_b"], cfg.eps)
            q, k, v = [u.view(1, T, cfg.heads, -1).transpose(1, 2)
                       for u in linear(a_in, W[p + "qkv_w"], W[p + "qkv_b"]).chunk(3, dim=-1)]
            a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(1, T, -1)
            x = x + linear(a, W[p + "proj_w"], W[p + "proj_b"])[0]
            m = gelu_erf(linear(layer_norm(x[None], W[p + "ln2_w"], W[p + "ln2_b"], cfg.eps), W[p + "fc1_w"], W[p + "fc1_b"]))
            x = x + linear(m, W[p + "fc2_w"], W[p + "fc2_b"])[0]
        out = layer_norm(x[None], W["final_ln_w"], W["final_ln_b"], cfg.eps)[0]
        return out, new_state


def _bf(v):
    """Round to bf16 and back (the reference's f(), pack8.py:254)."""
    return torch.as_tensor(v, dtype=torch.float32).to(torch.bfloat16).float()


def ssm_bf16(y, x, xm1, xm2, xm3, h0, conv_w, conv_b, a_param, wx, bx, wa, ba, first):
    """pack8.py:252-279 (ssm_ref) for one head restated in torch with the same rounding points: inputs
    [R, 64] (bf16 values), h0 fp32, conv_w [4, 64] oldest .. current, wx / wa [64 in, 64 out].
    Returns (z bf16 values as float32, h float32)."""
    f, F32 = _bf, (lambda v: torch.as_tensor(v, dtype=torch.float32))
    taps = [xm3, xm2, xm1, x]
    s = torch.zeros_like(F32(x))
    for i, tp in enumerate(taps):
        s = s + f(F32(tp) * f(conv_w[i])[None])
    xc = f(f(s) + f(conv_b)[None])
    gx_pre = f(f((xc.double() @ torch.as_tensor(wx, dtype=torch.float64)).float()) + f(bx)[None])
    ga_pre = f(f((xc.double() @ torch.as_tensor(wa, dtype=torch.float64)).float()) + f(ba)[None])
    gate_x = f(torch.sigmoid(gx_pre.double()).float())
    gate_a = f(torch.sigmoid(ga_pre.double()).float())
    sp = f(F.softplus(torch.as_tensor(a_param, dtype=torch.float64)).float())
    log_a = f(f(-8.0 * gate_a) * sp[None])
    a = f(torch.exp(log_a.double()).float())
    gated = f(xc * gate_x)
    if first:
        h = gated.clone()
        hb = gated
    else:
        e2 = f(torch.exp(f(2.0 * log_a).double()).float())
        mult = f(torch.sqrt(f(1.0 - e2)))
        nx = f(gated * mult)
        h = a * F32(h0) + nx
        hb = f(h)
    z = f(hb * F32(y))
    return z, h


def head_mlp(x, HW, name, eps):
    """One tracking head (step8.py:341-348): (Linear, LayerNorm, erf GELU) twice, then the output Linear; fp32."""
    for i, j in ((0, 1), (3, 4)):
        h = linear(x, HW[f"{name}.{i}_w"], HW[f"{name}.{i}_b"])
        mu = h.mean(-1, keepdim=True)
        var = ((h - mu) ** 2).mean(-1, keepdim=True)
        h = (h - mu) / torch.sqrt(var + eps) * _t(HW[f"{name}.{j}_w"]) + _t(HW[f"{name}.{j}_b"])
        x = 0.5 * h * (1.0 + torch.erf(h * 0.7071067811865476))
    return linear(x, HW[f"{name}.6_w"], HW[f"{name}.6_b"])


def heads(x, HW, cfg):
    """The TAPNext++ tracking heads on the query tokens x [Q, width] (step8.py:327-362): coordinate logits
    [Q, 2 * bins] (y bins | x bins); per axis the softmax of logits * temperature, restricted to a window of
    +-track_window bins around the argmax (the first maximum), renormalised, and its expectation over the bin
    indices + 0.5 -> tracks [Q, 2] (y, x); the visibility logit [Q].  fp32 throughout."""
    with torch.no_grad():
        x = _t(x).float()
        logits = head_mlp(x, HW, "coord", cfg.head_eps)
        n = logits.shape[-1] // 2
        idx = torch.arange(n, dtype=torch.float32)
        out = []
        for h in (logits[:, :n], logits[:, n:]):
            am = h.argmax(-1, keepdim=True).float()
            mask = (am - idx).abs() <= cfg.track_window
            z = h * cfg.track_temperature
            e = torch.exp(z - z.max(-1, keepdim=True).values)
            pr = e / e.sum(-1, keepdim=True) * mask
            pr = pr / pr.sum(-1, keepdim=True)
            out.append((pr * idx).sum(-1))
        tracks = torch.stack(out, -1) + 0.5
        vis = head_mlp(x, HW, "vis", cfg.head_eps)[:, 0]
        return tracks, logits, vis
