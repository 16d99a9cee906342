"""CPU fp32 restatement of the moondream2 text decoder that consumes the vision tower's features --
TEST INFRASTRUCTURE (only tests/ and bench.py import it).

Follows FastMD2's unfused torch path (moondream/gpu/md2fast.py):
  * rope(), md2fast.py:162-167: rotary on the first 32 dims of each 64-dim head, input halves (a | b),
    output interleaved pairs (a cos - b sin, a sin + b cos);
  * text_layers(), md2fast.py:169-199 (the `else` branch, fuse off): h = LN(x); qkv; rope on q and k; k, v
    written to the cache at positions pos0 .. pos0 + n; attention (no mask: over the n new keys; with the
    query mask: over the cache up to pos0 + n); x = fc2(gelu_tanh(fc1(h))) + (proj(a) + x) (the parallel
    block of md2fast.py:199 with mlp / lin_res, md2fast.py:54-67);
  * encode(), md2fast.py:201-206 from given image embeddings: x = [wte[bos]; emb], all 730 positions;
  * query(), md2fast.py:208-212: the question's tokens at positions 730 .. 761 with the causal query mask
    (md2fast.py:132-136), LN of the last real token, the yes / no rows of the lm head.
With i8 (quantize_weights()), the four linears of each layer follow the reference's int8 W8A8 layer instead
(FastMD2 with tlin_cls=HI8Lin, md2fast.py:88, 112-113; numerics in oracle/i8_ref.py): activation rows quantised
per token, exact int32 products, fp32 epilogue with GELU fused into fc1, bf16 outputs.
The rotary angles are pos * theta^(-2i / 32), i < 16, theta 10000 (the reference reads them from the HF
model's freqs_cis, which is not in the repository: restated).  Pinned by tests/golden/make_golden_text.py,
which runs the reference's own _text_layers / _query on the same weights and cos / sin.
"""
import numpy as np
import torch
import torch.nn.functional as F

from . import i8_ref
from .tower_ref import _t, layer_norm, linear


def gelu_tanh(x):
    return F.gelu(x, approximate="tanh")


def rope_angles(cfg, pos0, n):
    """cos, sin [n, rot / 2] for positions pos0 .. pos0 + n - 1."""
    inv = cfg.theta ** (-torch.arange(0, cfg.rot, 2, dtype=torch.float64) / cfg.rot)
    ang = torch.arange(pos0, pos0 + n, dtype=torch.float64)[:, None] * inv[None]
    return torch.cos(ang).float(), torch.sin(ang).float()


def rope(x, cos, sin, rot):
    """md2fast.py:162-167 on x [B, H, n, hd]."""
    xr, xp = x[..., :rot], x[..., rot:]
    a, b = xr[..., :rot // 2], xr[..., rot // 2:]
    cos, sin = cos[None, None], sin[None, None]
    o = torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2)
    return torch.cat([o, xp], dim=-1)


def query_mask(cfg):
    """md2fast.py:132-136: question position i sees the whole prefix and question positions <= i."""
    m = torch.zeros(cfg.q_len, cfg.ctx, dtype=torch.bool)
    m[:, :cfg.prefix] = True
    m[:, cfg.prefix:] = torch.tril(torch.ones(cfg.q_len, cfg.q_len, dtype=torch.bool))
    return m[None, None]


def quantize_weights(W, n_layers):
    """HI8Lin's weight quantisation (hgemm.py:100-103) of every text linear: {"tblocks.i.name": (wq, sw)}."""
    return {f"tblocks.{i}.{n}": i8_ref.quant_w(W[f"tblocks.{i}.{n}_w"])
            for i in range(n_layers) for n in ("qkv", "proj", "fc1", "fc2")}


def _lin(h, W, name, i8, gelu=False):
    """One text linear: fp32 (Lin) or, with i8, HI8Lin's int8 path (hgemm.py:126-137, GELU fused as
    md2fast.py:56 uses it)."""
    if i8 is None:
        y = linear(h, W[name + "_w"], W[name + "_b"])
        return gelu_tanh(y) if gelu else y
    wq, sw = i8[name]
    x2 = i8_ref.bf16_round(h.reshape(-1, h.shape[-1]).numpy())  # the layer's bf16 activations
    y = i8_ref.i8_linear(x2, wq, sw, np.asarray(W[name + "_b"], np.float32), gelu)
    return torch.from_numpy(y).reshape(*h.shape[:-1], -1)


def text_layers(x, W, cfg, pos0, cos, sin, mask, kc, vc, n_layers, i8=None):
    """md2fast.py:169-199 (unfused); x [1, n, D]; kc / vc lists of [1, H, ctx, hd] caches, updated."""
    H, hd = cfg.heads, cfg.head_dim
    n = x.shape[1]
    for i in range(n_layers):
        p = f"tblocks.{i}."
        h = layer_norm(x, W[p + "ln_w"], W[p + "ln_b"], cfg.eps)
        q, k, v = _lin(h, W, p + "qkv", i8).split([H * hd] * 3, dim=-1)
        q = rope(q.view(1, n, H, hd).transpose(1, 2), cos, sin, cfg.rot)
        k = rope(k.view(1, n, H, hd).transpose(1, 2), cos, sin, cfg.rot)
        v = v.view(1, n, H, hd).transpose(1, 2)
        kc[i][:, :, pos0:pos0 + n] = k
        vc[i][:, :, pos0:pos0 + n] = v
        if mask is None:
            a = F.scaled_dot_product_attention(q, k, v)
        else:
            a = F.scaled_dot_product_attention(q, kc[i][:, :, :pos0 + n], vc[i][:, :, :pos0 + n], attn_mask=mask)
        a = a.transpose(1, 2).reshape(1, n, H * hd)
        res = _lin(a, W, p + "proj", i8) + x
        x = _lin(_lin(h, W, p + "fc1", i8, gelu=True), W, p + "fc2", i8) + res
    return x


def encode(emb, bos, W, cfg, n_layers=None, i8=None):
    """md2fast.py:201-206: returns (prefix hidden states [730, D], kv caches)."""
    nl = cfg.n_layers if n_layers is None else n_layers
    with torch.no_grad():
        wte = _t(W["wte"])
        x = torch.cat([wte[bos][None], _t(emb)], dim=0)[None]
        kc = [torch.zeros(1, cfg.heads, cfg.ctx, cfg.head_dim) for _ in range(nl)]
        vc = [torch.zeros(1, cfg.heads, cfg.ctx, cfg.head_dim) for _ in range(nl)]
        cos, sin = rope_angles(cfg, 0, cfg.prefix)
        x = text_layers(x, W, cfg, 0, cos, sin, None, kc, vc, nl, i8)
        return x[0], (kc, vc)


def query(ids, last, W, cfg, cache, n_layers=None, i8=None):
    """md2fast.py:208-212: yes / no logits [n_yn] of the question ids [q_len] read at position `last`."""
    nl = cfg.n_layers if n_layers is None else n_layers
    kc, vc = cache
    with torch.no_grad():
        x = _t(W["wte"])[torch.as_tensor(ids)][None]
        cos, sin = rope_angles(cfg, cfg.prefix, cfg.q_len)
        x = text_layers(x, W, cfg, cfg.prefix, cos, sin, query_mask(cfg), kc, vc, nl, i8)
        h = layer_norm(x[0, last][None], W["tpost_ln_w"], W["tpost_ln_b"], cfg.eps)
        return linear(h, W["lm_small_w"], W["lm_small_b"])[0]
