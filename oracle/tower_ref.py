"""CPU fp32 restatement of FastMD2._vision (moondream/gpu/md2fast.py:147-160) -- TEST INFRASTRUCTURE.

Each function names the reference lines it follows.  Weights come as the dict produced by
strix_halo_maxx_b200.weights.tower_weights (float32 numpy or torch).  Pinned: tests/golden holds
outputs of the reference's own FastMD2._vision on the same seeded weights
(tests/golden/make_golden.py), and tests/test_oracle_golden.py checks this file against them.
"""
import torch
import torch.nn.functional as F


def _t(a):
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(a)


def normalize_u8(img_u8):
    """uint8 HWC [.., 378, 378, 3] -> float NCHW [-1, 1]: md2fast.py:148 `(x/255 - 0.5)/0.5`."""
    x = _t(img_u8)
    if x.dim() == 3:
        x = x[None]
    return x.permute(0, 3, 1, 2).float().div(255.0).sub(0.5).div(0.5)


def im2col(pix, patch=14):
    """[B, C, S, S] -> [B, (S/p)^2, C*p*p], K order (c, py, px): md2fast.py:149."""
    B, C, S, _ = pix.shape
    g = S // patch
    return pix.reshape(B, C, g, patch, g, patch).permute(0, 2, 4, 1, 3, 5).reshape(B, g * g, C * patch * patch)


def layer_norm(x, w, b, eps):
    """md2fast.py:43-44 (_ln), with the eps passed explicitly (the reference uses torch's 1e-5)."""
    return F.layer_norm(x, (x.shape[-1],), _t(w), _t(b), eps)


def gelu(x):
    """md2fast.py:47-48: GELU, tanh approximation."""
    return F.gelu(x, approximate="tanh")


def linear(x, w, b):
    """md2fast.py:39-40 (Lin.__call__)."""
    return F.linear(x, _t(w), _t(b))


def block(x, W, i, heads, eps):
    """One pre-LN encoder block, md2fast.py:153-157: x [B, T, width] float32."""
    p = f"blocks.{i}."
    B, T, C = x.shape
    h = layer_norm(x, W[p + "ln1_w"], W[p + "ln1_b"], eps)
    q, k, v = [t.view(B, T, heads, -1).transpose(1, 2) for t in linear(h, W[p + "qkv_w"], W[p + "qkv_b"]).chunk(3, dim=-1)]
    a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, T, C)
    x = linear(a, W[p + "proj_w"], W[p + "proj_b"]) + x                       # lin_res, md2fast.py:64-67
    h = layer_norm(x, W[p + "ln2_w"], W[p + "ln2_b"], eps)
    return linear(gelu(linear(h, W[p + "fc1_w"], W[p + "fc1_b"])), W[p + "fc2_w"], W[p + "fc2_b"]) + x   # mlp, md2fast.py:55-61


def tower(pix, W, cfg, eps=None, n_blocks=None):
    """Pixels [B, 3, 378, 378] in [-1, 1] -> post-LN features [B, 729, width]: md2fast.py:149-158."""
    eps = cfg.eps if eps is None else eps
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    with torch.no_grad():
        x = linear(im2col(_t(pix).float(), cfg.patch), W["patch_w"], W["patch_b"]) + _t(W["pos_emb"])[None]
        for i in range(nb):
            x = block(x, W, i, cfg.heads, eps)
        return layer_norm(x, W["post_ln_w"], W["post_ln_b"], eps)


def projection(feats, W):
    """Projection MLP over [.., 2*width] -> [.., proj_out]: md2fast.py:159-160 (mlp, md2fast.py:55-61)."""
    with torch.no_grad():
        return linear(gelu(linear(feats, W["proj_fc1_w"], W["proj_fc1_b"])), W["proj_fc2_w"], W["proj_fc2_b"])


def vision_u8(img_u8, W, cfg, eps=1e-5, n_blocks=None, fold_proj=False):
    """The whole of FastMD2._vision for one uint8 crop -> [729, proj_out] (md2fast.py:147-160).  fold_proj:
    proj_fc1's two K-halves summed in fp32 (md2fast.py:97-101) and applied to x instead of cat([x, x])."""
    x = tower(normalize_u8(img_u8), W, cfg, eps, n_blocks)[0]
    if fold_proj:
        return projection(x, fold_projection(W, cfg))
    return projection(torch.cat([x, x], dim=-1), W)


def fold_projection(W, cfg):
    """W with proj_fc1_w [hidden, 2 width] replaced by the sum of its K-halves [hidden, width] (md2fast.py:99)."""
    w1 = _t(W["proj_fc1_w"]).float()
    return dict(W, proj_fc1_w=w1[:, :cfg.width] + w1[:, cfg.width:])


def combine_crops(feats):
    """Multi-crop frame: crop 0 is the global crop, crops 1.. are local; the local features are
    averaged per token and concatenated after the global ones -> [T, 2*width] (
    the stock HF stitching is not vendored in the reference)."""
    return torch.cat([feats[0], feats[1:].mean(dim=0)], dim=-1)


def frame(crops, W, cfg, eps=None, n_blocks=None):
    """13 crops [13, 3, 378, 378] -> projected frame features [729, proj_out] (config 2)."""
    f = tower(crops, W, cfg, eps, n_blocks)
    return projection(combine_crops(f), W)
