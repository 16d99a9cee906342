"""Seeded random-init weights for the two encoders (no checkpoints are available offline).

Every tensor is drawn from its own numpy PCG64 stream, keyed by (seed, tensor index), so the draw
is identical on any machine and independent of generation order; weights are N(0, 0.02), biases
zero and LayerNorm gamma = 1, beta = 0 (the BASELINE configs).  `affine="random"` instead draws
biases N(0, 0.02), gamma 1 + N(0, 0.1) and beta N(0, 0.05) so tests exercise every epilogue term.

Names follow the reference's weight set: moondream/gpu/md2fast.py:89-103 (patch_emb, pos_emb,
vblocks[i].{ln1,qkv,proj,ln2,fc1,fc2}, post_ln, proj_fc1, proj_fc2).
"""
from concurrent.futures import ThreadPoolExecutor
import numpy as np

from .config import TowerConfig, TapNextConfig


def _draw(seed, idx, shape, kind, affine):
    rng = np.random.default_rng(np.random.SeedSequence([int(seed), int(idx)]))
    if kind == "w":
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    if kind == "normal1":
        return rng.standard_normal(shape, dtype=np.float32)
    if kind == "wout":  # last layer of a tracking head: wider, so the soft-argmax sees peaked logits
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.25)
    if kind == "conv":  # temporal conv taps
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.5)
    if kind == "scale":  # RMSNorm scale of the (1 + scale) convention
        if affine != "random":
            return np.zeros(shape, np.float32)
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
    if affine != "random":
        return np.ones(shape, np.float32) if kind == "gamma" else np.zeros(shape, np.float32)
    if kind == "gamma":
        return np.float32(1.0) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
    if kind == "beta":
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.05)
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)   # bias


def _generate(spec, seed, affine, threads=8):
    with ThreadPoolExecutor(threads) as ex:
        arrs = list(ex.map(lambda it: _draw(seed, it[0], it[1][1], it[1][2], affine), enumerate(spec)))
    return {name: a for (name, _, _), a in zip(spec, arrs)}


def tower_spec(cfg: TowerConfig, n_blocks=None, projection=True):
    W, F = cfg.width, cfg.ff
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    s = [("patch_w", (W, cfg.patch_k), "w"), ("patch_b", (W,), "bias"), ("pos_emb", (cfg.ntok, W), "w")]
    for i in range(nb):
        p = f"blocks.{i}."
        s += [(p + "ln1_w", (W,), "gamma"), (p + "ln1_b", (W,), "beta"),
              (p + "qkv_w", (cfg.qkv_dim, W), "w"), (p + "qkv_b", (cfg.qkv_dim,), "bias"),
              (p + "proj_w", (W, W), "w"), (p + "proj_b", (W,), "bias"),
              (p + "ln2_w", (W,), "gamma"), (p + "ln2_b", (W,), "beta"),
              (p + "fc1_w", (F, W), "w"), (p + "fc1_b", (F,), "bias"),
              (p + "fc2_w", (W, F), "w"), (p + "fc2_b", (W,), "bias")]
    s += [("post_ln_w", (W,), "gamma"), ("post_ln_b", (W,), "beta")]
    if projection:
        s += [("proj_fc1_w", (cfg.proj_hidden, 2 * W), "w"), ("proj_fc1_b", (cfg.proj_hidden,), "bias"),
              ("proj_fc2_w", (cfg.proj_out, cfg.proj_hidden), "w"), ("proj_fc2_b", (cfg.proj_out,), "bias")]
    return s


def tower_weights(cfg: TowerConfig, seed=0, n_blocks=None, projection=True, affine="zero"):
    """dict name -> float32 numpy array (see module docstring for the distribution)."""
    return _generate(tower_spec(cfg, n_blocks, projection), seed, affine)


def tapnext_spec(cfg: TapNextConfig, n_blocks=None):
    W, F = cfg.width, cfg.ff
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    s = [("patch_w", (W, cfg.patch_k), "w"), ("patch_b", (W,), "bias"), ("pos_emb", (cfg.n_img_tok, W), "w")]
    for i in range(nb):
        p = f"blocks.{i}."
        s += [(p + "ln1_w", (W,), "gamma"), (p + "ln1_b", (W,), "beta"),
              (p + "qkv_w", (3 * W, W), "w"), (p + "qkv_b", (3 * W,), "bias"),
              (p + "proj_w", (W, W), "w"), (p + "proj_b", (W,), "bias"),
              (p + "ln2_w", (W,), "gamma"), (p + "ln2_b", (W,), "beta"),
              (p + "fc1_w", (F, W), "w"), (p + "fc1_b", (F,), "bias"),
              (p + "fc2_w", (W, F), "w"), (p + "fc2_b", (W,), "bias"),
              # temporal pre-norm (RMSNorm gamma), RG-LRU input gate Wx, recurrence gate Wa (768 -> 768
              # each) and a_param (softplus argument)
              (p + "rms_w", (W,), "gamma"),
              (p + "gx_w", (W, W), "w"), (p + "gx_b", (W,), "bias"),
              (p + "ga_w", (W, W), "w"), (p + "ga_b", (W,), "bias"),
              (p + "a_param", (W,), "normal1")]
    s += [("final_ln_w", (W,), "gamma"), ("final_ln_b", (W,), "beta")]
    return s


def tapnext_weights(cfg: TapNextConfig, seed=0, n_blocks=None, affine="zero"):
    return _generate(tapnext_spec(cfg, n_blocks), seed, affine)


def tapnextpp_spec(cfg: TapNextConfig, n_blocks=None):
    """The full TAPNext++ block's weight set (tapnext/npu/step8.py:161-183, 205-215): per block the recurrent
    block (temporal RMSNorm scale, linear_yx 768 -> 1536, conv_1d 4 taps, block-diagonal RG-LRU gates
    [12, 64 in, 64 out], a_param, linear_out), the gated MLP (channel RMSNorm scale, ffw_up 768 -> 2 x 3072 as
    [gate | up], ffw_down 3072 -> 768) and the ViT block (ln_1, qkv, out_proj, ln_2, mlp.0, mlp.3)."""
    W, F = cfg.width, cfg.ff
    H, D = cfg.heads, cfg.head_dim
    nb = cfg.n_blocks if n_blocks is None else n_blocks
    s = [("patch_w", (W, cfg.patch_k), "w"), ("patch_b", (W,), "bias"), ("pos_emb", (cfg.n_img_tok, W), "w")]
    for i in range(nb):
        p = f"blocks.{i}."
        s += [(p + "rms0_scale", (W,), "scale"),
              (p + "yx_w", (2 * W, W), "w"), (p + "yx_b", (2 * W,), "bias"),
              (p + "conv_w", (4, W), "conv"), (p + "conv_b", (W,), "bias"),
              (p + "gx_w", (H, D, D), "w"), (p + "gx_b", (W,), "bias"),
              (p + "ga_w", (H, D, D), "w"), (p + "ga_b", (W,), "bias"),
              (p + "a_param", (W,), "normal1"),
              (p + "out_w", (W, W), "w"), (p + "out_b", (W,), "bias"),
              (p + "rms1_scale", (W,), "scale"),
              (p + "up_w", (2 * F, W), "w"), (p + "up_b", (2 * F,), "bias"),
              (p + "down_w", (W, F), "w"), (p + "down_b", (W,), "bias"),
              (p + "ln1_w", (W,), "gamma"), (p + "ln1_b", (W,), "beta"),
              (p + "qkv_w", (3 * W, W), "w"), (p + "qkv_b", (3 * W,), "bias"),
              (p + "proj_w", (W, W), "w"), (p + "proj_b", (W,), "bias"),
              (p + "ln2_w", (W,), "gamma"), (p + "ln2_b", (W,), "beta"),
              (p + "fc1_w", (F, W), "w"), (p + "fc1_b", (F,), "bias"),
              (p + "fc2_w", (W, F), "w"), (p + "fc2_b", (W,), "bias")]
    s += [("final_ln_w", (W,), "gamma"), ("final_ln_b", (W,), "beta")]
    return s


def tapnextpp_weights(cfg: TapNextConfig, seed=0, n_blocks=None, affine="zero"):
    return _generate(tapnextpp_spec(cfg, n_blocks), seed, affine)


def heads_spec(cfg: TapNextConfig):
    """The TAPNext++ tracking heads (model.coordinate_head / visible_head, indexed as step8.py:335 reads them:
    [0] Linear, [1] LayerNorm, [3] Linear, [4] LayerNorm, [6] Linear): weights [out, in] as torch stores them."""
    W, Hh, nb = cfg.width, cfg.head_hidden, cfg.track_bins
    s = []
    for name, n_out in (("coord", 2 * nb), ("vis", 1)):
        s += [(f"{name}.0_w", (Hh, W), "w"), (f"{name}.0_b", (Hh,), "bias"),
              (f"{name}.1_w", (Hh,), "gamma"), (f"{name}.1_b", (Hh,), "beta"),
              (f"{name}.3_w", (Hh, Hh), "w"), (f"{name}.3_b", (Hh,), "bias"),
              (f"{name}.4_w", (Hh,), "gamma"), (f"{name}.4_b", (Hh,), "beta"),
              (f"{name}.6_w", (n_out, Hh), "wout"), (f"{name}.6_b", (n_out,), "bias")]
    return s


def heads_weights(cfg: TapNextConfig, seed=0, affine="random"):
    return _generate(heads_spec(cfg), seed, affine)


def heads_input(cfg: TapNextConfig, seed=11, n=None):
    """Query tokens for the heads, N(0, 1) [n_queries, width] float32 (the GPU path feeds them as bf16; callers
    that compare against it round them to bf16 first)."""
    n = cfg.n_queries if n is None else n
    return np.random.default_rng(np.random.SeedSequence([int(seed), 0])).standard_normal((n, cfg.width), dtype=np.float32)


def text_spec(cfg, n_layers=None):
    """The text decoder's weight set, named after FastMD2's attributes (md2fast.py:111-117, 143): wte,
    tblocks[i].{ln, qkv, proj, fc1, fc2}, tpost_ln, lm_small (the yes / no rows of lm_head)."""
    D, Fh = cfg.dim, cfg.ff
    nl = cfg.n_layers if n_layers is None else n_layers
    s = [("wte", (cfg.vocab, D), "normal1")]
    for i in range(nl):
        p = f"tblocks.{i}."
        s += [(p + "ln_w", (D,), "gamma"), (p + "ln_b", (D,), "beta"),
              (p + "qkv_w", (3 * D, D), "w"), (p + "qkv_b", (3 * D,), "bias"),
              (p + "proj_w", (D, D), "w"), (p + "proj_b", (D,), "bias"),
              (p + "fc1_w", (Fh, D), "w"), (p + "fc1_b", (Fh,), "bias"),
              (p + "fc2_w", (D, Fh), "w"), (p + "fc2_b", (D,), "bias")]
    s += [("tpost_ln_w", (D,), "gamma"), ("tpost_ln_b", (D,), "beta"),
          ("lm_small_w", (cfg.n_yn, D), "w"), ("lm_small_b", (cfg.n_yn,), "bias")]
    return s


def text_weights(cfg, seed=0, n_layers=None, affine="zero"):
    return _generate(text_spec(cfg, n_layers), seed, affine)


def text_weights_device(cfg, device, seed=0, n_layers=None):
    """Timing weights for the text decoder drawn directly on the device from a seeded torch generator:
    N(0, 0.02) matrices (N(0, 1) embeddings), LayerNorm gamma 1 and beta / bias 0 (the parity tests use the
    host generator of text_weights instead)."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    W = {}
    for name, shape, kind in text_spec(cfg, n_layers):
        if kind == "gamma":
            W[name] = torch.ones(shape, device=device)
        elif kind in ("beta", "bias"):
            W[name] = torch.zeros(shape, device=device)
        else:
            W[name] = torch.randn(shape, device=device, generator=g) * (1.0 if kind == "normal1" else 0.02)
    return W


def text_inputs(cfg, seed=5):
    """Image-token embeddings N(0, 1) [729, dim] (the projection output), bos id, and a question: token ids
    [q_len] in the synthetic vocabulary with its last real position."""
    rng = np.random.default_rng(np.random.SeedSequence([int(seed), 11]))
    emb = rng.standard_normal((cfg.prefix - 1, cfg.dim), dtype=np.float32)
    n_real = int(rng.integers(cfg.q_len // 2, cfg.q_len + 1))
    ids = np.zeros(cfg.q_len, np.int64)
    ids[:n_real] = rng.integers(1, cfg.vocab, n_real)
    return emb, 0, ids, n_real - 1


def crop_pixels(n, cfg: TowerConfig, seed=1, first=0):
    """Crops n pixels U[-1,1] as float32 [n, 3, img, img]; crop i uses stream (seed, 1_000_000 + first + i)."""
    out = np.empty((n, cfg.in_ch, cfg.img, cfg.img), np.float32)

    def one(i):
        rng = np.random.default_rng(np.random.SeedSequence([int(seed), 1_000_000 + first + i]))
        out[i] = rng.random((cfg.in_ch, cfg.img, cfg.img), dtype=np.float32) * np.float32(2) - np.float32(1)
    with ThreadPoolExecutor(8) as ex:
        list(ex.map(one, range(n)))
    return out


def tapnext_inputs(cfg: TapNextConfig, n_frames, seed=2):
    """frames U[-1,1] [F, 3, img, img] and point-query tokens N(0,1) [F, n_queries, width]."""
    rng = np.random.default_rng(np.random.SeedSequence([int(seed), 7]))
    frames = rng.random((n_frames, cfg.in_ch, cfg.img, cfg.img), dtype=np.float32) * np.float32(2) - np.float32(1)
    queries = rng.standard_normal((n_frames, cfg.n_queries, cfg.width), dtype=np.float32)
    return frames, queries


def crop_u8(n, cfg: TowerConfig, seed=3):
    """n uint8 HWC crops [n, img, img, 3] (the input FastMD2._vision takes, md2fast.py:147-148)."""
    out = np.empty((n, cfg.img, cfg.img, cfg.in_ch), np.uint8)
    for i in range(n):
        rng = np.random.default_rng(np.random.SeedSequence([int(seed), 2_000_000 + i]))
        out[i] = rng.integers(0, 256, (cfg.img, cfg.img, cfg.in_ch), dtype=np.uint8)
    return out


def block_input(cfg: TowerConfig, seed=4, batch=1):
    """Config 0 block input: activations N(0, 1) [batch, 729, width]."""
    rng = np.random.default_rng(np.random.SeedSequence([int(seed), 3_000_000]))
    return rng.standard_normal((batch, cfg.ntok, cfg.width), dtype=np.float32)
