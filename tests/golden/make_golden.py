"""Generate the golden vectors that pin oracle/tower_ref.py to the reference.

Runs the reference's own FastMD2._vision (moondream/gpu/md2fast.py:147-160), imported read-only
from the reference checkout, on a FastMD2 shell that holds seeded random fp32 `Lin` weights
(strix_halo_maxx_b200.weights; the shell is built the way md2fast.py:89-109 lays the weights out).
The reference math is not modified: two observation-only wrappers record the input of the last
`_ln` call (the post-LN input) and the features handed to the projection `mlp`.

Usage (in a container that has the reference checkout):
    python tests/golden/make_golden.py --ref <path to strix-halo-maxx checkout>
Writes tests/golden/*.npz: per case the token indices `rows`, their full outputs `out_rows`,
per-token L2 norms, sums and 8 random projections of every output token, and a weight checksum `wsum`.
Inputs and weights are regenerated from their seeds by the tests (numpy PCG64, platform independent).
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from strix_halo_maxx_b200.config import TowerConfig          # noqa: E402
from strix_halo_maxx_b200 import weights as wg               # noqa: E402

ROWS = np.unique(np.linspace(0, 728, 24).round().astype(np.int64))


def token_probe(dim):
    """Fixed random directions [dim, 8]: the fixture stores out @ probe for every token."""
    return np.random.default_rng(np.random.SeedSequence([9, dim])).standard_normal((dim, 8))


def weight_checksum(W):
    return np.array([float(np.abs(W["patch_w"]).sum()), float(np.abs(W["blocks.0.qkv_w"]).sum()),
                     float(np.abs(W["pos_emb"]).sum())], np.float64)


def shell(md2fast, W, cfg, n_blocks):
    """A FastMD2 with only the vision attributes _vision reads (md2fast.py:89-109), fp32 on CPU."""
    f32 = torch.float32
    L = lambda n: md2fast.Lin(torch.from_numpy(W[n + "_w"]), torch.from_numpy(W[n + "_b"]), f32)
    t = lambda n: torch.from_numpy(W[n]).contiguous()
    m = object.__new__(md2fast.FastMD2)
    m.dtype = f32
    m.patch_emb = L("patch")
    m.pos_emb = t("pos_emb")[None]
    m.vblocks = [dict(ln1=(t(f"blocks.{i}.ln1_w"), t(f"blocks.{i}.ln1_b")), qkv=L(f"blocks.{i}.qkv"), proj=L(f"blocks.{i}.proj"),
                      ln2=(t(f"blocks.{i}.ln2_w"), t(f"blocks.{i}.ln2_b")), fc1=L(f"blocks.{i}.fc1"), fc2=L(f"blocks.{i}.fc2"))
                 for i in range(n_blocks)]
    m.post_ln = (t("post_ln_w"), t("post_ln_b"))
    m.fold_proj = False
    m.proj_fc1 = L("proj_fc1")
    m.proj_fc2 = L("proj_fc2")
    m.vh = cfg.heads
    m.hattn = False
    md2fast.USE_FUSED_RES = False
    return m


class Recorder:
    """Observation-only wrappers around md2fast._ln and md2fast.mlp."""
    def __init__(self, md2fast):
        self.md, self.ln_in, self.proj_in = md2fast, None, None
        self._ln, self._mlp = md2fast._ln, md2fast.mlp

    def __enter__(self):
        def ln(x, wb):
            self.ln_in = x.detach().clone()
            return self._ln(x, wb)

        def mlp(fc1, fc2, h, res=None, pre=None):
            if res is None:
                self.proj_in = h.detach().clone()
            return self._mlp(fc1, fc2, h, res=res, pre=pre)
        self.md._ln, self.md.mlp = ln, mlp
        return self

    def __exit__(self, *a):
        self.md._ln, self.md.mlp = self._ln, self._mlp


def save(name, meta, out, W):
    out = out.detach().float().numpy()
    np.savez(os.path.join(HERE, name + ".npz"), meta=json.dumps(meta), rows=ROWS, out_rows=out[ROWS].astype(np.float32),
             tok_norm=np.linalg.norm(out.astype(np.float64), axis=-1), tok_sum=out.astype(np.float64).sum(-1),
             tok_proj=out.astype(np.float64) @ token_probe(out.shape[-1]),
             wsum=weight_checksum(W))
    print(name, out.shape, "norm mean", float(np.linalg.norm(out, axis=-1).mean()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the strix-halo-maxx checkout")
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.ref, "moondream", "gpu"))
    import md2fast
    torch.set_num_threads(os.cpu_count())
    cfg = TowerConfig()

    # (1) whole _vision on a uint8 crop, 27 blocks, BASELINE weights (zero biases, unit LN)
    for n_blocks, affine, wseed in ((27, "zero", 0), (2, "random", 5)):
        W = wg.tower_weights(cfg, seed=wseed, n_blocks=n_blocks, affine=affine)
        img = wg.crop_u8(1, cfg, seed=3)[0]
        m = shell(md2fast, W, cfg, n_blocks)
        with torch.no_grad(), Recorder(md2fast) as rec:
            out = m._vision(torch.from_numpy(img))
        meta = dict(case="vision_u8", n_blocks=n_blocks, affine=affine, wseed=wseed, img_seed=3, eps=1e-5)
        save(f"vision_u8_{n_blocks}_{affine}", meta, out, W)
        save(f"tower_u8_{n_blocks}_{affine}", dict(meta, case="tower_u8"), rec.proj_in[:, :cfg.width], W)

    # (2) the tower on U[-1,1] pixels: _vision normalises x/255*2-1, so it is given (pix + 1) * 127.5 (fp32)
    W = wg.tower_weights(cfg, seed=0, n_blocks=27)
    pix = wg.crop_pixels(1, cfg, seed=1)[0]
    img = torch.from_numpy(((pix + 1.0) * 127.5).transpose(1, 2, 0).copy())
    m = shell(md2fast, W, cfg, 27)
    with torch.no_grad(), Recorder(md2fast) as rec:
        m._vision(img)
    save("tower_pix_27_zero", dict(case="tower_pix", n_blocks=27, affine="zero", wseed=0, pix_seed=1, eps=1e-5),
         rec.proj_in[:, :cfg.width], W)

    # (3) config 0: one block on x ~ N(0,1): patch_emb returns x, pos_emb 0; the block output is the post-LN input
    W = wg.tower_weights(cfg, seed=6, n_blocks=1, affine="random")
    x0 = torch.from_numpy(wg.block_input(cfg, seed=4)[0])[None]
    m = shell(md2fast, W, cfg, 1)
    m.patch_emb = lambda _x: x0
    m.pos_emb = torch.zeros(1)
    with torch.no_grad(), Recorder(md2fast) as rec:
        m._vision(torch.zeros(cfg.img, cfg.img, 3, dtype=torch.uint8))
    save("block_1_random", dict(case="block", n_blocks=1, affine="random", wseed=6, x_seed=4, eps=1e-5), rec.ln_in[0], W)

    # (4) _vision with fold_proj=True: proj_fc1's two K-halves summed into one [8192, 1152] weight, applied to x
    #     instead of cat([x, x]) -- built the way FastMD2.__init__ folds it (md2fast.py:97-101)
    W = wg.tower_weights(cfg, seed=5, n_blocks=2, affine="random")
    img = wg.crop_u8(1, cfg, seed=3)[0]
    m = shell(md2fast, W, cfg, 2)
    w1 = torch.from_numpy(W["proj_fc1_w"]).float()
    w1 = (w1[:, :cfg.width] + w1[:, cfg.width:]).to(torch.float32)
    m.fold_proj = True
    m.proj_fc1 = md2fast.Lin(w1, torch.from_numpy(W["proj_fc1_b"]), torch.float32)
    with torch.no_grad():
        out = m._vision(torch.from_numpy(img))
    save("vision_u8_2_random_foldproj", dict(case="vision_u8", n_blocks=2, affine="random", wseed=5, img_seed=3, eps=1e-5,
                                             fold_proj=True), out, W)


if __name__ == "__main__":
    main()
