"""Generate tests/golden/text_2_random.npz: pins oracle/text_ref.py to the reference's text decoder.

Runs the reference's own FastMD2._text_layers and FastMD2._query (moondream/gpu/md2fast.py:169-212), imported
read-only from a checkout of the reference, on a FastMD2 shell holding the seeded fp32 text weights of
strix_halo_maxx_b200.weights.text_weights (2 layers, random affine terms), laid out as md2fast.py:111-143
does, with the unfused attention path (fuse off, no hattn).  The rotary cos / sin come from
oracle.text_ref.rope_angles (the reference reads them from the HF model's freqs_cis, which is not in the
repository).  The prefix is [wte[bos]; image embeddings] as _encode builds it (md2fast.py:201-206).

    python tests/golden/make_golden_text.py /path/to/reference

Stores: the yes / no logits, and for the prefix hidden states (the last layer's output) 24 full rows, per-row
norms and 8 random projections of every row.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from strix_halo_maxx_b200.config import TEXT                  # noqa: E402
from strix_halo_maxx_b200 import weights as wg                 # noqa: E402
from oracle.text_ref import rope_angles, query_mask            # noqa: E402

N_LAYERS = 2
ROWS = np.unique(np.linspace(0, TEXT.prefix - 1, 24).round().astype(np.int64))


def probe(dim):
    return np.random.default_rng(np.random.SeedSequence([19, dim])).standard_normal((dim, 8))


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python " + os.path.basename(__file__) + " /path/to/reference")
    ref = sys.argv[1]
    sys.path.insert(0, os.path.join(ref, "moondream", "gpu"))
    import md2fast  # noqa: E402
    cfg, f32 = TEXT, torch.float32
    W = wg.text_weights(cfg, seed=3, n_layers=N_LAYERS, affine="random")
    emb, bos, ids, last = wg.text_inputs(cfg, seed=5)
    t = lambda n: torch.from_numpy(W[n]).contiguous()
    L = lambda n: md2fast.Lin(t(n + "_w"), t(n + "_b"), f32)
    m = object.__new__(md2fast.FastMD2)
    m.th, m.hd, m.fuse, m.hattn, m.dtype = cfg.heads, cfg.head_dim, False, False, f32
    m.tblocks = [dict(ln=(t(f"tblocks.{i}.ln_w"), t(f"tblocks.{i}.ln_b")), qkv=L(f"tblocks.{i}.qkv"),
                      proj=L(f"tblocks.{i}.proj"), fc1=L(f"tblocks.{i}.fc1"), fc2=L(f"tblocks.{i}.fc2"))
                 for i in range(N_LAYERS)]
    m.kc = [torch.zeros(1, cfg.heads, cfg.ctx, cfg.head_dim) for _ in range(N_LAYERS)]
    m.vc = [torch.zeros(1, cfg.heads, cfg.ctx, cfg.head_dim) for _ in range(N_LAYERS)]
    m.wte, m.prefix, m.L = t("wte"), cfg.prefix, cfg.q_len
    m.tpost_ln, m.full_logits = (t("tpost_ln_w"), t("tpost_ln_b")), False
    m.lm_small = L("lm_small")
    md2fast.USE_FUSED_RES = False
    cos_pre, sin_pre = rope_angles(cfg, 0, cfg.prefix)
    m.cos_q, m.sin_q = rope_angles(cfg, cfg.prefix, cfg.q_len)
    m.qmask = query_mask(cfg)
    m.tok_buf = torch.from_numpy(ids)[None]
    m.last_idx = torch.tensor([last])
    with torch.no_grad():
        x = torch.cat([m.wte[bos][None], torch.from_numpy(emb)], dim=0)[None]
        xp = m._text_layers(x, 0, cfg.prefix, cos_pre, sin_pre, None)[0].numpy()
        logits = m._query()[0].numpy()
    out = dict(logits=logits.astype(np.float32), rows=ROWS, out_rows=xp[ROWS].astype(np.float32),
               norms=np.linalg.norm(xp, axis=1).astype(np.float32), probes=(xp @ probe(cfg.dim)).astype(np.float32))
    path = os.path.join(HERE, "text_2_random.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, "logits", logits)


if __name__ == "__main__":
    main()
