"""Generate tests/golden/heads_ref_cases.npz from the reference's own TAPNext++ tracking heads,
Step8.heads_np (tapnext/npu/step8.py:327-362), read from a checkout of the reference.

step8.py cannot be imported here: at import it loads the NPU runtime (pyxrt) and execs the vendored model
file (/tapnext/model.py), neither of which is in the repository.  heads_np itself needs only numpy, torch
and step8's f32 helper, so this script takes those two function definitions out of step8.py's source
(ast, unmodified) and runs them on a stand-in object whose model.coordinate_head / model.visible_head are
torch nn.Sequential heads in the layout heads_np indexes ([0] Linear, [1] LayerNorm, [2] GELU, [3] Linear,
[4] LayerNorm, [5] GELU, [6] Linear), holding seeded weights (strix_halo_maxx_b200.weights.heads_weights).

    python tests/golden/make_golden_heads.py /path/to/reference

Input: 256 query tokens N(0, 1) rounded to bf16 (the device step outputs bf16 tokens; heads_np takes them as
float32, step8.py:352).  Recorded: tracks [256, 2], logits [256, 512], visibility logits [256].
"""
import ast
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from strix_halo_maxx_b200.config import TAPNEXT       # noqa: E402
from strix_halo_maxx_b200 import weights as wg        # noqa: E402


def load_heads_np(ref_root):
    path = os.path.join(ref_root, "tapnext", "npu", "step8.py")
    tree = ast.parse(open(path).read(), path)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "f32"]
    for n in tree.body:
        if isinstance(n, ast.ClassDef) and n.name == "Step8":
            keep += [m for m in n.body if isinstance(m, ast.FunctionDef) and m.name == "heads_np"]
    assert len(keep) == 2, "f32 / Step8.heads_np not found"
    ns = {"np": np, "torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns["heads_np"]


def head_module(W, name, cfg):
    n_out = W[f"{name}.6_w"].shape[0]
    seq = torch.nn.Sequential(torch.nn.Linear(cfg.width, cfg.head_hidden), torch.nn.LayerNorm(cfg.head_hidden, eps=cfg.head_eps),
                              torch.nn.GELU(), torch.nn.Linear(cfg.head_hidden, cfg.head_hidden),
                              torch.nn.LayerNorm(cfg.head_hidden, eps=cfg.head_eps), torch.nn.GELU(),
                              torch.nn.Linear(cfg.head_hidden, n_out))
    with torch.no_grad():
        for i in (0, 1, 3, 4, 6):
            seq[i].weight.copy_(torch.from_numpy(W[f"{name}.{i}_w"]))
            seq[i].bias.copy_(torch.from_numpy(W[f"{name}.{i}_b"]))
    return seq


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python " + os.path.basename(__file__) + " /path/to/reference")
    heads_np = load_heads_np(sys.argv[1])
    cfg = TAPNEXT
    W = wg.heads_weights(cfg, seed=21)
    stub = types.SimpleNamespace(model=types.SimpleNamespace(coordinate_head=head_module(W, "coord", cfg),
                                                             visible_head=head_module(W, "vis", cfg)))
    x = torch.from_numpy(wg.heads_input(cfg, seed=11)).to(torch.bfloat16).float().numpy()
    tracks, logits, vis = heads_np(stub, x)
    path = os.path.join(HERE, "heads_ref_cases.npz")
    np.savez_compressed(path, wseed=21, xseed=11, tracks=np.asarray(tracks, np.float32),
                        logits=np.asarray(logits, np.float32), vis=np.asarray(vis, np.float32))
    print("wrote", path, "tracks", tracks.shape, "range", float(tracks.min()), float(tracks.max()),
          "vis", vis.shape, "logit std", float(logits.std()))


if __name__ == "__main__":
    main()
