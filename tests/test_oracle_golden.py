"""Pin the CPU oracle (oracle/tower_ref.py) to the reference: the fixtures in tests/golden were produced
by the reference's own FastMD2._vision (moondream/gpu/md2fast.py:147-160) on the same seeded weights
and inputs (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from strix_halo_maxx_b200.config import TowerConfig
from strix_halo_maxx_b200 import weights as wg
from oracle import tower_ref
from helpers import load_golden, golden_rel, rglru_case, RGLRU_TOL

CFG = TowerConfig()
TOL = 2e-4   # fp32 vs fp32 (same algorithm, possibly different summation order)


def _weights(meta):
    W = wg.tower_weights(CFG, seed=meta["wseed"], n_blocks=meta["n_blocks"], affine=meta["affine"])
    return W


@pytest.mark.parametrize("name", ["vision_u8_27_zero", "vision_u8_2_random", "vision_u8_2_random_foldproj"])
def test_vision_u8(name):
    g = load_golden(name)
    m = g["meta"]
    W = _weights(m)
    assert np.allclose(g["wsum"], [np.abs(W["patch_w"]).sum(), np.abs(W["blocks.0.qkv_w"]).sum(),
                                   np.abs(W["pos_emb"]).sum()], rtol=1e-6), "weight generator drifted"
    img = wg.crop_u8(1, CFG, seed=m["img_seed"])[0]
    out = tower_ref.vision_u8(img, W, CFG, eps=m["eps"], n_blocks=m["n_blocks"], fold_proj=m.get("fold_proj", False))
    assert max(golden_rel(out, g)) < TOL


@pytest.mark.parametrize("name", ["tower_u8_27_zero", "tower_u8_2_random"])
def test_tower_u8(name):
    g = load_golden(name)
    m = g["meta"]
    W = _weights(m)
    img = wg.crop_u8(1, CFG, seed=m["img_seed"])[0]
    out = tower_ref.tower(tower_ref.normalize_u8(img), W, CFG, eps=m["eps"], n_blocks=m["n_blocks"])[0]
    assert max(golden_rel(out, g)) < TOL


def test_tower_pixels():
    g = load_golden("tower_pix_27_zero")
    m = g["meta"]
    W = _weights(m)
    pix = wg.crop_pixels(1, CFG, seed=m["pix_seed"])
    out = tower_ref.tower(torch.from_numpy(pix), W, CFG, eps=m["eps"], n_blocks=27)[0]
    assert max(golden_rel(out, g)) < TOL


def test_block():
    g = load_golden("block_1_random")
    m = g["meta"]
    W = _weights(m)
    x = torch.from_numpy(wg.block_input(CFG, seed=m["x_seed"]))
    out = tower_ref.block(x, W, 0, CFG.heads, m["eps"])[0]
    assert max(golden_rel(out, g)) < TOL


def test_golden_detects_a_planted_error():
    """The comparison is not vacuous: an oracle with a wrong eps (1e-6 instead of the reference's 1e-5) on
    the 2-block affine case, or a transposed im2col, fails it."""
    g = load_golden("tower_u8_2_random")
    m = g["meta"]
    W = _weights(m)
    img = wg.crop_u8(1, CFG, seed=m["img_seed"])[0]
    pix = tower_ref.normalize_u8(img)
    bad = tower_ref.tower(pix.transpose(2, 3), W, CFG, eps=m["eps"], n_blocks=2)[0]
    assert max(golden_rel(bad, g)) > 1e-2


@pytest.mark.parametrize("case,first", [("first", True), ("next", False)])
def test_ssm_restatement_matches_reference_ssm_ref(case, first):
    """oracle.tapnextpp_ref.ssm_bf16 against the outputs of the reference's own tapnext/npu/pack8.py
    ssm_ref (tests/golden/make_golden_ssm.py): bit-exact z and h."""
    import numpy as np
    from oracle.tapnextpp_ref import ssm_bf16
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "ssm_ref_cases.npz"))
    a = {k.split(".", 1)[1]: g[k] for k in g.files if k.startswith(case + ".")}
    z, h = ssm_bf16(a["y"], a["x"], a["xm1"], a["xm2"], a["xm3"], a["h0"], a["conv_w"], a["conv_b"], a["a_param"],
                    a["wx"], a["bx"], a["wa"], a["ba"], first)
    assert np.array_equal(z.numpy(), a["z"]) and np.array_equal(h.numpy(), a["h"])


def test_ssm_restatement_detects_a_planted_error():
    """The same check fails for a restatement with the conv taps in the wrong order."""
    import numpy as np
    from oracle.tapnextpp_ref import ssm_bf16
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "ssm_ref_cases.npz"))
    a = {k.split(".", 1)[1]: g[k] for k in g.files if k.startswith("next.")}
    z, _ = ssm_bf16(a["y"], a["x"], a["xm1"], a["xm2"], a["xm3"], a["h0"], a["conv_w"][::-1].copy(), a["conv_b"],
                    a["a_param"], a["wx"], a["bx"], a["wa"], a["ba"], False)
    assert not np.array_equal(z.numpy(), a["z"])


def _rglru_stream(W, frames, c=8.0):
    from oracle import tapnext_ref
    h, errs = None, []
    for x, ref in frames:
        h = tapnext_ref.rglru(torch.from_numpy(x), W, "", h, c)
        r = torch.from_numpy(ref)
        errs.append(float(((h - r).norm(dim=-1) / r.norm(dim=-1)).max()))
    return errs


def test_rglru_restatement_matches_reference_ssm_ref():
    """oracle.tapnext_ref.rglru (the RG-LRU of the TAPNext-style step, dense 768 x 768 gates) against the reference's
    own ssm_ref (tapnext/npu/pack8.py:252-279) run with 12 heads of block-diagonal gates and identity conv taps:
    a first frame and the next one, state carried, every row within 1e-2 (ssm_ref's bf16 rounding points)."""
    W, frames = rglru_case()
    errs = _rglru_stream(W, frames)
    assert max(errs) < RGLRU_TOL, errs


@pytest.mark.parametrize("plant", ["transposed_gates", "swapped_gates", "coefficient_4"])
def test_rglru_restatement_detects_a_planted_error(plant):
    """The same fixture rejects gate matrices used transposed, the input and recurrence gates swapped, and the
    wrong recurrence coefficient (c = 4 instead of 8, which only the second frame sees)."""
    W, frames = rglru_case()
    c = 8.0
    if plant == "transposed_gates":
        W = {**W, "gx_w": W["gx_w"].T.copy(), "ga_w": W["ga_w"].T.copy()}
    elif plant == "swapped_gates":
        W = {**W, "gx_w": W["ga_w"], "ga_w": W["gx_w"], "gx_b": W["ga_b"], "ga_b": W["gx_b"]}
    else:
        c = 4.0
    assert max(_rglru_stream(W, frames, c)) > 10 * RGLRU_TOL


def _heads_case():
    from strix_halo_maxx_b200.config import TAPNEXT
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "heads_ref_cases.npz"))
    HW = wg.heads_weights(TAPNEXT, seed=int(g["wseed"]))
    x = torch.from_numpy(wg.heads_input(TAPNEXT, seed=int(g["xseed"]))).to(torch.bfloat16).float()
    return TAPNEXT, HW, x, g


def test_heads_restatement_matches_reference_heads_np():
    """oracle.tapnextpp_ref.heads against the reference's own Step8.heads_np (tapnext/npu/step8.py:327-362,
    tests/golden/make_golden_heads.py): logits, tracks and visibility, fp32 against fp32."""
    from oracle import tapnextpp_ref
    cfg, HW, x, g = _heads_case()
    tracks, logits, vis = tapnextpp_ref.heads(x, HW, cfg)
    assert np.allclose(logits.numpy(), g["logits"], rtol=1e-4, atol=1e-4)
    assert np.abs(tracks.numpy() - g["tracks"]).max() < 1e-3          # pixels
    assert np.allclose(vis.numpy(), g["vis"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("plant", ["window_10", "temperature_1"])
def test_heads_restatement_detects_a_planted_error(plant):
    """The fixture rejects a soft-argmax window of +-10 bins and a temperature of 1 (instead of +-20, 0.5)."""
    import dataclasses
    from oracle import tapnextpp_ref
    cfg, HW, x, g = _heads_case()
    bad = dataclasses.replace(cfg, track_window=10) if plant == "window_10" else dataclasses.replace(cfg, track_temperature=1.0)
    tracks, _, _ = tapnextpp_ref.heads(x, HW, bad)
    assert np.abs(tracks.numpy() - g["tracks"]).max() > 0.1


def _text_case():
    from strix_halo_maxx_b200.config import TEXT
    from oracle import text_ref
    W = wg.text_weights(TEXT, seed=3, n_layers=2, affine="random")
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "text_2_random.npz"))
    return TEXT, text_ref, W, emb, bos, ids, last, g


def test_text_oracle_matches_reference_text_layers_and_query():
    """oracle.text_ref against the reference's own FastMD2._text_layers / _query outputs
    (tests/golden/make_golden_text.py): the prefix hidden states and the yes / no logits."""
    TEXT, text_ref, W, emb, bos, ids, last, g = _text_case()
    x, cache = text_ref.encode(emb, bos, W, TEXT, n_layers=2)
    logits = text_ref.query(ids, last, W, TEXT, cache, n_layers=2)
    assert np.allclose(x.numpy()[g["rows"]], g["out_rows"], rtol=1e-5, atol=1e-5)
    assert np.allclose(np.linalg.norm(x.numpy(), axis=1), g["norms"], rtol=1e-5)
    assert np.allclose(logits.numpy(), g["logits"], rtol=1e-5, atol=1e-5)


def test_text_oracle_detects_a_planted_error():
    """The same fixture rejects a restatement with the wrong rotary base (theta 1000 instead of 10000).
    (A wrong pair layout of the rotated dims would not show: it permutes q and k alike, so q.k is unchanged.)"""
    import dataclasses
    TEXT, text_ref, W, emb, bos, ids, last, g = _text_case()
    x, _ = text_ref.encode(emb, bos, W, dataclasses.replace(TEXT, theta=1000.0), n_layers=2)
    assert not np.allclose(x.numpy()[g["rows"]], g["out_rows"], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("h,w", [(480, 640), (375, 500), (1080, 1920), (300, 200), (378, 378)])
def test_resize_restatement_matches_pillow_bit_for_bit(h, w):
    """oracle.resize_ref (Pillow's two-pass LANCZOS restated) against Pillow's own Image.resize, the call
    FastMD2.set_image makes (md2fast.py:223-228)."""
    from PIL import Image
    from oracle.resize_ref import resize_lanczos
    rng = np.random.default_rng(h * w)
    img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    yy, xx = np.mgrid[0:h, 0:w]
    img[..., 1] = ((np.sin(xx / 13.0) + np.cos(yy / 7.0)) * 60 + 128).astype(np.uint8)
    ref = np.asarray(Image.fromarray(img).resize((378, 378), Image.Resampling.LANCZOS))
    assert np.array_equal(resize_lanczos(img, 378, 378), ref)


def _i8_golden():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "i8_quant_gemm.npz"))


def test_i8_restatement_matches_reference_numerics_bit_for_bit():
    """oracle/i8_ref.py against the reference's own numpy HI8Lin numerics (tests/golden/make_golden_i8.py):
    activation and weight quantisation, the exact int32 products and the fp32 epilogue, with and without GELU."""
    from oracle import i8_ref
    g = _i8_golden()
    q, sx = i8_ref.quant_rows(g["x"])
    wq, sw = i8_ref.quant_w(g["w"])
    assert np.array_equal(q, g["q"]) and np.array_equal(sx, g["sx"])
    assert np.array_equal(wq, g["wq"]) and np.array_equal(sw, g["sw"])
    acc = i8_ref.i8_matmul(q, wq)
    assert np.array_equal(acc, g["acc"])
    assert np.array_equal(i8_ref.epilogue(acc, sx, sw, g["bias"], False), g["y0"])
    assert np.allclose(i8_ref.epilogue(acc, sx, sw, g["bias"], True), g["y1"], rtol=1e-6, atol=1e-7)
    # the edge rows: scale floors, half-way points rounded away from zero (activations) / to even (weights)
    assert sx[0] == np.float32(1e-5) / np.float32(127) and not q[0].any()
    assert sw[0] == np.float32(1e-8) / np.float32(127) and not wq[0].any()
    assert sx[3] == 1.0 and sw[1] == 1.0
    xh, wh = g["x"][3], g["w"][1]
    half_x, half_w = (xh % 1) == 0.5, (wh % 1) == 0.5
    assert half_x.sum() > 100 and half_w.sum() > 100
    assert np.array_equal(q[3][half_x], (np.sign(xh) * np.ceil(np.abs(xh)))[half_x].astype(np.int8))
    assert np.array_equal(wq[1][half_w], np.rint(wh)[half_w].astype(np.int8))
    assert (np.abs(q[3][half_x]) % 2 == 1).any() and (np.abs(wq[1][half_w]) % 2 == 0).all()


def test_i8_restatement_detects_a_planted_error():
    """A quantiser that rounds half to even (instead of away from zero) is caught by the fixture."""
    from oracle import i8_ref
    g = _i8_golden()
    x = g["x"].astype(np.float32)
    s = (np.maximum(np.abs(x).max(axis=1), np.float32(1e-5)) / np.float32(127.0)).astype(np.float32)
    wrong = np.clip(np.rint(x / s[:, None]), -127, 127).astype(np.int8)
    assert not np.array_equal(wrong, g["q"])
    assert np.array_equal(i8_ref.quant_rows(x)[0], g["q"])
