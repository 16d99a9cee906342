"""Tower parity on the GPU against the CPU fp32 oracle (pinned to the reference by tests/golden): per
output token max relative error <= 2e-2 and cosine >= 0.999."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200.config import TowerConfig
from strix_halo_maxx_b200 import weights as wg
from strix_halo_maxx_b200.tower import VisionTower, vt_vision, enable
from strix_halo_maxx_b200._lib import device_status
from oracle import tower_ref
from helpers import assert_tokens_close, load_golden, golden_rel, TOK_REL

CFG = TowerConfig()
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status():
    device_status(clear=True)
    yield
    assert device_status(clear=True) == 0


@pytest.fixture(scope="module")
def w27():
    return wg.tower_weights(CFG, seed=0, n_blocks=27)


@pytest.fixture(scope="module")
def tower27(w27):
    return VisionTower(w27, CFG, device=DEV)


@pytest.mark.parametrize("fold_ln", [True, False])
def test_config0_one_block_random_affine(fold_ln):
    W = wg.tower_weights(CFG, seed=6, n_blocks=1, affine="random")
    x = torch.from_numpy(wg.block_input(CFG, seed=4, batch=2))
    ref = tower_ref.block(x, W, 0, CFG.heads, CFG.eps)
    out = VisionTower(W, CFG, device=DEV, fold_ln=fold_ln).run_blocks(x.to(DEV))
    assert_tokens_close(out.cpu(), ref, what="config 0 block")


def test_config1_full_tower(tower27, w27):
    pix = torch.from_numpy(wg.crop_pixels(1, CFG, seed=1))
    ref = tower_ref.tower(pix, w27, CFG)
    out = tower27.forward(pix.to(DEV))
    r, c = assert_tokens_close(out.float().cpu(), ref, what="config 1 tower (27 blocks)")
    print(f"config 1: max per-token rel {r:.3e}, min cos {c:.6f}")


def test_config1_full_tower_unfolded_layernorm(w27):
    pix = torch.from_numpy(wg.crop_pixels(1, CFG, seed=1))
    ref = tower_ref.tower(pix, w27, CFG)
    out = VisionTower(w27, CFG, device=DEV, fold_ln=False).forward(pix.to(DEV))
    assert_tokens_close(out.float().cpu(), ref, what="config 1 tower, LayerNorm as separate passes")


def test_batch_of_crops_is_bit_identical_to_single_crops(tower27):
    pix = torch.from_numpy(wg.crop_pixels(3, CFG, seed=11)).to(DEV)
    both = tower27.forward(pix).clone()
    one = tower27.forward(pix[1:2]).clone()
    assert torch.equal(both[1], one[0])


def test_bench_chunk_of_130_crops_is_bit_identical_to_single_crops(tower27):
    """At the bench's chunk size (130 crops, M = 94,770) the GEMMs run as CTA pairs (proj with the staged TMA
    epilogue) while a single crop's proj takes 128 x 64 tiles: every row is computed the same way regardless,
    so crops must come out bit-identical."""
    pix = torch.from_numpy(wg.crop_pixels(130, CFG, seed=12)).to(DEV)
    chunk = tower27.forward(pix).clone()
    for i in (0, 64, 129):
        one = tower27.forward(pix[i:i + 1]).clone()
        assert torch.equal(chunk[i], one[0]), i


def test_uint8_input_and_eps_1e5_against_reference_golden():
    """The product path against the reference's own FastMD2._vision output (golden, eps 1e-5, 27 blocks)."""
    g = load_golden("vision_u8_27_zero")
    W = wg.tower_weights(CFG, seed=0, n_blocks=27)
    t = VisionTower(W, CFG, eps=1e-5, device=DEV)
    img = torch.from_numpy(wg.crop_u8(1, CFG, seed=3)[0]).to(DEV)
    out = t.vision_u8(img).float().cpu()
    rows_rel, proj_rel, _ = golden_rel(out, g)
    assert rows_rel <= TOK_REL and proj_rel <= TOK_REL, (rows_rel, proj_rel)


@pytest.mark.parametrize("fold_ln", [True, False])
def test_affine_two_blocks_with_projection(fold_ln):
    W = wg.tower_weights(CFG, seed=5, n_blocks=2, affine="random")
    img = wg.crop_u8(1, CFG, seed=3)[0]
    ref = tower_ref.vision_u8(img, W, CFG, eps=1e-5, n_blocks=2)
    t = VisionTower(W, CFG, eps=1e-5, device=DEV, fold_ln=fold_ln)
    out = t.vision_u8(torch.from_numpy(img).to(DEV))
    assert_tokens_close(out.float().cpu(), ref, what="vision_u8 2 blocks affine")


def _fastmd2_shell(W, n_blocks, fold_proj=False):
    """An object with the vision attributes of a FastMD2 instance, laid out the way FastMD2.__init__ lays them out
    (md2fast.py:89-109, incl. the fold_proj branch, md2fast.py:97-101) with the reference's Lin holder
    (md2fast.py:33-40: .w, .b), as tests/golden/make_golden.py builds the shell it runs the reference on."""
    class Shell:
        def _vision(self, img_u8):
            raise AssertionError("not swapped")
    from oracle.tower_ref import _t

    class Lin:
        def __init__(self, w, b):
            self.w, self.b = _t(w).contiguous(), _t(b).contiguous()
    m = Shell()
    m.dtype = torch.float32
    m.patch_emb = Lin(W["patch_w"], W["patch_b"])
    m.pos_emb = _t(W["pos_emb"])[None]
    m.vblocks = [dict(ln1=(_t(W[f"blocks.{i}.ln1_w"]), _t(W[f"blocks.{i}.ln1_b"])), qkv=Lin(W[f"blocks.{i}.qkv_w"], W[f"blocks.{i}.qkv_b"]),
                      proj=Lin(W[f"blocks.{i}.proj_w"], W[f"blocks.{i}.proj_b"]), ln2=(_t(W[f"blocks.{i}.ln2_w"]), _t(W[f"blocks.{i}.ln2_b"])),
                      fc1=Lin(W[f"blocks.{i}.fc1_w"], W[f"blocks.{i}.fc1_b"]), fc2=Lin(W[f"blocks.{i}.fc2_w"], W[f"blocks.{i}.fc2_b"]))
                 for i in range(n_blocks)]
    m.post_ln = (_t(W["post_ln_w"]), _t(W["post_ln_b"]))
    m.fold_proj = fold_proj
    w1 = _t(W["proj_fc1_w"]).float()
    if fold_proj:
        w1 = w1[:, :CFG.width] + w1[:, CFG.width:]
    m.proj_fc1 = Lin(w1, W["proj_fc1_b"])
    m.proj_fc2 = Lin(W["proj_fc2_w"], W["proj_fc2_b"])
    m.vh = CFG.heads
    m.hattn = False
    return Shell, m


def test_drop_in_swaps_fastmd2_vision():
    """vt_vision replaces FastMD2._vision the way bf16emu.enable does (bf16emu.py:148-153)."""
    W = wg.tower_weights(CFG, seed=5, n_blocks=2, affine="random")
    Shell, m = _fastmd2_shell(W, 2)
    enable(Shell)
    img = wg.crop_u8(1, CFG, seed=3)[0]
    out = m._vision(torch.from_numpy(img).to(DEV))
    ref = tower_ref.vision_u8(img, W, CFG, eps=1e-5, n_blocks=2)
    assert_tokens_close(out.float().cpu(), ref, what="FastMD2._vision swap")


def test_drop_in_fold_proj_against_reference_golden():
    """A FastMD2 built with fold_proj=True (proj_fc1's K-halves summed, applied to x instead of cat([x, x]),
    md2fast.py:97-101, 159) takes the drop-in too: its output against the reference's own _vision output for
    that instance (tests/golden/vision_u8_2_random_foldproj.npz)."""
    g = load_golden("vision_u8_2_random_foldproj")
    m_ = g["meta"]
    W = wg.tower_weights(CFG, seed=m_["wseed"], n_blocks=m_["n_blocks"], affine=m_["affine"])
    Shell, m = _fastmd2_shell(W, m_["n_blocks"], fold_proj=True)
    enable(Shell)
    img = wg.crop_u8(1, CFG, seed=m_["img_seed"])[0]
    out = m._vision(torch.from_numpy(img).to(DEV)).float().cpu()
    assert out.shape == (729, 2048)
    rows_rel, proj_rel, _ = golden_rel(out, g)
    assert rows_rel <= TOK_REL and proj_rel <= TOK_REL, (rows_rel, proj_rel)
    assert m._vt_tower.p1_k == CFG.width


def test_config2_frame_projection():
    W = wg.tower_weights(CFG, seed=7, n_blocks=4, affine="random")
    crops = torch.from_numpy(wg.crop_pixels(13, CFG, seed=12))
    ref = tower_ref.frame(crops, W, CFG, n_blocks=4)
    out = VisionTower(W, CFG, device=DEV).frame(crops.to(DEV))
    assert out.shape == (729, 2048)
    assert_tokens_close(out.float().cpu(), ref, what="config 2 frame")


def test_config2_frame_27_blocks(w27, tower27):
    """Config 2 as BASELINE states it: 13 crops through the full 27-block tower, combine, projection MLP."""
    crops = torch.from_numpy(wg.crop_pixels(13, CFG, seed=14))
    ref = tower_ref.frame(crops, w27, CFG)
    out = tower27.frame(crops.to(DEV))
    r, c = assert_tokens_close(out.float().cpu(), ref, what="config 2 frame (27 blocks)")
    print(f"config 2: max per-token rel {r:.3e}, min cos {c:.6f}")


def test_config2_identical_crops_reduce_to_single_crop_projection():
    """Known answer: 13 identical crops -> combine = cat([x, x]) -> the single-crop _vision projection."""
    W = wg.tower_weights(CFG, seed=7, n_blocks=2)
    t = VisionTower(W, CFG, device=DEV)
    pix = torch.from_numpy(wg.crop_pixels(1, CFG, seed=13)).to(DEV)
    frame = t.frame(pix.expand(13, -1, -1, -1).contiguous()).clone()
    f = t.forward(pix)[0]
    single = t.project(torch.cat([f, f], dim=-1)).clone()
    assert torch.equal(frame, single)
