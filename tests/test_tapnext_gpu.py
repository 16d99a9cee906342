"""TAPNext-style step (config 3) on the GPU against the CPU restatement, state carried over frames."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200.config import TapNextConfig
from strix_halo_maxx_b200 import weights as wg
from strix_halo_maxx_b200.tapnext import TapNextStep
from strix_halo_maxx_b200._lib import device_status
from oracle import tapnext_ref
from helpers import assert_tokens_close

CFG = TapNextConfig()


NORMS = {"in_gemm": dict(), "row_pass": dict(rows_in_gemm=False), "unfolded": dict(fold_ln=False)}


@pytest.mark.parametrize("n_blocks,n_frames,affine,norms", [(12, 16, "zero", "in_gemm"), (3, 16, "random", "in_gemm"),
                                                           (3, 16, "random", "row_pass"), (3, 16, "random", "unfolded")])
def test_tapnext_stream(n_blocks, n_frames, affine, norms):
    """Config 3 as BASELINE states it (12 blocks, 16 frames, state carried) and a random-affine stack, with the
    norms folded into the GEMMs and their row factors merged in those GEMMs' epilogues (default), folded with a
    row-moment pass before each, and as separate norm passes: every frame within the per-token tolerance."""
    device_status(clear=True)
    W = wg.tapnext_weights(CFG, seed=8, n_blocks=n_blocks, affine=affine)
    frames, queries = wg.tapnext_inputs(CFG, n_frames, seed=2)
    eng = TapNextStep(W, CFG, device="cuda", **NORMS[norms])
    state = None
    for f in range(n_frames):
        ref, state = tapnext_ref.step(frames[f], queries[f], W, CFG, state, n_blocks)
        out = eng.step(torch.from_numpy(frames[f]).cuda(), torch.from_numpy(queries[f]).cuda())
        assert_tokens_close(out.float().cpu(), ref, what=f"frame {f}")
    assert device_status(clear=True) == 0


def test_rglru_gate_against_reference_ssm_ref():
    """The device RG-LRU (gate GEMM + recurrence, the path every TAPNext block runs) against the reference's own
    ssm_ref (tapnext/npu/pack8.py:252-279) with 12 heads of block-diagonal gates and identity conv taps
    (tests/golden/rglru_ref_cases.npz): a first frame and the next one, state carried on the device, every row
    of h within the same 1e-2 as the CPU restatement (ssm_ref rounds its intermediates to bf16), and x += h."""
    from helpers import rglru_case, RGLRU_TOL
    from strix_halo_maxx_b200.tapnext import RgLruGate
    device_status(clear=True)
    W, frames = rglru_case()
    R, C = frames[0][0].shape
    G = torch.empty(R, 2 * C, dtype=torch.float32, device="cuda")
    gate = RgLruGate(W["gx_w"], W["gx_b"], W["ga_w"], W["ga_b"], W["a_param"], 8.0, torch.device("cuda"), G)
    state = torch.zeros(R, C, dtype=torch.float32, device="cuda")
    for f, (x, h_ref) in enumerate(frames):
        t = torch.from_numpy(x).cuda().to(torch.bfloat16)  # the fixture's x is bf16-valued: exact
        xres = torch.zeros(R, C, dtype=torch.float32, device="cuda")
        gate(t, state, xres, first=(f == 0))
        ref = torch.from_numpy(h_ref)
        rel = float(((state.cpu() - ref).norm(dim=-1) / ref.norm(dim=-1)).max())
        assert rel < RGLRU_TOL, f"frame {f}: max per-row rel {rel:.3e}"
        assert torch.equal(xres, state)
    assert device_status(clear=True) == 0


def test_tapnext_graph_replay_matches_eager():
    """Frames after the first replay one captured CUDA graph: bit-identical to launching eagerly."""
    W = wg.tapnext_weights(CFG, seed=8, n_blocks=3, affine="random")
    frames, queries = wg.tapnext_inputs(CFG, 5, seed=4)
    eg, ee = TapNextStep(W, CFG, device="cuda"), TapNextStep(W, CFG, device="cuda", graphs=False)
    for f in range(5):
        fr, q = torch.from_numpy(frames[f]).cuda(), torch.from_numpy(queries[f]).cuda()
        assert torch.equal(eg.step(fr, q), ee.step(fr, q)), f"frame {f}"
    assert eg._graph is not None
