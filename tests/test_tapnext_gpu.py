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


@pytest.mark.parametrize("n_blocks,n_frames,affine", [(12, 3, "zero"), (3, 16, "random")])
def test_tapnext_stream(n_blocks, n_frames, affine):
    device_status(clear=True)
    W = wg.tapnext_weights(CFG, seed=8, n_blocks=n_blocks, affine=affine)
    frames, queries = wg.tapnext_inputs(CFG, n_frames, seed=2)
    eng = TapNextStep(W, CFG, device="cuda")
    state = None
    for f in range(n_frames):
        ref, state = tapnext_ref.step(frames[f], queries[f], W, CFG, state, n_blocks)
        out = eng.step(torch.from_numpy(frames[f]).cuda(), torch.from_numpy(queries[f]).cuda())
        assert_tokens_close(out.float().cpu(), ref, what=f"frame {f}")
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
