"""The text decoder on the GPU against the CPU oracle (oracle/text_ref.py, pinned to the reference's own
_text_layers / _query): its rotary / cache and causal attention kernels, then image prefill + question."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from strix_halo_maxx_b200.config import TEXT
from strix_halo_maxx_b200 import ops, weights as wg
from strix_halo_maxx_b200.text import TextDecoder, rope_tables
from strix_halo_maxx_b200._lib import device_status
from oracle import text_ref as R
from helpers import assert_tokens_close, rel

BF = torch.bfloat16
DEV = "cuda"


@pytest.mark.parametrize("n,pos0", [(730, 0), (32, 730), (5, 100)])
def test_rope_qkv_matches_oracle_and_fills_the_cache(n, pos0):
    H, hd, ctx = TEXT.heads, TEXT.head_dim, TEXT.ctx
    g = torch.Generator().manual_seed(n)
    qkv = torch.randn(n, 3 * H * hd, generator=g).to(BF)
    cos, sin = rope_tables(TEXT, DEV)
    q = torch.empty(H, n, hd, dtype=BF, device=DEV)
    kc = torch.zeros(H, ctx, hd, dtype=BF, device=DEV)
    vc = torch.zeros(H, ctx, hd, dtype=BF, device=DEV)
    ops.rope_qkv(qkv.to(DEV), pos0, cos, sin, q, kc, vc)
    c, s = R.rope_angles(TEXT, pos0, n)
    qr, kr, vr = [t.float().view(1, n, H, hd).transpose(1, 2) for t in qkv.split(H * hd, dim=-1)]
    q_ref = R.rope(qr, c, s, TEXT.rot)[0]
    k_ref = R.rope(kr, c, s, TEXT.rot)[0]
    assert torch.allclose(q.float().cpu(), q_ref, rtol=1e-2, atol=1e-2)
    assert torch.allclose(kc[:, pos0:pos0 + n].float().cpu(), k_ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(vc[:, pos0:pos0 + n].cpu(), vr[0].to(BF))
    assert kc[:, :pos0].abs().sum() == 0 and kc[:, pos0 + n:].abs().sum() == 0


@pytest.mark.parametrize("n,pos0", [(32, 730), (7, 0), (1, 2000)])
def test_attn_causal_matches_masked_sdpa(n, pos0):
    H, hd = 32, 64
    ctx = pos0 + n + 3
    g = torch.Generator().manual_seed(7 + n)
    q = torch.randn(H, n, hd, generator=g).to(BF)
    kc = torch.randn(H, ctx, hd, generator=g).to(BF)
    vc = torch.randn(H, ctx, hd, generator=g).to(BF)
    out = torch.empty(n, H * hd, dtype=BF, device=DEV)
    ops.attn_causal(q.to(DEV), kc.to(DEV), vc.to(DEV), pos0, out)
    mask = torch.arange(pos0 + n)[None, :] <= (pos0 + torch.arange(n))[:, None]
    ref = F.scaled_dot_product_attention(q.float()[None], kc[:, :pos0 + n].float()[None], vc[:, :pos0 + n].float()[None],
                                         attn_mask=mask[None, None])[0].transpose(0, 1).reshape(n, H * hd)
    assert rel(out.float().cpu(), ref) < 1e-2


@pytest.mark.parametrize("n_layers,affine", [(2, "random"), (24, "zero")])
def test_text_decoder_prefill_and_question(n_layers, affine):
    device_status(clear=True)
    W = wg.text_weights(TEXT, seed=3, n_layers=n_layers, affine=affine)
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    x_ref, cache = R.encode(emb, bos, W, TEXT, n_layers=n_layers)
    logits_ref = R.query(ids, last, W, TEXT, cache, n_layers=n_layers)
    dec = TextDecoder(W, TEXT, device=DEV)
    x = dec.encode(torch.from_numpy(emb).to(DEV), bos)
    assert_tokens_close(x.float().cpu(), x_ref, what="prefix hidden states")
    logits = dec.query(torch.from_numpy(ids).to(DEV), last).float().cpu()
    assert rel(logits, logits_ref) < 3e-2, (logits, logits_ref)
    assert device_status(clear=True) == 0


def test_text_question_graph_replay_matches_eager():
    """Questions after the first replay one captured graph (ids and the last-token index in static device
    buffers): logits bit-identical to the eager path for different questions."""
    W = wg.text_weights(TEXT, seed=3, n_layers=2, affine="random")
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    dg, de = TextDecoder(W, TEXT, device=DEV), TextDecoder(W, TEXT, device=DEV, graphs=False)
    e = torch.from_numpy(emb).to(DEV)
    dg.encode(e, bos)
    de.encode(e, bos)
    g = torch.Generator().manual_seed(1)
    for r in range(3):
        q = torch.from_numpy(ids).to(DEV) if r == 0 else torch.randint(1, TEXT.vocab, (TEXT.q_len,), generator=g).to(DEV)
        lst = last if r == 0 else TEXT.q_len - 1 - 3 * r
        assert torch.equal(dg.query(q, lst), de.query(q, lst)), f"question {r}"
    assert dg._qgraph is not None


def test_text_prefill_graph_replay_matches_eager():
    """Image prefills after the first replay one captured graph (features and bos in static buffers):
    hidden states bit-identical to the eager path, and the question after it too."""
    W = wg.text_weights(TEXT, seed=3, n_layers=2, affine="random")
    emb, bos, ids, last = wg.text_inputs(TEXT, seed=5)
    dg, de = TextDecoder(W, TEXT, device=DEV), TextDecoder(W, TEXT, device=DEV, graphs=False)
    g = torch.Generator().manual_seed(2)
    for r in range(3):
        e = torch.from_numpy(emb).to(DEV) if r == 0 else torch.randn(TEXT.prefix - 1, TEXT.dim, generator=g).to(DEV)
        b = bos if r == 0 else r
        assert torch.equal(dg.encode(e, b), de.encode(e, b)), f"prefill {r}"
        q = torch.from_numpy(ids).to(DEV)
        assert torch.equal(dg.query(q, last), de.query(q, last)), f"question after prefill {r}"
    assert dg._egraph is not None
