"""The moondream2 SigLIP-style vision tower on B200: the hot path FastMD2._vision computes
(moondream/gpu/md2fast.py:147-160), re-planned for sm_100a.

Per block (md2fast.py:153-157), with the residual stream x kept in fp32 in HBM and each LayerNorm folded
into the GEMM that follows it (default, fold_ln=True):
    mom = (mean, rstd) of x rows   vt_row_moments  from the chunk statistics the last residual GEMM wrote
    qkv = LN1(x) . Wqkv^T + b      vt_gemm_fused  A = bf16 x, W * gamma1; epilogue applies
                                                  rstd * (acc - mean * rowsum(W')) + b + W beta1 and
                                                  writes attention tiles
    a   = attention(qkv)           vt_attn_tiles_fwd  tcgen05, S / O in TMEM, d 72 -> 80
    x   = x + a . Wo^T + b         vt_gemm_fused  residual epilogue, fp32 in place, also writes the bf16
                                                  copy of x and its per-32-column (mean, M2) statistics
    f   = gelu(LN2(x) . W1^T + b)  vt_gemm_fused  folded LN2 (after vt_row_moments) + GELU-tanh epilogue
    x   = x + f . W2^T + b         vt_gemm_fused  residual epilogue + bf16 copy + statistics
With fold_ln=False the two LayerNorms run as vt_layernorm passes (fp32 x -> bf16) before qkv / fc1.
Patch embed (md2fast.py:148-150): vt_im2col (normalise + (c, py, px) patch order, K 588 in a 592 pitch)
then vt_gemm_ex with the positional embedding as a row-periodic (period 729) fp32 addend.
post-LN (md2fast.py:158) -> bf16 features; projection (md2fast.py:159-160) -> two GEMMs.

Crops are independent through every GEMM, so a batch of B crops is one M = 729*B GEMM (tiles span crop
boundaries); attention stays per crop (grid over crops x heads).  Buffers are allocated once per batch
size and reused, so a forward allocates nothing and can be captured in a CUDA graph.
"""
import torch

from .config import TOWER, TowerConfig
from . import ops
from .ops import BF16, _pad8

F32 = torch.float32


def _dev_mat(a, dev):
    """fp32 [N, K] -> bf16 [N, pad8(K)] on device (pad columns zero); returns (buffer, pitch)."""
    t = torch.as_tensor(a)
    N, K = t.shape
    buf = torch.zeros(N, _pad8(K), dtype=BF16, device=dev)
    buf[:, :K] = t.to(dev, BF16)
    return buf, buf.stride(0)


def _dev_vec(a, dev):
    return torch.as_tensor(a).to(dev, F32).contiguous()


class _Bufs:
    def __init__(self, cfg: TowerConfig, B, dev):
        M = B * cfg.ntok
        W = cfg.width
        self.B, self.M = B, M
        self.a_pe = torch.zeros(M, _pad8(cfg.patch_k), dtype=BF16, device=dev)
        self.x = torch.empty(M, W, dtype=F32, device=dev)
        self.h = torch.empty(M, W, dtype=BF16, device=dev)
        self.tiles = ops.attn_tiles(B, cfg.ntok, cfg.heads, cfg.head_dim, dev)
        self.xb = torch.empty(M, W, dtype=BF16, device=dev)                 # bf16 copy of x (folded LN)
        self.stats = torch.empty(M, W // 32, 2, dtype=F32, device=dev)     # per-32-column (mean, M2) of x
        self.moments = torch.empty(M, 2, dtype=F32, device=dev)            # (mean, rstd) per row of x
        self.a = torch.empty(M, W, dtype=BF16, device=dev)
        self.f = torch.empty(M, _pad8(cfg.ff), dtype=BF16, device=dev)
        self.feats = torch.empty(M, W, dtype=BF16, device=dev)


class VisionTower:
    """Patch-embed + n_blocks pre-LN blocks + post-LN (+ projection MLP) with device-resident weights.

    weights: dict as produced by strix_halo_maxx_b200.weights.tower_weights (fp32 numpy or torch).
    eps: LayerNorm eps (the benchmark configs use 1e-6; the reference's _ln uses torch's 1e-5).
    """

    def __init__(self, weights, cfg: TowerConfig = TOWER, eps=None, device="cuda", projection=True, fold_ln=True):
        self.cfg = cfg
        self.fold_ln = fold_ln
        self.eps = cfg.eps if eps is None else float(eps)
        dev = self.dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        W = weights
        self.n_blocks = sum(1 for k in W if k.endswith(".qkv_w"))
        self.pe_w, self.pe_ld = _dev_mat(W["patch_w"], dev)
        self.pe_b = _dev_vec(W["patch_b"], dev)
        self.pos = _dev_vec(W["pos_emb"], dev).reshape(cfg.ntok, cfg.width)
        self.blocks = []
        for i in range(self.n_blocks):
            p = f"blocks.{i}."
            blk = {}
            for n in ("qkv", "proj", "fc1", "fc2"):
                blk[n + "_w"], blk[n + "_ld"] = _dev_mat(W[p + n + "_w"], dev)
                blk[n + "_b"] = _dev_vec(W[p + n + "_b"], dev)
            for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b"):
                blk[n] = _dev_vec(W[p + n], dev)
            if fold_ln:   # LN1 into qkv, LN2 into fc1: W * gamma, rowsum, b + W beta
                for n, ln in (("qkv", "ln1"), ("fc1", "ln2")):
                    wf, c, bf = ops.fold_layernorm(W[p + n + "_w"], W[p + n + "_b"], W[p + ln + "_w"], W[p + ln + "_b"])
                    blk[n + "_wf"], blk[n + "_ldf"] = _dev_mat(wf, dev)
                    blk[n + "_c"] = _dev_vec(c, dev)
                    blk[n + "_bf"] = _dev_vec(bf, dev)
            self.blocks.append(blk)
        self.post_w = _dev_vec(W["post_ln_w"], dev)
        self.post_b = _dev_vec(W["post_ln_b"], dev)
        self.has_projection = projection and "proj_fc1_w" in W
        if self.has_projection:
            # fc1 over cat([x, x]) ([proj_hidden, 2 width]), or with its two K-halves already summed
            # ([proj_hidden, width]) as FastMD2(fold_proj=True) builds it (md2fast.py:97-101)
            self.p1_k = int(W["proj_fc1_w"].shape[1])
            assert self.p1_k in (cfg.width, 2 * cfg.width), "proj_fc1 must take width or 2 * width inputs"
            self.p1_w, self.p1_ld = _dev_mat(W["proj_fc1_w"], dev)
            self.p1_b = _dev_vec(W["proj_fc1_b"], dev)
            self.p2_w, self.p2_ld = _dev_mat(W["proj_fc2_w"], dev)
            self.p2_b = _dev_vec(W["proj_fc2_b"], dev)
        self._bufs = {}
        self._proj_bufs = {}
        self.op_timer = None   # optional callable(name, flops) -> context manager (bench.py times every launch)

    # ------------------------------------------------------------------ buffers
    def buffers(self, B):
        if B not in self._bufs:
            self._bufs[B] = _Bufs(self.cfg, B, self.dev)
        return self._bufs[B]

    def _op(self, name, flops, fn, *args, **kw):
        if self.op_timer is None:
            return fn(*args, **kw)
        with self.op_timer(name, flops):
            return fn(*args, **kw)

    def _gemm(self, name, x2, w, ldw, K, N, bias, **kw):
        return self._op("gemm_" + name, 2 * x2.shape[0] * K * N, ops.gemm, x2, w, ldw, K, N, bias, **kw)

    # ------------------------------------------------------------------ forward
    def forward(self, pix, out=None, n_blocks=None):
        """pix: [B, 3, 378, 378] fp32 / bf16 (values in [-1, 1]) or uint8 [B, 378, 378, 3] on the device.
        Returns post-LN features [B, 729, width] bf16 (written into `out` when given)."""
        cfg = self.cfg
        B = pix.shape[0]
        nb = self.n_blocks if n_blocks is None else n_blocks
        if B == 0:
            return torch.empty(0, cfg.ntok, cfg.width, dtype=BF16, device=self.dev) if out is None else out
        bf = self.buffers(B)
        T, Wd, H, D = cfg.ntok, cfg.width, cfg.heads, cfg.head_dim
        self._op("im2col", 0, ops.im2col, pix, cfg.patch, bf.a_pe)
        fold = dict(out2=bf.xb, stats_out=bf.stats) if self.fold_ln else {}
        self._gemm("patch", bf.a_pe[:, :cfg.patch_k], self.pe_w, self.pe_ld, cfg.patch_k, Wd, self.pe_b,
                   res=self.pos, res_period=T, out=bf.x, **fold)
        self._blocks(bf, B, nb)
        dst = bf.feats if out is None else out.reshape(B * T, Wd)
        self._op("layernorm", 0, ops.layer_norm, bf.x, self.post_w, self.post_b, self.eps, out=dst)
        return dst.reshape(B, T, Wd)

    def run_blocks(self, x, n_blocks=None):
        """Config 0: the encoder blocks alone on a residual input x [B, 729, width] fp32 (device);
        returns the fp32 residual stream after the last block (a view of an internal buffer)."""
        B = x.shape[0]
        bf = self.buffers(B)
        bf.x.copy_(x.reshape(bf.M, self.cfg.width))
        if self.fold_ln:
            self._op("rowstats", 0, ops.row_stats, bf.x, bf.stats, bf.xb)
        self._blocks(bf, B, self.n_blocks if n_blocks is None else n_blocks)
        return bf.x.reshape(B, self.cfg.ntok, self.cfg.width)

    def _blocks(self, bf, B, nb):
        cfg = self.cfg
        T, Wd, H, D = cfg.ntok, cfg.width, cfg.heads, cfg.head_dim
        if self.fold_ln:
            fold = dict(out2=bf.xb, stats_out=bf.stats)
            for blk in self.blocks[:nb]:
                self._op("row_moments", 0, ops.row_moments, bf.stats, self.eps, bf.moments)
                self._gemm("qkv", bf.xb, blk["qkv_wf"], blk["qkv_ldf"], Wd, cfg.qkv_dim, blk["qkv_bf"], out=bf.tiles,
                           ln=(bf.moments, blk["qkv_c"]), tiles=(T, H, D))
                self._op("attention", 4 * B * T * T * D * H, ops.attention_tiles, bf.tiles, B, T, H, D, bf.a)
                self._gemm("proj", bf.a, blk["proj_w"], blk["proj_ld"], Wd, Wd, blk["proj_b"], res=bf.x, out=bf.x,
                           **fold)
                self._op("row_moments", 0, ops.row_moments, bf.stats, self.eps, bf.moments)
                self._gemm("fc1", bf.xb, blk["fc1_wf"], blk["fc1_ldf"], Wd, cfg.ff, blk["fc1_bf"], gelu=True,
                           out=bf.f[:, :cfg.ff], ln=(bf.moments, blk["fc1_c"]))
                self._gemm("fc2", bf.f[:, :cfg.ff], blk["fc2_w"], blk["fc2_ld"], cfg.ff, Wd, blk["fc2_b"], res=bf.x,
                           out=bf.x, **fold)
            return
        for blk in self.blocks[:nb]:
            self._op("layernorm", 0, ops.layer_norm, bf.x, blk["ln1_w"], blk["ln1_b"], self.eps, out=bf.h)
            self._gemm("qkv", bf.h, blk["qkv_w"], blk["qkv_ld"], Wd, cfg.qkv_dim, blk["qkv_b"], out=bf.tiles,
                       tiles=(T, H, D))
            self._op("attention", 4 * B * T * T * D * H, ops.attention_tiles, bf.tiles, B, T, H, D, bf.a)
            self._gemm("proj", bf.a, blk["proj_w"], blk["proj_ld"], Wd, Wd, blk["proj_b"], res=bf.x, out=bf.x)
            self._op("layernorm", 0, ops.layer_norm, bf.x, blk["ln2_w"], blk["ln2_b"], self.eps, out=bf.h)
            self._gemm("fc1", bf.h, blk["fc1_w"], blk["fc1_ld"], Wd, cfg.ff, blk["fc1_b"], gelu=True,
                       out=bf.f[:, :cfg.ff])
            self._gemm("fc2", bf.f[:, :cfg.ff], blk["fc2_w"], blk["fc2_ld"], cfg.ff, Wd, blk["fc2_b"], res=bf.x,
                       out=bf.x)

    def project(self, feats2):
        """Projection MLP (md2fast.py:159-160): [T, 2*width] bf16 ([T, width] for a folded fc1) ->
        [T, proj_out] bf16."""
        assert self.has_projection and feats2.shape[-1] == self.p1_k
        cfg = self.cfg
        T = feats2.shape[0]
        if T not in self._proj_bufs:
            self._proj_bufs[T] = (torch.empty(T, cfg.proj_hidden, dtype=BF16, device=self.dev),
                                  torch.empty(T, cfg.proj_out, dtype=BF16, device=self.dev))
        hid, out = self._proj_bufs[T]
        x2 = ops.as_gemm_operand(feats2)
        self._gemm("proj_fc1", x2, self.p1_w, self.p1_ld, self.p1_k, cfg.proj_hidden, self.p1_b, gelu=True, out=hid)
        self._gemm("proj_fc2", hid, self.p2_w, self.p2_ld, cfg.proj_hidden, cfg.proj_out, self.p2_b, out=out)
        return out

    def vision_u8(self, img_u8):
        """The whole of FastMD2._vision: uint8 [378, 378, 3] -> [729, proj_out] bf16 (one crop: cat([x, x]),
        or x itself when fc1 is folded, md2fast.py:159)."""
        f = self.forward(img_u8.reshape(1, *img_u8.shape[-3:]))
        if self.p1_k == self.cfg.width:
            return self.project(f[0])
        cat = torch.empty(self.cfg.ntok, 2 * self.cfg.width, dtype=BF16, device=self.dev)
        cat[:, :self.cfg.width] = f[0]
        cat[:, self.cfg.width:] = f[0]
        return self.project(cat)

    def frame(self, crops):
        """Config 2: 1 global + n local crops [1+n, 3, 378, 378] -> projected frame features [729, proj_out]."""
        return self.frame_from_features(self.forward(crops))

    def frame_from_features(self, feats):
        """The frame's tail: crop features [1+n, 729, width] bf16 (global crop first) -> combined [729, 2 width]
        (global features, then the per-token mean of the local crops) -> projection [729, proj_out]."""
        assert self.p1_k == 2 * self.cfg.width, "the multi-crop frame needs the unfolded [hidden, 2 width] fc1"
        comb = torch.empty(self.cfg.ntok, 2 * self.cfg.width, dtype=BF16, device=self.dev)
        ops.crop_combine(feats, comb)
        return self.project(comb)


# ---------------------------------------------------------------------- drop-in for FastMD2._vision
def _lin_weight(lin):
    """(weight [N, K], bias [N]) of a reference `Lin` (md2fast.py:33-40) or a VtLin."""
    if isinstance(lin, ops.VtLin):
        return lin.w.float().cpu(), (None if lin.b is None else lin.b.float().cpu())
    return lin.w.float().cpu(), (None if lin.b is None else lin.b.float().cpu())


def weights_from_fastmd2(m):
    """The vision weights of a FastMD2 instance (md2fast.py:89-103) as a tower_weights-style dict."""
    W = {}

    def put(name, lin):
        w, b = _lin_weight(lin)
        W[name + "_w"] = w
        W[name + "_b"] = torch.zeros(w.shape[0]) if b is None else b

    put("patch", m.patch_emb)
    W["pos_emb"] = m.pos_emb.float().cpu().reshape(-1, m.pos_emb.shape[-1])
    for i, b in enumerate(m.vblocks):
        p = f"blocks.{i}."
        for n in ("qkv", "proj", "fc1", "fc2"):
            put(p + n, b[n])
        W[p + "ln1_w"], W[p + "ln1_b"] = (t.float().cpu() for t in b["ln1"])
        W[p + "ln2_w"], W[p + "ln2_b"] = (t.float().cpu() for t in b["ln2"])
    W["post_ln_w"], W["post_ln_b"] = (t.float().cpu() for t in m.post_ln)
    # with fold_proj=True proj_fc1 holds the summed K-halves [hidden, width]; VisionTower takes either shape
    put("proj_fc1", m.proj_fc1)
    put("proj_fc2", m.proj_fc2)
    return W


def vt_vision(self, img_u8):
    """Drop-in for FastMD2._vision (md2fast.py:147-160): uint8 [378, 378, 3] -> [729, 2048] bf16.
    The tower is built from the instance's weights on first use and cached on it; LayerNorm eps is
    torch's default 1e-5, the value the reference's _ln uses (md2fast.py:43-44)."""
    t = getattr(self, "_vt_tower", None)
    if t is None:
        dev = img_u8.device if img_u8.is_cuda else torch.device("cuda")
        t = self._vt_tower = VisionTower(weights_from_fastmd2(self), TOWER, eps=1e-5, device=dev)
    return t.vision_u8(img_u8.to(t.dev))


def enable(fastmd2_cls):
    """Swap the B200 tower into a FastMD2 class, the way the reference's bf16emu.enable swaps its
    emulation in (moondream/gpu/bf16emu.py:148-153).  Returns the previous _vision."""
    prev = fastmd2_cls._vision
    fastmd2_cls._vision = vt_vision
    return prev
