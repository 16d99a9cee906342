"""TAPNext-style per-frame streaming step on B200: 8x8 patch conv of a 256x256 frame
(1024 tokens) + position embedding, 256 point-query tokens appended (token layout of
tapnext/npu/step8.py:251-267), 12 x [pre-LN ViT block (12 heads x 64, MLP 3072 GELU) + residual temporal block (RMSNorm pre-norm, RG-LRU,
+ x; the shape of the reference's recurrent block, step8.py:474-480)]
and the encoder LayerNorm.  The RG-LRU (tapnext/npu/r9/cpuemu.py:33-47) keeps one fp32 state
[1280, 768] per block, carried across frames in device memory owned by this object; reset() starts a
new video.

Per block the kernels are the tower's (vt_gemm_qkv_tiles + vt_attn_tiles_fwd with d = 64, vt_gemm_fused) plus
the RG-LRU.  With fold_ln=True (default) every norm is folded into the GEMM after it, as in the tower:
    (mean, rstd) of x                   from the chunk statistics the last writer of x left (see below)
    qkv = LN1(x) . Wqkv^T + b           folded LN1 (A = bf16 copy of x, W * gamma1), tile scatter
    x  += attn . Wo^T + b               residual epilogue + bf16 copy + chunk statistics
    f   = gelu(LN2(x) . W1^T + b)       folded LN2
    x  += f . W2^T + b                  residual epilogue + bf16 copy + chunk statistics
    (0, rstd) of x                      the same, RMSNorm
    G   = RMSNorm(x) . [Wx; Wa]^T + b   folded RMSNorm (W * gamma), N = 1536, fp32 out
    vt_rglru_fold                       t = bf16(x rstd gamma), gates, recurrence, state, x += h, and the bf16 copy
                                        and chunk statistics of the new x for the next block's LN1
By default (rows_in_gemm=True) no row-moment pass runs: each folded GEMM merges the chunk statistics into its
rows' (mean, rstd) in its own epilogue (vt_gemm_fused_lnstats), and the gate GEMM also stores the RMS factors
that vt_rglru_fold reads; rows_in_gemm=False keeps the vt_row_moments / vt_row_rms passes.
With fold_ln=False the norms run as vt_layernorm / vt_rmsnorm passes and the gate step as RgLruGate.
"""
import torch

from .config import TAPNEXT, TapNextConfig
from . import ops
from .ops import BF16, _pad8
from .tower import _dev_mat, _dev_vec

F32 = torch.float32


class RgLruGate:
    """The RG-LRU temporal update of one block (tapnext/npu/r9/cpuemu.py:33-47) on the device:
    G = t . [Wx; Wa]^T + [bx; ba] (one GEMM, fp32 out), then vt_rglru: gates, recurrence, state and x += h.
    gx_w / ga_w are [768 out, 768 in] (dense; the reference's block-diagonal gates are the special case that
    tests/golden/rglru_ref_cases.npz pins), a_param [768] (kept on the device as softplus(a_param), computed once in
    float64 and rounded to fp32); G an fp32 [rows >= M, 2 * 768] buffer."""

    def __init__(self, gx_w, gx_b, ga_w, ga_b, a_param, c, dev, G):
        g = torch.cat([torch.as_tensor(gx_w), torch.as_tensor(ga_w)], 0)
        self.W = g.shape[1]
        self.w, self.ld = _dev_mat(g, dev)
        self.b = _dev_vec(torch.cat([torch.as_tensor(gx_b), torch.as_tensor(ga_b)]), dev)
        self.softplus_a = _dev_vec(torch.nn.functional.softplus(torch.as_tensor(a_param).double()).float(), dev)
        self.c = c
        self.G = G  # fp32 [rows, 2 W] scratch for the gate pre-activations, shareable between blocks

    def __call__(self, t, state, x, first):
        """t [M, W] bf16 (the normed input), state [M, W] fp32 and x [M, W] fp32 updated in place."""
        ops.gemm(t, self.w, self.ld, self.W, 2 * self.W, self.b, out=self.G[:t.shape[0]])
        ops.rglru(self.G[:t.shape[0]], self.softplus_a, t, state, x, self.c, first)


class TapNextStep:
    def __init__(self, weights, cfg: TapNextConfig = TAPNEXT, device="cuda", graphs=True, fold_ln=True,
                 rows_in_gemm=True):
        self.cfg = cfg
        self.fold_ln = fold_ln
        self.rows_in_gemm = rows_in_gemm
        self.use_graphs = graphs
        self._graph = None
        self._frame_in = self._q_in = None
        dev = self.dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        W = weights
        self.n_blocks = sum(1 for k in W if k.endswith(".qkv_w"))
        self.pe_w, self.pe_ld = _dev_mat(W["patch_w"], dev)
        self.pe_b = _dev_vec(W["patch_b"], dev)
        self.pos = _dev_vec(W["pos_emb"], dev).reshape(cfg.n_img_tok, cfg.width)
        self.blocks = []
        self.G = torch.empty(cfg.ntok, 2 * cfg.width, dtype=F32, device=dev)
        for i in range(self.n_blocks):
            p = f"blocks.{i}."
            blk = {}
            for n in ("qkv", "proj", "fc1", "fc2"):
                blk[n + "_w"], blk[n + "_ld"] = _dev_mat(W[p + n + "_w"], dev)
                blk[n + "_b"] = _dev_vec(W[p + n + "_b"], dev)
            blk["lru"] = RgLruGate(W[p + "gx_w"], W[p + "gx_b"], W[p + "ga_w"], W[p + "ga_b"], W[p + "a_param"],
                                   cfg.lru_c, dev, self.G)
            for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "rms_w"):
                blk[n] = _dev_vec(W[p + n], dev)
            if fold_ln:   # LN1 into qkv, LN2 into fc1 (W * gamma, rowsum, b + W beta); RMSNorm gamma into the gates
                for n, ln in (("qkv", "ln1"), ("fc1", "ln2")):
                    wf, c, bf = ops.fold_layernorm(W[p + n + "_w"], W[p + n + "_b"], W[p + ln + "_w"], W[p + ln + "_b"])
                    blk[n + "_wf"], blk[n + "_ldf"] = _dev_mat(wf, dev)
                    blk[n + "_c"] = _dev_vec(c, dev)
                    blk[n + "_bf"] = _dev_vec(bf, dev)
                g = torch.cat([torch.as_tensor(W[p + "gx_w"]), torch.as_tensor(W[p + "ga_w"])], 0).float()
                gb = torch.cat([torch.as_tensor(W[p + "gx_b"]), torch.as_tensor(W[p + "ga_b"])]).float()
                wf, c, _ = ops.fold_layernorm(g, gb, W[p + "rms_w"], torch.zeros(g.shape[1]))
                blk["gate_wf"], blk["gate_ldf"] = _dev_mat(wf, dev)
                blk["gate_c"] = _dev_vec(c, dev)
                blk["gate_b"] = _dev_vec(gb, dev)
            self.blocks.append(blk)
        self.fin_w = _dev_vec(W["final_ln_w"], dev)
        self.fin_b = _dev_vec(W["final_ln_b"], dev)
        T, Wd = cfg.ntok, cfg.width
        self.a_pe = torch.zeros(cfg.n_img_tok, _pad8(cfg.patch_k), dtype=BF16, device=dev)
        self.x = torch.empty(T, Wd, dtype=F32, device=dev)
        self.t = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.h = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.tiles = ops.attn_tiles(1, T, cfg.heads, cfg.head_dim, dev)
        self.a = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.f = torch.empty(T, _pad8(cfg.ff), dtype=BF16, device=dev)
        self.state = torch.zeros(self.n_blocks, T, Wd, dtype=F32, device=dev)
        if fold_ln:
            self.xb = torch.empty(T, Wd, dtype=BF16, device=dev)                  # bf16 copy of x
            self.stats = torch.empty(T, Wd // 32, 2, dtype=F32, device=dev)      # per-32-column (mean, M2) of x
            self.mom = torch.empty(T, 2, dtype=F32, device=dev)                  # (mean | 0, rstd) per row
        self.out = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.first = True

    def reset(self):
        self.first = True

    def step(self, frame, queries):
        """frame [3, 256, 256] fp32/bf16 in [-1, 1], queries [256, 768] fp32 (device) -> [1280, 768] bf16.
        With graphs=True every frame after a video's first replays one CUDA graph of the whole step (captured
        the first time), after copying frame and queries into static input buffers: same kernels, same
        buffers, bit-identical results, none of the ~110 launches' host time per frame."""
        if not self.use_graphs or self.first:
            self._run(frame, queries, self.first)
        else:
            if self._frame_in is None:
                self._frame_in, self._q_in = torch.empty_like(frame), torch.empty_like(queries)
            self._frame_in.copy_(frame)
            self._q_in.copy_(queries)
            if self._graph is None:
                self._graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self._graph):
                    self._run(self._frame_in, self._q_in, False)
            self._graph.replay()
        self.first = False
        return self.out

    def _run(self, frame, queries, first):
        cfg = self.cfg
        T, Wd, NI = cfg.ntok, cfg.width, cfg.n_img_tok
        ops.im2col(frame.reshape(1, *frame.shape[-3:]), cfg.patch, self.a_pe)
        ops.gemm(self.a_pe[:, :cfg.patch_k], self.pe_w, self.pe_ld, cfg.patch_k, Wd, self.pe_b,
                 res=self.pos, res_period=NI, out=self.x[:NI])
        self.x[NI:].copy_(queries)
        if self.fold_ln:
            self._blocks_folded(first)
            ops.layer_norm(self.x, self.fin_w, self.fin_b, cfg.eps, out=self.out)
            return
        for i, blk in enumerate(self.blocks):
            ops.layer_norm(self.x, blk["ln1_w"], blk["ln1_b"], cfg.eps, out=self.h)
            ops.gemm_qkv_tiles(self.h, blk["qkv_w"], blk["qkv_ld"], Wd, blk["qkv_b"], self.tiles, T, cfg.heads,
                               cfg.head_dim)
            ops.attention_tiles(self.tiles, 1, T, cfg.heads, cfg.head_dim, self.a)
            ops.gemm(self.a, blk["proj_w"], blk["proj_ld"], Wd, Wd, blk["proj_b"], res=self.x, out=self.x)
            ops.layer_norm(self.x, blk["ln2_w"], blk["ln2_b"], cfg.eps, out=self.h)
            ops.gemm(self.h, blk["fc1_w"], blk["fc1_ld"], Wd, cfg.ff, blk["fc1_b"], gelu=True, out=self.f[:, :cfg.ff])
            ops.gemm(self.f[:, :cfg.ff], blk["fc2_w"], blk["fc2_ld"], cfg.ff, Wd, blk["fc2_b"], res=self.x, out=self.x)
            ops.rms_norm(self.x, blk["rms_w"], cfg.eps, out=self.t)
            blk["lru"](self.t, self.state[i], self.x, first)
        ops.layer_norm(self.x, self.fin_w, self.fin_b, cfg.eps, out=self.out)

    def _norm(self, c, rms, keep=False):
        """gemm keyword arguments of a norm of x folded into the GEMM that follows (c = its rowsum vector):
        the row factors merged from x's chunk statistics in that GEMM's epilogue (stored in self.mom when keep),
        or, with rows_in_gemm=False, computed into self.mom by a row-moment pass launched here."""
        cfg = self.cfg
        if self.rows_in_gemm:
            return dict(ln_rows=(self.stats, cfg.eps, rms, c, self.mom if keep else None))
        (ops.row_rms if rms else ops.row_moments)(self.stats, cfg.eps, self.mom)
        return dict(ln=(self.mom, c))

    def _blocks_folded(self, first):
        cfg = self.cfg
        T, Wd = cfg.ntok, cfg.width
        fold = dict(out2=self.xb, stats_out=self.stats)
        ops.row_stats(self.x, self.stats, self.xb)
        for i, blk in enumerate(self.blocks):
            ops.gemm(self.xb, blk["qkv_wf"], blk["qkv_ldf"], Wd, 3 * Wd, blk["qkv_bf"], out=self.tiles,
                     tiles=(T, cfg.heads, cfg.head_dim), **self._norm(blk["qkv_c"], False))
            ops.attention_tiles(self.tiles, 1, T, cfg.heads, cfg.head_dim, self.a)
            ops.gemm(self.a, blk["proj_w"], blk["proj_ld"], Wd, Wd, blk["proj_b"], res=self.x, out=self.x, **fold)
            ops.gemm(self.xb, blk["fc1_wf"], blk["fc1_ldf"], Wd, cfg.ff, blk["fc1_bf"], gelu=True,
                     out=self.f[:, :cfg.ff], **self._norm(blk["fc1_c"], False))
            ops.gemm(self.f[:, :cfg.ff], blk["fc2_w"], blk["fc2_ld"], cfg.ff, Wd, blk["fc2_b"], res=self.x, out=self.x,
                     **fold)
            ops.gemm(self.xb, blk["gate_wf"], blk["gate_ldf"], Wd, 2 * Wd, blk["gate_b"], out=self.G,
                     **self._norm(blk["gate_c"], True, keep=True))
            ops.rglru_fold(self.G, blk["lru"].softplus_a, self.mom, blk["rms_w"], self.state[i], self.x, self.xb,
                           self.stats, cfg.lru_c, first)
