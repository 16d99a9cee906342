"""The full TAPNext++ per-frame block step on B200 (the reference's block, tapnext/npu/step8.py:469-486;
the BASELINE config 3 step in tapnext.py simplifies it).  Token layout and sizes as config 3: 8x8 patches
of a 256x256 frame (1024 tokens) + position embedding, then the point-query tokens, width 768, 12 heads x 64.

Per block, in the reference's order:
    t   = RMSNorm(x) (1 + scale)                       vt_rmsnorm
    y, xx = t Wyx^T + byx                              one vt_gemm (linear_yx, N = 1536), bf16
    z   = RG-LRU(conv_1d(xx)) * gelu_tanh(y)           vt_ssm_step (4-tap history ring, fp32 state, GELU of y)
    x  += z Wout^T + bout                              vt_gemm, fp32 residual epilogue
    G   = RMSNorm(x) (1 + scale) Wup^T + bup           vt_rmsnorm, vt_gemm (N = 2 x 3072: [gate | up])
    x  += (gelu_tanh(gate) * up) Wdown^T + bdown       vt_gated_gelu_mul, vt_gemm + residual
    x  += MHA(LN_1(x))                                 the tower's qkv-tile GEMM + tcgen05 attention (d 64)
    x  += gelu_erf(LN_2(x) W0^T + b0) W3^T + b3        vt_gemm, vt_gelu_erf, vt_gemm + residual
and the encoder LayerNorm after the last block, then (with heads=) the tracking heads on the query tokens
(TrackHeads; the reference's host heads, step8.py:327-362).  The recurrent state (h fp32 and the last three xx of every
block) lives on the device, owned by this object; reset() starts a new video.

A frame is ~200 kernel launches, more host time than the B200 needs to run them, so with graphs=True
(default) every frame after a video's first replays a CUDA graph of the whole step, one per position of the
history ring (frame % 3), captured the first time that position comes up; the frame and the queries are
copied into static input buffers first.  The graphs launch the same kernels on the same buffers as the
eager step, so the results are bit-identical (tests/test_tapnextpp_gpu.py).
"""
import torch
import torch.nn.functional as F

from .config import TAPNEXT, TapNextConfig
from . import ops
from .ops import BF16, _pad8
from .tower import _dev_mat, _dev_vec

F32 = torch.float32


class TrackHeads:
    """The tracking heads on the query tokens, on the device in fp32 (the reference runs them on the host after
    every frame: Step8.heads_np, tapnext/npu/step8.py:327-362).  Per head: Linear width -> hidden, LayerNorm,
    erf GELU, Linear hidden -> hidden, LayerNorm, erf GELU, Linear -> 2 x bins coordinate logits (y | x) or one
    visibility logit; then per axis the soft-argmax over +-window bins of the first maximum at the temperature,
    + 0.5.  The two heads run side by side: their first Linear as one [width, 2 hidden] product, their second
    and third as one product each with a block-diagonal weight (the other head's rows are zeros, so every output's
    k-ordered fp32 sum is the head's own), and their LayerNorms as one pass.
    HW: weights as strix_halo_maxx_b200.weights.heads_weights names them ([out, in], torch's layout).
    __call__(x [Q, width] bf16) -> (tracks [Q, 2], logits [Q, 2 bins], vis [Q]) fp32 views of buffers this
    object owns (valid until the next call)."""

    def __init__(self, HW, cfg: TapNextConfig = TAPNEXT, device="cuda", n_queries=None):
        self.cfg = cfg
        dev = torch.device(device)
        Q = cfg.n_queries if n_queries is None else n_queries
        Hh, nb = cfg.head_hidden, cfg.track_bins
        t = lambda name: torch.as_tensor(HW[name]).float()                          # noqa: E731
        self.w0 = torch.cat([t("coord.0_w").t(), t("vis.0_w").t()], 1).contiguous().to(dev)   # [width, 2 Hh]
        self.b0 = torch.cat([t("coord.0_b"), t("vis.0_b")]).to(dev)
        self.g1 = torch.stack([t("coord.1_w"), t("vis.1_w")]).to(dev)
        self.be1 = torch.stack([t("coord.1_b"), t("vis.1_b")]).to(dev)
        # second Linear: [2 Hh, 2 Hh] = diag(coord.3_w^T, vis.3_w^T)
        self.w3 = torch.zeros(2 * Hh, 2 * Hh)
        self.w3[:Hh, :Hh], self.w3[Hh:, Hh:] = t("coord.3_w").t(), t("vis.3_w").t()
        self.w3 = self.w3.to(dev)
        self.b3 = torch.cat([t("coord.3_b"), t("vis.3_b")]).to(dev)
        self.g4 = torch.stack([t("coord.4_w"), t("vis.4_w")]).to(dev)
        self.be4 = torch.stack([t("coord.4_b"), t("vis.4_b")]).to(dev)
        # third Linear: [2 Hh, 2 nb + 4]: coord.6_w^T in rows [0, Hh) x columns [0, 2 nb), vis.6_w^T in rows
        # [Hh, 2 Hh) x column 2 nb; three zero columns keep the row pitch a multiple of 16 bytes
        self.nout = 2 * nb + 4
        self.w6 = torch.zeros(2 * Hh, self.nout)
        self.w6[:Hh, :2 * nb], self.w6[Hh:, 2 * nb:2 * nb + 1] = t("coord.6_w").t(), t("vis.6_w").t()
        self.w6 = self.w6.to(dev)
        self.b6 = torch.cat([t("coord.6_b"), t("vis.6_b"), torch.zeros(3)]).to(dev)
        self.y1 = torch.empty(Q, 2 * Hh, dtype=F32, device=dev)                    # [coord | vis] per query
        self.y2 = torch.empty(Q, 2 * Hh, dtype=F32, device=dev)
        self.out = torch.empty(Q, self.nout, dtype=F32, device=dev)                # [logits | vis | 0 0 0]
        self.tracks = torch.empty(Q, 2, dtype=F32, device=dev)

    def __call__(self, x):
        cfg = self.cfg
        Q, Hh = x.shape[0], cfg.head_hidden
        assert Q <= self.y1.shape[0]
        nb2 = 2 * cfg.track_bins
        y1, y2, out, tr = self.y1[:Q], self.y2[:Q], self.out[:Q], self.tracks[:Q]
        ops.head_linear(x, self.w0, self.b0, y1)
        ops.head_ln_gelu(y1.view(2 * Q, Hh), self.g1, self.be1, cfg.head_eps)
        ops.head_linear(y1, self.w3, self.b3, y2)
        ops.head_ln_gelu(y2.view(2 * Q, Hh), self.g4, self.be4, cfg.head_eps)
        ops.head_linear(y2, self.w6, self.b6, out)
        lg = out[:, :nb2]
        ops.soft_argmax(lg, cfg.track_bins, cfg.track_window, cfg.track_temperature, tr)
        return tr, lg, out[:, nb2]


class TapNextPPStep:
    def __init__(self, weights, cfg: TapNextConfig = TAPNEXT, device="cuda", graphs=True, heads=None, fold_ln=True,
                 rows_in_gemm=True):
        self.cfg = cfg
        self.rows_in_gemm = rows_in_gemm
        self.fold_ln = fold_ln
        self.use_graphs = graphs
        self._graphs = {}
        self._frame_in = self._q_in = None
        dev = self.dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        W = weights
        Wd, Fh = cfg.width, cfg.ff
        self.n_blocks = sum(1 for k in W if k.endswith(".yx_w"))
        self.pe_w, self.pe_ld = _dev_mat(W["patch_w"], dev)
        self.pe_b = _dev_vec(W["patch_b"], dev)
        self.pos = _dev_vec(W["pos_emb"], dev).reshape(cfg.n_img_tok, Wd)
        self.blocks = []
        for i in range(self.n_blocks):
            p = f"blocks.{i}."
            b = {}
            # linear_yx as one 768 -> 1536 GEMM ([y | x], the reference's layout); the GELU of y is taken in
            # vt_ssm_step (gelu_y), which reads y from the same buffer
            b["yx_w"], b["yx_ld"] = _dev_mat(W[p + "yx_w"], dev)
            b["yx_b"] = _dev_vec(W[p + "yx_b"], dev)
            for n in ("out", "up", "down", "qkv", "proj", "fc1", "fc2"):
                b[n + "_w"], b[n + "_ld"] = _dev_mat(W[p + n + "_w"], dev)
                b[n + "_b"] = _dev_vec(W[p + n + "_b"], dev)
            b["rms0"] = _dev_vec(1.0 + torch.as_tensor(W[p + "rms0_scale"]).float(), dev)
            b["rms1"] = _dev_vec(1.0 + torch.as_tensor(W[p + "rms1_scale"]).float(), dev)
            for n in ("conv_w", "conv_b", "gx_w", "gx_b", "ga_w", "ga_b", "ln1_w", "ln1_b", "ln2_w", "ln2_b"):
                b[n] = _dev_vec(W[p + n], dev)
            b["softplus_a"] = _dev_vec(F.softplus(torch.as_tensor(W[p + "a_param"]).double()).float(), dev)
            if fold_ln:
                # each norm folded into the GEMM after it: W * gamma (bf16), c = rowsum, b + W beta; the RMSNorms'
                # gamma is (1 + scale) and their GEMM epilogues use mean 0
                zero = torch.zeros(Wd)
                for n, g, be in (("yx", 1.0 + torch.as_tensor(W[p + "rms0_scale"]).float(), zero),
                                 ("up", 1.0 + torch.as_tensor(W[p + "rms1_scale"]).float(), zero),
                                 ("qkv", W[p + "ln1_w"], W[p + "ln1_b"]), ("fc1", W[p + "ln2_w"], W[p + "ln2_b"])):
                    wf, c, bf = ops.fold_layernorm(W[p + n + "_w"], W[p + n + "_b"], g, be)
                    if n == "up":  # gate / up rows interleaved by 16: the GEMM epilogue forms gelu(gate) * up
                        wf, c, bf = (ops.gate_up_interleave(torch.as_tensor(t), Fh) for t in (wf, c, bf))
                    b[n + "_wf"], b[n + "_ldf"] = _dev_mat(wf, dev)
                    b[n + "_c"] = _dev_vec(c, dev)
                    b[n + "_bf"] = _dev_vec(bf, dev)
            self.blocks.append(b)
        self.fin_w = _dev_vec(W["final_ln_w"], dev)
        self.fin_b = _dev_vec(W["final_ln_b"], dev)
        T = cfg.ntok
        self.a_pe = torch.zeros(cfg.n_img_tok, _pad8(cfg.patch_k), dtype=BF16, device=dev)
        self.x = torch.empty(T, Wd, dtype=F32, device=dev)
        self.t = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.yx = torch.empty(T, 2 * Wd, dtype=BF16, device=dev)
        self.z = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.G = torch.empty(T, 2 * Fh, dtype=BF16, device=dev)
        self.m = torch.empty(T, Fh, dtype=BF16, device=dev)
        self.tiles = ops.attn_tiles(1, T, cfg.heads, cfg.head_dim, dev)
        self.a = torch.empty(T, Wd, dtype=BF16, device=dev)
        self.f = torch.empty(T, Fh, dtype=BF16, device=dev)
        self.h = torch.zeros(self.n_blocks, T, Wd, dtype=F32, device=dev)
        self.hist = torch.zeros(self.n_blocks, 3, T, Wd, dtype=BF16, device=dev)
        self.out = torch.empty(T, Wd, dtype=BF16, device=dev)
        if fold_ln:
            self.xb = torch.empty(T, Wd, dtype=BF16, device=dev)                  # bf16 copy of x
            self.stats = torch.empty(T, Wd // 32, 2, dtype=F32, device=dev)      # per-32-column (mean, M2) of x
            self.mom = torch.empty(T, 2, dtype=F32, device=dev)                  # (mean | 0, rstd) per row
        # optional tracking heads (weights as weights.heads_weights): run on the query tokens inside the step
        self.heads = TrackHeads(heads, cfg, dev) if heads is not None else None
        self.reset()

    def reset(self):
        """A new video: zero conv history, no recurrent state."""
        self.hist.zero_()
        self.frame = 0

    def step(self, frame, queries):
        """frame [3, 256, 256] in [-1, 1], queries [n_queries, 768] fp32 (device) -> [ntok, 768] bf16."""
        k = self.frame % 3  # history roles: x_(t-3) = slot k, x_(t-2) = k+1, x_(t-1) = k+2 (mod 3)
        if not self.use_graphs or self.frame == 0:
            self._run(frame, queries, k, self.frame == 0)
        else:
            if self._frame_in is None:
                self._frame_in, self._q_in = torch.empty_like(frame), torch.empty_like(queries)
            self._frame_in.copy_(frame)
            self._q_in.copy_(queries)
            g = self._graphs.get(k)
            if g is None:
                g = self._graphs[k] = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._run(self._frame_in, self._q_in, k, False)
            g.replay()
        self.frame += 1
        return self.out

    def track(self, frame, queries):
        """The reference's Step8.step (tapnext/npu/step8.py:316-325): one frame, then the heads on the query
        tokens -> (tracks [Q, 2], logits [Q, 2 bins], visibility logits [Q], query tokens [Q, width] bf16).
        Needs heads= at construction; the heads run inside the step (and its CUDA graph)."""
        assert self.heads is not None, "TapNextPPStep(heads=...) is needed for tracks"
        out = self.step(frame, queries)
        h = self.heads
        Q, nb2 = self.cfg.n_queries, 2 * self.cfg.track_bins
        return h.tracks[:Q], h.out[:Q, :nb2], h.out[:Q, nb2], out[self.cfg.n_img_tok:]

    def _run(self, frame, queries, k, first):
        cfg = self.cfg
        T, Wd, NI, Fh = cfg.ntok, cfg.width, cfg.n_img_tok, cfg.ff
        ops.im2col(frame.reshape(1, *frame.shape[-3:]), cfg.patch, self.a_pe)
        ops.gemm(self.a_pe[:, :cfg.patch_k], self.pe_w, self.pe_ld, cfg.patch_k, Wd, self.pe_b,
                 res=self.pos, res_period=NI, out=self.x[:NI])
        self.x[NI:].copy_(queries)
        if self.fold_ln:
            self._blocks_folded(k, first)
        else:
            self._blocks(k, first)
        ops.layer_norm(self.x, self.fin_w, self.fin_b, cfg.eps, out=self.out)
        if self.heads is not None:
            self.heads(self.out[NI:])

    def _blocks(self, k, first):
        cfg = self.cfg
        T, Wd, Fh = cfg.ntok, cfg.width, cfg.ff
        for i, b in enumerate(self.blocks):
            hist = (self.hist[i, k], self.hist[i, (k + 1) % 3], self.hist[i, (k + 2) % 3])
            # recurrent block (step8.py:474-481)
            ops.rms_norm(self.x, b["rms0"], cfg.eps, out=self.t)
            ops.gemm(self.t, b["yx_w"], b["yx_ld"], Wd, 2 * Wd, b["yx_b"], out=self.yx)
            ops.ssm_step(self.yx[:, :Wd], self.yx[:, Wd:], hist, self.h[i], b["conv_w"], b["conv_b"],
                         b["softplus_a"], b["gx_w"], b["gx_b"], b["ga_w"], b["ga_b"], self.z, first, gelu_y=True)
            ops.gemm(self.z, b["out_w"], b["out_ld"], Wd, Wd, b["out_b"], res=self.x, out=self.x)
            # gated MLP (step8.py:482-483)
            ops.rms_norm(self.x, b["rms1"], cfg.eps, out=self.t)
            ops.gemm(self.t, b["up_w"], b["up_ld"], Wd, 2 * Fh, b["up_b"], out=self.G)
            ops.gated_gelu_mul(self.G, self.m)
            ops.gemm(self.m, b["down_w"], b["down_ld"], Fh, Wd, b["down_b"], res=self.x, out=self.x)
            # ViT block (step8.py:484-486)
            ops.layer_norm(self.x, b["ln1_w"], b["ln1_b"], cfg.eps, out=self.t)
            ops.gemm_qkv_tiles(self.t, b["qkv_w"], b["qkv_ld"], Wd, b["qkv_b"], self.tiles, T, cfg.heads, cfg.head_dim)
            ops.attention_tiles(self.tiles, 1, T, cfg.heads, cfg.head_dim, self.a)
            ops.gemm(self.a, b["proj_w"], b["proj_ld"], Wd, Wd, b["proj_b"], res=self.x, out=self.x)
            ops.layer_norm(self.x, b["ln2_w"], b["ln2_b"], cfg.eps, out=self.t)
            ops.gemm(self.t, b["fc1_w"], b["fc1_ld"], Wd, Fh, b["fc1_b"], out=self.f)
            ops.gelu_erf(self.f)
            ops.gemm(self.f, b["fc2_w"], b["fc2_ld"], Fh, Wd, b["fc2_b"], res=self.x, out=self.x)

    def _norm(self, c, rms):
        """gemm keyword arguments of a norm of x folded into the GEMM that follows (c = its rowsum vector): the row
        factors merged from x's chunk statistics in that GEMM's epilogue, or, with rows_in_gemm=False, computed
        into self.mom by a vt_row_rms / vt_row_moments pass launched here."""
        cfg = self.cfg
        if self.rows_in_gemm:
            return dict(ln_rows=(self.stats, cfg.eps, rms, c, None))
        (ops.row_rms if rms else ops.row_moments)(self.stats, cfg.eps, self.mom)
        return dict(ln=(self.mom, c))

    def _blocks_folded(self, k, first):
        """The same blocks with every norm folded into the GEMM after it: the residual GEMMs (linear_out,
        ffw_down, out_proj, mlp.3) also write the bf16 copy of x and its 32-column chunk statistics, from which
        the next folded GEMM's epilogue takes its rows' norm factors (see _norm)."""
        cfg = self.cfg
        T, Wd, Fh = cfg.ntok, cfg.width, cfg.ff
        fold = dict(out2=self.xb, stats_out=self.stats)
        ops.row_stats(self.x, self.stats, self.xb)
        for i, b in enumerate(self.blocks):
            hist = (self.hist[i, k], self.hist[i, (k + 1) % 3], self.hist[i, (k + 2) % 3])
            # recurrent block (step8.py:474-481)
            ops.gemm(self.xb, b["yx_wf"], b["yx_ldf"], Wd, 2 * Wd, b["yx_bf"], out=self.yx, **self._norm(b["yx_c"], True))
            ops.ssm_step(self.yx[:, :Wd], self.yx[:, Wd:], hist, self.h[i], b["conv_w"], b["conv_b"],
                         b["softplus_a"], b["gx_w"], b["gx_b"], b["ga_w"], b["ga_b"], self.z, first, gelu_y=True)
            ops.gemm(self.z, b["out_w"], b["out_ld"], Wd, Wd, b["out_b"], res=self.x, out=self.x, **fold)
            # gated MLP (step8.py:482-483)
            ops.gemm(self.xb, b["up_wf"], b["up_ldf"], Wd, 2 * Fh, b["up_bf"], out=self.m, gelu="gated",
                     **self._norm(b["up_c"], True))
            ops.gemm(self.m, b["down_w"], b["down_ld"], Fh, Wd, b["down_b"], res=self.x, out=self.x, **fold)
            # ViT block (step8.py:484-486)
            ops.gemm(self.xb, b["qkv_wf"], b["qkv_ldf"], Wd, 3 * Wd, b["qkv_bf"], out=self.tiles,
                     tiles=(T, cfg.heads, cfg.head_dim), **self._norm(b["qkv_c"], False))
            ops.attention_tiles(self.tiles, 1, T, cfg.heads, cfg.head_dim, self.a)
            ops.gemm(self.a, b["proj_w"], b["proj_ld"], Wd, Wd, b["proj_b"], res=self.x, out=self.x, **fold)
            ops.gemm(self.xb, b["fc1_wf"], b["fc1_ldf"], Wd, Fh, b["fc1_bf"], out=self.f, **self._norm(b["fc1_c"], False))
            # the exact GELU as its own pass: in fc1's epilogue (one 256 x 256 tile per CTA pair at 1280 rows, so
            # nothing hides it) it measured 20 us per frame slower
            ops.gelu_erf(self.f)
            ops.gemm(self.f, b["fc2_w"], b["fc2_ld"], Fh, Wd, b["fc2_b"], res=self.x, out=self.x, **fold)
