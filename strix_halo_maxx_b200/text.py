"""The moondream2 text decoder that consumes the tower's features, on B200: FastMD2's image prefill and question
prefill (moondream/gpu/md2fast.py:169-212) with the tower's kernels plus the rotary / KV-cache and causal
attention kernels of csrc/text.cu.

Per layer (md2fast.py:169-199, the parallel block):
    h = LN(x)                                   vt_layernorm, bf16
    qkv = h Wqkv^T + b                          vt_gemm (N = 3 x 2048)
    rope(q, k), cache k / v                     vt_rope_qkv
    a = attention                               prefix: tcgen05 attention over its 730 keys (no mask, as
                                                md2fast.py:182-183); question: vt_attn_causal over the cache
    x += a Wproj^T + b                          vt_gemm, fp32 residual epilogue
    x += gelu_tanh(h W1^T + b1) W2^T + b2       vt_gemm (GELU epilogue), vt_gemm + residual
The yes / no logits are LN(x[last]) Wyn^T + byn (md2fast.py:210-212).  The four linears run either as the
tower's bf16 tcgen05 GEMMs (int8=False, the reference's FastMD2 with tlin_cls=HLin) or as W8A8 int8 tcgen05
GEMMs (int8=True, tlin_cls=HI8Lin, md2fast.py:88, 112-113): per layer the LN output is quantised once, in the
LayerNorm kernel (vt_layernorm_quant), and shared by qkv and fc1 (md2fast.py:174); the attention output and the
fc1 output (GELU fused into its epilogue) are quantised before proj and fc2 (vt_quant_rows + vt_gemm_i8,
ops.I8Lin).  The KV caches ([layers][H][762][64]
bf16) live on the device, owned by this object: encode() fills positions 0 .. 729, query() 730 .. 761.
"""
import torch

from .config import TEXT, TextConfig
from . import ops
from .ops import BF16
from .tower import _dev_mat, _dev_vec

F32 = torch.float32


def rope_tables(cfg: TextConfig, device):
    """cos, sin fp32 [ctx, rot / 2]: angle pos * theta^(-2i / rot), evaluated in float64."""
    inv = cfg.theta ** (-torch.arange(0, cfg.rot, 2, dtype=torch.float64) / cfg.rot)
    ang = torch.arange(cfg.ctx, dtype=torch.float64)[:, None] * inv[None]
    return torch.cos(ang).float().contiguous().to(device), torch.sin(ang).float().contiguous().to(device)


class TextDecoder:
    def __init__(self, weights, cfg: TextConfig = TEXT, device="cuda", graphs=True, int8=False):
        self.cfg = cfg
        self.use_graphs = graphs
        self.int8 = int8
        self._qgraph = self._egraph = None
        dev = self.dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        W = weights
        self.n_layers = sum(1 for k in W if k.endswith(".qkv_w"))
        self.wte = _dev_vec(W["wte"], dev)
        self.layers = []
        for i in range(self.n_layers):
            p = f"tblocks.{i}."
            b = {"ln_w": _dev_vec(W[p + "ln_w"], dev), "ln_b": _dev_vec(W[p + "ln_b"], dev)}
            for n in ("qkv", "proj", "fc1", "fc2"):
                if int8:
                    b[n] = ops.I8Lin(W[p + n + "_w"], W[p + n + "_b"], dev)
                    continue
                b[n + "_w"], b[n + "_ld"] = _dev_mat(W[p + n + "_w"], dev)
                b[n + "_b"] = _dev_vec(W[p + n + "_b"], dev)
            self.layers.append(b)
        self.post_w, self.post_b = _dev_vec(W["tpost_ln_w"], dev), _dev_vec(W["tpost_ln_b"], dev)
        self.yn_w, self.yn_ld = _dev_mat(W["lm_small_w"], dev)
        self.yn_b = _dev_vec(W["lm_small_b"], dev)
        self.cos, self.sin = rope_tables(cfg, dev)
        D, H, hd, P = cfg.dim, cfg.heads, cfg.head_dim, cfg.prefix
        self.x = torch.empty(P, D, dtype=F32, device=dev)
        self.h = torch.empty(P, D, dtype=BF16, device=dev)
        self.qkv = torch.empty(P, 3 * D, dtype=BF16, device=dev)
        self.qflat = torch.empty(H * P * hd, dtype=BF16, device=dev)
        self.a = torch.empty(P, D, dtype=BF16, device=dev)
        self.f = torch.empty(P, cfg.ff, dtype=BF16, device=dev)
        self.kc = torch.zeros(self.n_layers, H, cfg.ctx, hd, dtype=BF16, device=dev)
        self.vc = torch.zeros(self.n_layers, H, cfg.ctx, hd, dtype=BF16, device=dev)
        self.hl = torch.empty(1, D, dtype=BF16, device=dev)
        self.xl = torch.empty(1, D, dtype=F32, device=dev)
        self._ids = torch.zeros(cfg.q_len, dtype=torch.int64, device=dev)
        self._last = torch.zeros(1, dtype=torch.int64, device=dev)
        self._bos = torch.zeros(1, dtype=torch.int64, device=dev)
        self._emb = torch.zeros(P - 1, D, dtype=F32, device=dev)
        self.logits = torch.empty(1, 8, dtype=F32, device=dev)
        self.attn = ops.VtAttn(H, P, hd, dev)
        if int8:  # quantised activations (padded 16-byte row pitches) and their per-token scales
            pad = lambda k: (k + ops.I8_PAD + 15) // 16 * 16
            self.hq = torch.empty(P, pad(D), dtype=torch.int8, device=dev)[:, :D]
            self.aq = torch.empty(P, pad(D), dtype=torch.int8, device=dev)[:, :D]
            self.fq = torch.empty(P, pad(cfg.ff), dtype=torch.int8, device=dev)[:, :cfg.ff]
            self.hs, self.as_, self.fs = (torch.empty(P, dtype=F32, device=dev) for _ in range(3))
        # split-K workspace of the question's GEMMs (32 rows; the widest output is fc1's)
        self.ws = ops.gemm_workspace(cfg.q_len, max(3 * D, cfg.ff), dev)

    def _layers(self, n, pos0, full):
        cfg = self.cfg
        D, H, hd, Fh = cfg.dim, cfg.heads, cfg.head_dim, cfg.ff
        x, h, qkv, a, f = self.x[:n], self.h[:n], self.qkv[:n], self.a[:n], self.f[:n]
        q = self.qflat[:H * n * hd].view(H, n, hd)
        ws = None if full else self.ws  # the question's GEMMs are too small to fill the GPU: split K
        if self.int8:
            return self._layers_i8(n, pos0, full, q, ws)
        for i, b in enumerate(self.layers):
            ops.layer_norm(x, b["ln_w"], b["ln_b"], cfg.eps, out=h)
            ops.gemm(h, b["qkv_w"], b["qkv_ld"], D, 3 * D, b["qkv_b"], out=qkv, ws=ws)
            ops.rope_qkv(qkv, pos0, self.cos, self.sin, q, self.kc[i], self.vc[i])
            if full:  # the prefix: no mask, its own n keys (md2fast.py:182-183)
                self.attn(q[None], self.kc[i][None, :, pos0:pos0 + n], self.vc[i][None, :, pos0:pos0 + n], out=a[None])
            else:     # the question: causal over the cache (md2fast.py:184-185 with the query mask)
                ops.attn_causal(q, self.kc[i], self.vc[i], pos0, a)
            ops.gemm(a, b["proj_w"], b["proj_ld"], D, D, b["proj_b"], res=x, out=x, ws=ws)
            ops.gemm(h, b["fc1_w"], b["fc1_ld"], D, Fh, b["fc1_b"], gelu=True, out=f, ws=ws)
            ops.gemm(f, b["fc2_w"], b["fc2_ld"], Fh, D, b["fc2_b"], res=x, out=x, ws=ws)

    def _layers_i8(self, n, pos0, full, q, ws):
        """The same layers with the W8A8 linears (HI8Lin, md2fast.py:169-199 with SHARE_QUANT)."""
        cfg = self.cfg
        x, h, qkv, a, f = self.x[:n], self.h[:n], self.qkv[:n], self.a[:n], self.f[:n]
        hq, aq, fq = self.hq[:n], self.aq[:n], self.fq[:n]
        hs, as_, fs = self.hs[:n], self.as_[:n], self.fs[:n]
        for i, b in enumerate(self.layers):
            # LN + per-token quantisation in one kernel; the int8 rows are shared by qkv and fc1 (md2fast.py:174)
            pre = ops.layer_norm_quant(x, b["ln_w"], b["ln_b"], cfg.eps, hq, hs)
            b["qkv"](h, pre=pre, out=qkv, ws=ws)
            ops.rope_qkv(qkv, pos0, self.cos, self.sin, q, self.kc[i], self.vc[i])
            if full:
                self.attn(q[None], self.kc[i][None, :, pos0:pos0 + n], self.vc[i][None, :, pos0:pos0 + n], out=a[None])
            else:
                ops.attn_causal(q, self.kc[i], self.vc[i], pos0, a)
            b["proj"](a, pre=b["proj"].quant(a, aq, as_), res=x, out=x, ws=ws)
            b["fc1"](h, gelu=True, pre=pre, out=f, ws=ws)
            b["fc2"](f, pre=b["fc2"].quant(f, fq, fs), res=x, out=x, ws=ws)

    def encode(self, emb, bos):
        """Image prefill (md2fast.py:201-206): emb [729, D] fp32 / bf16 on the device, bos id.  The image
        features and the bos id go into static device buffers, so with graphs=True every prefill after the
        first replays one CUDA graph of its ~190 launches (same kernels and buffers as the eager path)."""
        self._emb.copy_(emb)
        self._bos.fill_(int(bos))
        if not self.use_graphs:
            self._encode()
        elif self._egraph is None:
            self._encode()  # first prefill eagerly (one-time library and buffer set-up), then capture
            self._egraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._egraph):
                self._encode()
        else:
            self._egraph.replay()
        return self.x

    def _encode(self):
        torch.index_select(self.wte, 0, self._bos, out=self.x[:1])
        self.x[1:self.cfg.prefix].copy_(self._emb)
        self._layers(self.cfg.prefix, 0, True)

    def query(self, ids, last):
        """Question prefill (md2fast.py:208-212): ids [q_len] int64 on the device, `last` the index of the
        question's last real token -> yes / no logits [n_yn] fp32.  The ids and `last` go into static
        device buffers, so with graphs=True (default) every question after the first replays one CUDA graph
        of the ~170 launches (same kernels and buffers as the eager path, bit-identical logits)."""
        cfg = self.cfg
        self._ids.copy_(ids)
        self._last.fill_(int(last))
        if not self.use_graphs:
            self._query()
        elif self._qgraph is None:
            self._query()  # first question eagerly (one-time library set-up), then capture
            self._qgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._qgraph):
                self._query()
        else:
            self._qgraph.replay()
        return self.logits[0, :cfg.n_yn]

    def _query(self):
        cfg = self.cfg
        torch.index_select(self.wte, 0, self._ids, out=self.x[:cfg.q_len])
        self._layers(cfg.q_len, cfg.prefix, False)
        torch.index_select(self.x, 0, self._last, out=self.xl)
        ops.layer_norm(self.xl, self.post_w, self.post_b, cfg.eps, out=self.hl)
        ops.gemm(self.hl, self.yn_w, self.yn_ld, cfg.dim, cfg.n_yn, self.yn_b, out=self.logits[:, :cfg.n_yn], ws=self.ws)


def op_times(dev, n=20, reps=5):
    """Warm time (us) of each kernel of a decoder layer at the prefill (730) and question (32) row counts:
    every op captured n times in one CUDA graph, replayed `reps` times; inputs L2-resident."""
    F32_ = torch.float32

    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(n):
                    fn()
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return round(e0.elapsed_time(e1) / (n * reps) * 1000, 2)

    D, Fh = TEXT.dim, TEXT.ff
    out = {}
    for M in (TEXT.prefix, TEXT.q_len):
        ws = ops.gemm_workspace(M, Fh, dev) if M == TEXT.q_len else None
        x = torch.randn(M, D, device=dev)
        w_ln, b_ln = torch.ones(D, device=dev), torch.zeros(D, device=dev)
        h = torch.empty(M, D, device=dev, dtype=BF16)
        hq, hs = torch.empty(M, D, device=dev, dtype=torch.int8), torch.empty(M, device=dev)
        f = torch.randn(M, Fh, device=dev).to(BF16)
        fq, fs = torch.empty(M, Fh, device=dev, dtype=torch.int8), torch.empty(M, device=dev)
        r = {"ln": graph_us(lambda: ops.layer_norm(x, w_ln, b_ln, 1e-5, out=h)),
             "ln_quant": graph_us(lambda: ops.layer_norm_quant(x, w_ln, b_ln, 1e-5, hq, hs)),
             "quant_2048": graph_us(lambda: ops.quant_rows(h, hq, hs)),
             "quant_8192": graph_us(lambda: ops.quant_rows(f, fq, fs))}
        for name, N, K, res, gelu in (("qkv", 3 * D, D, False, False), ("proj", D, D, True, False),
                                      ("fc1", Fh, D, False, True), ("fc2", D, Fh, True, False)):
            a = torch.randn(M, K, device=dev).to(BF16)
            wt = torch.randn(N, K, device=dev) * 0.02
            bias = torch.zeros(N, device=dev)
            lin, wb = ops.I8Lin(wt, bias, dev), wt.to(BF16)
            aq, asc = ops.quant_rows(a)
            o = torch.zeros(M, N, device=dev, dtype=F32_ if res else BF16)
            rr = o if res else None
            r[name + "_bf16"] = graph_us(lambda: ops.gemm(a, wb, K, K, N, bias, gelu=gelu, res=rr, out=o, ws=ws))
            r[name + "_i8"] = graph_us(lambda: ops.gemm_i8(aq, asc, lin.wq, lin.ldw, K, N, lin.sw, bias, gelu=gelu,
                                                           res=rr, out=o, ws=ws))
        out[M] = r
    return out


def main(argv=None):
    """python -m strix_halo_maxx_b200.text [--int8] [--bf16] [--reps N] [--eager] [--layers L] [--ops]: the decoder on
    device-random weights (weights.text_weights_device); prints the mean prefill / question ms of each
    selected variant (both by default).  With --reps 0 it runs one eager prefill and one question per variant
    and prints nothing else: the command to put under a profiler's launch list."""
    import argparse
    from .weights import text_weights_device
    ap = argparse.ArgumentParser()
    ap.add_argument("--int8", action="store_true")
    ap.add_argument("--bf16", action="store_true")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--eager", action="store_true", help="no CUDA-graph replay")
    ap.add_argument("--layers", type=int, default=None, help="fewer layers than the model's 24 (small profiles)")
    ap.add_argument("--ops", action="store_true", help="warm per-kernel times of one layer (op_times) instead")
    a = ap.parse_args(argv)
    if a.ops:
        for M, r in op_times(torch.device("cuda", torch.cuda.current_device())).items():
            print(M, r, flush=True)
        return
    variants = [v for v, on in (("bf16", a.bf16), ("int8", a.int8)) if on] or ["bf16", "int8"]
    dev = torch.device("cuda", torch.cuda.current_device())
    W = text_weights_device(TEXT, dev, seed=0, n_layers=a.layers)
    g = torch.Generator(device=dev).manual_seed(1)
    emb = torch.randn(TEXT.prefix - 1, TEXT.dim, device=dev, generator=g)
    ids = torch.randint(1, TEXT.vocab, (TEXT.q_len,), device=dev, generator=g)
    for v in variants:
        dec = TextDecoder(W, TEXT, device=dev, graphs=not a.eager and a.reps > 0, int8=(v == "int8"))
        res = {}
        for name, fn in (("prefill_ms", lambda: dec.encode(emb, 0)), ("question_ms", lambda: dec.query(ids, TEXT.q_len - 1))):
            if a.reps <= 0:
                fn()
                continue
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            res[name] = round(e0.elapsed_time(e1) / a.reps, 4)
        torch.cuda.synchronize()
        if res:
            print(v, res, flush=True)
        del dec


if __name__ == "__main__":
    main()
