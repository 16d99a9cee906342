"""Op-level drop-ins for the reference's plugin API, backed by libvt_b200.so.

* VtLin  -- the `lin_cls` the reference's FastMD2 builds every linear with (md2fast.py:33-40, 87-103):
  VtLin(weight, bias, dtype) -> __call__(x, gelu=False, res=None), class flags fused_gelu / fused_res
  (hgemm.HLin, hgemm.py:139-178).
* VtAttn -- hattn.Attn(H, T, D) -> __call__(q, k, v, out=None) -> (B, T, H*D) (hattn.py:17-37).
* I8Lin  -- the `tlin_cls` of the reference's int8 text model, hgemm.HI8Lin (hgemm.py:95-137): W8A8 with
  quant(x) -> (q, s) and __call__(x, gelu=False, res=None, pre=None); quant_rows / layer_norm_quant / gemm_i8
  are its kernels.
* layer_norm / im2col / crop_combine / rglru -- thin wrappers of the remaining kernels.

Every call launches on torch's current stream and raises VtError on a non-zero return code.
"""
import os

import torch

from ._lib import lib, check as _check

BF16 = torch.bfloat16

# Number of kernel launches made through this module (bench.py reports the count of its timed region).
LAUNCHES = 0


def check(rc, what):
    global LAUNCHES
    _check(rc, what)
    LAUNCHES += 1


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _pad8(n):
    return (n + 7) // 8 * 8


def as_gemm_operand(x2):
    """bf16 2-D view with unit column stride, a row pitch that is a multiple of 8 and a 16-B aligned base."""
    if x2.dtype == BF16 and x2.stride(-1) == 1 and x2.stride(0) % 8 == 0 and x2.data_ptr() % 16 == 0 \
            and x2.stride(0) >= x2.shape[1]:
        return x2
    M, K = x2.shape
    buf = torch.empty(M, _pad8(K), dtype=BF16, device=x2.device)
    buf[:, :K] = x2
    return buf[:, :K]


def gemm(x2, w, ldw, K, N, bias=None, gelu=False, res=None, res_period=0, out=None, out_f32=False, out2=None,
         stats_out=None, ln=None, tiles=None, ws=None, ln_rows=None):
    """out[M, N] = x2 . w^T + bias (+ GELU) (+ res), see vt_gemm_fused in include/vt_b200.h.
    stats_out: [M, N/32, 2] fp32 row-chunk statistics of the (fp32) output; ln: (moments [M, 2], c) of a
    LayerNorm folded into this GEMM; ln_rows: (stats [M, nchunk, 2], eps, rms, c, moments_out or None), the same
    fold (a LayerNorm, or an RMSNorm when rms) with the row factors merged in the epilogue from the chunk
    statistics (vt_gemm_fused_lnstats); tiles: (T, H, D) to scatter into the attention-tile buffer `out`;
    ws: a zero-filled workspace (gemm_workspace) that lets small GEMMs split K (vt_gemm_fused_ws);
    gelu="gated": w holds [gate | up] rows interleaved in blocks of 16 (gate_up_interleave) and out [M, N/2]
    receives bf16(gelu_tanh(gate)) * up."""
    M = x2.shape[0]
    gelu = 2 if gelu == "gated" else int(gelu)
    if out is None:
        No = N // 2 if gelu == 2 else N
        out = torch.empty(M, _pad8(No), dtype=torch.float32 if out_f32 else BF16, device=x2.device)[:, :No]
    ln_mom, ln_c = ln if ln is not None else (None, None)
    tT, tH, tD = tiles if tiles is not None else (0, 0, 0)
    if ln_rows is not None:
        st, eps, rms, c, mom_out = ln_rows
        assert ln is None and st.shape[0] >= M and st.is_contiguous()
        rc = lib().vt_gemm_fused_lnstats(
            _stream(), x2.data_ptr(), x2.stride(0), w.data_ptr(), ldw, M, N, K, _ptr(bias), out.data_ptr(),
            out.stride(0) if tiles is None else 0, int(tiles is None and out.dtype == torch.float32), int(gelu),
            _ptr(res), 0 if res is None else res.stride(0), int(res_period), int(res is not None and res.dtype == BF16),
            _ptr(out2), 0 if out2 is None else out2.stride(0), _ptr(stats_out), st.data_ptr(), st.shape[1],
            float(eps), int(rms), c.data_ptr(), _ptr(mom_out), tT, tH, tD, _ptr(ws),
            0 if ws is None else ws.numel() * ws.element_size())
        check(rc, "vt_gemm_fused_lnstats")
        return out
    rc = lib().vt_gemm_fused_ws(_stream(), x2.data_ptr(), x2.stride(0), w.data_ptr(), ldw, M, N, K, _ptr(bias),
                                out.data_ptr(), out.stride(0) if tiles is None else 0,
                                int(tiles is None and out.dtype == torch.float32), int(gelu), _ptr(res),
                                0 if res is None else res.stride(0), int(res_period),
                                int(res is not None and res.dtype == BF16), _ptr(out2),
                                0 if out2 is None else out2.stride(0), _ptr(stats_out), _ptr(ln_mom), _ptr(ln_c),
                                tT, tH, tD, _ptr(ws), 0 if ws is None else ws.numel() * ws.element_size())
    check(rc, "vt_gemm_fused_ws")
    return out


def gate_up_interleave(t, F):
    """Rows (or entries) [gate 0..F) | up 0..F) of a gated MLP's up projection, reordered into blocks of 16
    gate rows followed by the matching 16 up rows (the layout gemm(gelu="gated") reads)."""
    assert t.shape[0] == 2 * F and F % 16 == 0
    g, u = t[:F], t[F:]
    return torch.stack([g.reshape(F // 16, 16, *t.shape[1:]), u.reshape(F // 16, 16, *t.shape[1:])], 1).reshape(t.shape)


def _pad16(n):
    return (n + 15) // 16 * 16


def quant_rows(x2, q=None, s=None):
    """Per-token int8 quantisation (vt_quant_rows; the reference's quant_rows, moondream/gpu/hgemm.py:10-16):
    x2 bf16 [M, K] -> (q int8 [M, K] with a 16-byte row pitch, s fp32 [M])."""
    M, K = x2.shape
    if q is None:
        q = torch.empty(M, _pad16(K + I8_PAD), dtype=torch.int8, device=x2.device)[:, :K]
    if s is None:
        s = torch.empty(M, dtype=torch.float32, device=x2.device)
    rc = lib().vt_quant_rows(_stream(), x2.data_ptr(), x2.stride(0), M, K, q.data_ptr(), q.stride(0), s.data_ptr())
    check(rc, "vt_quant_rows")
    return q, s


def layer_norm_quant(x2, w, b, eps, q, s, out=None):
    """LayerNorm of x2 [M, N] (fp32 or bf16) fused with the per-token int8 quantisation of its bf16 output
    (vt_layernorm_quant): fills q int8 [M, N] and s fp32 [M] (and the bf16 output `out` when given)."""
    M, N = x2.shape
    rc = lib().vt_layernorm_quant(_stream(), x2.data_ptr(), x2.stride(0), int(x2.dtype == BF16), w.data_ptr(),
                                  b.data_ptr(), M, N, float(eps), q.data_ptr(), q.stride(0), s.data_ptr(), _ptr(out),
                                  0 if out is None else out.stride(0))
    check(rc, "vt_layernorm_quant")
    return q, s


def gemm_i8(q, sx, wq, ldw, K, N, sw, bias=None, gelu=False, res=None, out=None, out_f32=False, ws=None):
    """out[M, N] = ((float)(q . wq^T) * sx[m]) * sw[n] + bias (+ GELU-tanh on the fp32 value) (+ res), the W8A8
    GEMM vt_gemm_i8 (the reference's i8gemm_launch, moondream/gpu/hip/i8gemm.hip:480-533)."""
    M = q.shape[0]
    if out is None:
        out = torch.empty(M, _pad8(N), dtype=torch.float32 if out_f32 else BF16, device=q.device)[:, :N]
    rc = lib().vt_gemm_i8(_stream(), q.data_ptr(), q.stride(0), wq.data_ptr(), ldw, sx.data_ptr(), sw.data_ptr(),
                          M, N, K, _ptr(bias), out.data_ptr(), out.stride(0), int(out.dtype == torch.float32),
                          int(gelu), _ptr(res), 0 if res is None else res.stride(0),
                          int(res is not None and res.dtype == BF16), _ptr(ws),
                          0 if ws is None else ws.numel() * ws.element_size())
    check(rc, "vt_gemm_i8")
    return out


# Bytes of padding per int8 weight / activation row, the reference's HGEMM_WPAD switch (moondream/gpu/hgemm.py:85,
# 104-110, default 64 there against DRAM-channel aliasing of power-of-two rows).  Measured on B200 (text
# decoder, graph replay): 64 bytes made the int8 prefill 3.60 -> 3.64-3.71 ms, so the default here is 0.
I8_PAD = int(os.environ.get("VT_I8_WPAD", "0"))


class I8Lin:
    """W8A8 int8 linear layer, the mirror of the reference's HI8Lin (moondream/gpu/hgemm.py:95-137): weights
    quantised once per output channel, s = max(max|w|, 1e-8) / 127 and wq = round-half-even(w / s) clamped to
    +-127 (hgemm.py:100-103), kept [N, K] with a 16-byte row pitch; each call quantises its activation rows
    (vt_quant_rows, or takes `pre` = (q, s) already quantised, as md2fast.py:174 shares the LN output's) and
    runs vt_gemm_i8 (GELU-tanh on the fp32 value when gelu)."""
    fused_gelu = True

    def __init__(self, weight, bias, device):
        w = torch.as_tensor(weight).to(device=device, dtype=torch.float32)
        self.N, self.K = w.shape
        # true division, as the reference's numpy statement of these numerics does (moondream/npu/p4/
        # pack_i8.py:56-61): torch on CUDA would turn a division by a Python scalar into a multiplication
        # by its rounded reciprocal, one ulp off for some channels
        s = w.abs().amax(dim=1).clamp_min(1e-8)
        s = s / torch.full_like(s, 127.0)
        wq = (w / s[:, None]).round().clamp(-127, 127).to(torch.int8)
        self.ldw = _pad16(self.K + I8_PAD)
        self.wq = torch.zeros(self.N, self.ldw, dtype=torch.int8, device=device)
        self.wq[:, :self.K] = wq
        self.sw = s.contiguous()
        self.b = None if bias is None else torch.as_tensor(bias).to(device=device, dtype=torch.float32).contiguous()

    def quant(self, x2, q=None, s=None):
        return quant_rows(x2, q, s)

    def __call__(self, x, gelu=False, res=None, pre=None, out=None, out_f32=False, ws=None):
        """x [..., K] (any leading shape, as hgemm.py:127 reshapes it) -> [..., N]; `out` (2-D) is filled and
        returned as given."""
        shp = x.shape
        assert shp[-1] == self.K, (shp, self.K)
        q, sx = pre if pre is not None else quant_rows(as_gemm_operand(x.reshape(-1, self.K)))
        r2 = None if res is None else res.reshape(-1, self.N)
        y = gemm_i8(q, sx, self.wq, self.ldw, self.K, self.N, self.sw, self.b, gelu=gelu, res=r2, out=out,
                    out_f32=out_f32, ws=ws)
        return y if out is not None else y.reshape(*shp[:-1], self.N)


def gemm_workspace(M, N, device):
    """Zero-filled split-K workspace for GEMMs with outputs up to M x N (vt_gemm_ws_bytes)."""
    return torch.zeros(max(lib().vt_gemm_ws_bytes(M, N), 16), dtype=torch.uint8, device=device)


def row_stats(x2, stats, xb=None):
    """Chunk statistics (and the bf16 copy xb) of an fp32 residual stream x2 [M, N] for a folded LayerNorm."""
    M, N = x2.shape
    rc = lib().vt_rowstats(_stream(), x2.data_ptr(), x2.stride(0), _ptr(xb), 0 if xb is None else xb.stride(0),
                           stats.data_ptr(), M, N)
    check(rc, "vt_rowstats")
    return stats


def row_moments(stats, eps, out):
    """(mean, rstd) per row [M, 2] from chunk statistics [M, nchunk, 2] (the ln input of gemm)."""
    M, nchunk = stats.shape[0], stats.shape[1]
    rc = lib().vt_row_moments(_stream(), stats.data_ptr(), M, nchunk, float(eps), out.data_ptr())
    check(rc, "vt_row_moments")
    return out


def row_rms(stats, eps, out):
    """(0, rstd) per row [M, 2] of an RMSNorm from chunk statistics [M, nchunk, 2] (vt_row_rms)."""
    M, nchunk = stats.shape[0], stats.shape[1]
    rc = lib().vt_row_rms(_stream(), stats.data_ptr(), M, nchunk, float(eps), out.data_ptr())
    check(rc, "vt_row_rms")
    return out


def rglru_fold(G, softplus_a, rms_moments, rms_gamma, state, x, xb, stats, c, first):
    """RG-LRU step with its RMSNorm folded into the gate GEMM (vt_rglru_fold): state, x updated in place; xb and
    stats receive the bf16 copy and chunk statistics of the new x.  softplus_a [W] = softplus(a_param)."""
    M, W = x.shape
    rc = lib().vt_rglru_fold(_stream(), G.data_ptr(), G.stride(0), softplus_a.data_ptr(), rms_moments.data_ptr(),
                             rms_gamma.data_ptr(), state.data_ptr(), state.stride(0), x.data_ptr(), x.stride(0),
                             xb.data_ptr(), xb.stride(0), stats.data_ptr(), M, W, float(c), int(bool(first)))
    check(rc, "vt_rglru_fold")


def fold_layernorm(w, b, gamma, beta):
    """Weights of a linear with the preceding LayerNorm's affine folded in: (bf16 W * diag(gamma),
    fp32 c = row sums of that bf16 matrix, fp32 b + W beta).  w [N, K], b [N], gamma / beta [K] (fp32)."""
    w = torch.as_tensor(w).float()
    wf = (w * torch.as_tensor(gamma).float()[None, :]).to(BF16)
    c = wf.float().sum(dim=1)
    bf = torch.as_tensor(b).float() + w @ torch.as_tensor(beta).float()
    return wf, c, bf


class VtLin:
    """bf16 tcgen05 GEMM with fused bias, GELU-tanh and residual epilogues; weights kept (N, K)-major
    with the row pitch padded to a multiple of 8 elements (16 B, the TMA stride rule), K=588 included."""
    fused_gelu = True
    fused_res = True

    def __init__(self, weight, bias, dtype=BF16, device=None):
        w = weight.detach()
        dev = torch.device(device) if device is not None else (w.device if w.is_cuda else torch.device("cuda"))
        self.N, self.K = w.shape
        self.ldw = _pad8(self.K)
        self.wbuf = torch.zeros(self.N, self.ldw, dtype=BF16, device=dev)
        self.wbuf[:, :self.K] = w.to(dev, BF16)
        self.w = self.wbuf[:, :self.K]
        self.b = None if bias is None else bias.detach().to(dev, torch.float32).contiguous()
        self.dtype = dtype

    def __call__(self, x, gelu=False, res=None):
        shp = x.shape
        assert shp[-1] == self.K, (shp, self.K)
        x2 = as_gemm_operand(x.reshape(-1, self.K))
        if res is None:
            out = gemm(x2, self.wbuf, self.ldw, self.K, self.N, self.b, gelu=gelu)
        else:
            if gelu:
                raise ValueError("VtLin: gelu and res are not fused together")
            r2 = res.reshape(-1, self.N)
            if r2.stride(-1) != 1 or r2.stride(0) % 8 or r2.data_ptr() % 16 or r2.dtype not in (BF16, torch.float32):
                r2 = r2.to(BF16 if r2.dtype != torch.float32 else torch.float32).contiguous()
            out = gemm(x2, self.wbuf, self.ldw, self.K, self.N, self.b, res=r2, out_f32=(r2.dtype == torch.float32))
        return out.reshape(*shp[:-1], self.N)


def attn_tiles(B, T, H, D, device):
    """Zero-filled attention-tile buffer (see vt_attn_tiles_bytes in include/vt_b200.h)."""
    n = lib().vt_attn_tiles_bytes(B, T, H, D)
    if n <= 0:
        raise ValueError(f"attention tiles: unsupported shape B={B} T={T} H={H} D={D}")
    return torch.zeros(n // 2, dtype=BF16, device=device)


def attention_tiles(tiles, B, T, H, D, out, scale=None):
    """tcgen05 attention from an attention-tile buffer into out [B*T, >= H*D] (row pitch out.stride(0))."""
    rc = lib().vt_attn_tiles_fwd(_stream(), tiles.data_ptr(), out.data_ptr(), B, T, H, D, T * out.stride(0),
                                 out.stride(0), D, D ** -0.5 if scale is None else scale)
    check(rc, "vt_attn_tiles_fwd")
    return out


def gemm_qkv_tiles(x2, w, ldw, K, bias, tiles, T, H, D):
    """QKV projection written straight into attention tiles (the tower's fused path)."""
    rc = lib().vt_gemm_qkv_tiles(_stream(), x2.data_ptr(), x2.stride(0), w.data_ptr(), ldw, _ptr(bias),
                                 tiles.data_ptr(), x2.shape[0], K, T, H, D)
    check(rc, "vt_gemm_qkv_tiles")
    return tiles


class VtAttn:
    """Flash attention for one (H, T, D) problem, the contract of hattn.Attn (hattn.py:17-37): q, k, v are
    (B, H, T, D) views (any strides over B / H / T, contiguous D) -- e.g. the chunks of a fused QKV
    output -- and the result is (B, T, H*D).  Like hattn.Attn holds its V^T buffer, this object holds
    the attention-tile buffer the pack kernel fills (one per batch size)."""

    def __init__(self, H, T, D, device="cuda"):
        self.H, self.T, self.D = H, T, D
        self.scale = D ** -0.5
        self.device = device
        self._tiles = {}

    def __call__(self, q, k, v, out=None):
        B, H, T, D = q.shape
        assert (H, T, D) == (self.H, self.T, self.D), (q.shape, self.H, self.T, self.D)
        assert q.stride(3) == 1 and k.stride(3) == 1 and v.stride(3) == 1
        if out is None:
            out = torch.empty(B, T, H * D, dtype=BF16, device=q.device)
        tiles = self._tiles.get(B)
        if tiles is None:
            tiles = self._tiles[B] = attn_tiles(B, T, H, D, q.device)
        rc = lib().vt_attn_pack(_stream(), q.data_ptr(), k.data_ptr(), v.data_ptr(), tiles.data_ptr(), B, T, H, D,
                                q.stride(0), q.stride(2), q.stride(1), k.stride(0), k.stride(2), k.stride(1),
                                v.stride(0), v.stride(2), v.stride(1))
        check(rc, "vt_attn_pack")
        rc = lib().vt_attn_tiles_fwd(_stream(), tiles.data_ptr(), out.data_ptr(), B, T, H, D, out.stride(0),
                                     out.stride(1), D, self.scale)
        check(rc, "vt_attn_tiles_fwd")
        return out


def layer_norm(x2, w, b, eps, out=None, out_f32=False):
    M, N = x2.shape
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if out_f32 else BF16, device=x2.device)
    rc = lib().vt_layernorm(_stream(), x2.data_ptr(), x2.stride(0), int(x2.dtype == BF16), w.data_ptr(), b.data_ptr(),
                            out.data_ptr(), out.stride(0), int(out.dtype == torch.float32), M, N, float(eps))
    check(rc, "vt_layernorm")
    return out


def rms_norm(x2, w, eps, out=None, out_f32=False):
    M, N = x2.shape
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if out_f32 else BF16, device=x2.device)
    rc = lib().vt_rmsnorm(_stream(), x2.data_ptr(), x2.stride(0), int(x2.dtype == BF16), w.data_ptr(),
                          out.data_ptr(), out.stride(0), int(out.dtype == torch.float32), M, N, float(eps))
    check(rc, "vt_rmsnorm")
    return out


PIX_KIND = {torch.float32: 0, BF16: 1, torch.uint8: 2}


def im2col(pix, patch, out):
    """pix [B, C, S, S] fp32/bf16 (NCHW) or uint8 [B, S, S, C] (NHWC) -> out [B*(S/P)^2, >= C*P*P] bf16."""
    kind = PIX_KIND[pix.dtype]
    pix = pix.contiguous()
    if kind == 2:
        B, S, _, C = pix.shape
    else:
        B, C, S, _ = pix.shape
    rc = lib().vt_im2col(_stream(), pix.data_ptr(), kind, B, C, S, patch, out.data_ptr(), out.stride(0))
    check(rc, "vt_im2col")
    return out


def crop_combine(feats, out):
    """feats [n, T, W] bf16 -> out [T, 2W]: global crop 0 then the mean of crops 1..n-1."""
    n, T, W = feats.shape
    rc = lib().vt_crop_combine(_stream(), feats.data_ptr(), feats.stride(0), feats.stride(1), n, T, W,
                               out.data_ptr(), out.stride(0))
    check(rc, "vt_crop_combine")
    return out


def rglru(G, softplus_a, u, state, x, c, first):
    """RG-LRU step on the bf16 input u [M, W]: state [M, W] and x [M, W] fp32 updated in place; softplus_a [W] =
    softplus(a_param) per channel."""
    M, W = x.shape
    rc = lib().vt_rglru(_stream(), G.data_ptr(), G.stride(0), softplus_a.data_ptr(), u.data_ptr(), u.stride(0),
                        state.data_ptr(), state.stride(0), x.data_ptr(), x.stride(0), M, W, float(c), int(bool(first)))
    check(rc, "vt_rglru")


def ssm_step(yg, xx, hist, h, conv_w, conv_b, softplus_a, wx, bx, wa, ba, z, first, gelu_y=False):
    """TAPNext++ recurrent step (vt_ssm_step): yg, xx [R, W] bf16 views; hist = (x_(t-3), x_(t-2), x_(t-1))
    bf16 [R, W] -- x_t is written over hist[0], so the caller rotates; h [R, W] fp32 state in place;
    z [R, W] bf16 out.  gelu_y: yg is the raw y linear output and the kernel applies its GELU-tanh."""
    R, W = z.shape
    old, mid, new = hist
    rc = lib().vt_ssm_step(_stream(), yg.data_ptr(), xx.data_ptr(), yg.stride(0), old.data_ptr(), mid.data_ptr(),
                           new.data_ptr(), old.stride(0), h.data_ptr(), h.stride(0), conv_w.data_ptr(),
                           conv_b.data_ptr(), softplus_a.data_ptr(), wx.data_ptr(), bx.data_ptr(), wa.data_ptr(),
                           ba.data_ptr(), z.data_ptr(), z.stride(0), R, W, int(bool(first)), int(bool(gelu_y)))
    check(rc, "vt_ssm_step")
    return z


def gated_gelu_mul(G, out):
    """out [R, F] = gelu_tanh(G[:, :F]) * G[:, F:] in bf16 (vt_gated_gelu_mul)."""
    R, F = out.shape
    rc = lib().vt_gated_gelu_mul(_stream(), G.data_ptr(), G.stride(0), out.data_ptr(), out.stride(0), R, F)
    check(rc, "vt_gated_gelu_mul")
    return out


def gelu_erf(x):
    """Exact GELU in place on a bf16 [R, N] matrix (vt_gelu_erf)."""
    R, N = x.shape
    rc = lib().vt_gelu_erf(_stream(), x.data_ptr(), x.stride(0), R, N)
    check(rc, "vt_gelu_erf")
    return x


def rope_qkv(qkv, pos0, cos_t, sin_t, q, kc, vc):
    """vt_rope_qkv: qkv [n, 3*H*64] bf16 -> q [H, n, 64]; k, v into the caches kc / vc [H, ctx, 64]."""
    n = qkv.shape[0]
    H, ctx = kc.shape[0], kc.shape[1]
    rc = lib().vt_rope_qkv(_stream(), qkv.data_ptr(), qkv.stride(0), n, H, int(pos0), cos_t.data_ptr(), sin_t.data_ptr(),
                           q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ctx)
    check(rc, "vt_rope_qkv")
    return q


def attn_causal(q, kc, vc, pos0, out, scale=None):
    """vt_attn_causal: q [H, n, 64] at positions pos0 .. over the caches -> out [n, H*64] bf16."""
    H, n, hd = q.shape
    ctx = kc.shape[1]
    s = float(hd ** -0.5 if scale is None else scale)
    rc = lib().vt_attn_causal(_stream(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), n, H, int(pos0), ctx, s,
                              out.data_ptr(), out.stride(0))
    check(rc, "vt_attn_causal")
    return out


def head_linear(x2, wt, bias, out):
    """out [M, N] fp32 = x2 [M, K] (bf16 or fp32, unit column stride) . wt [K, N] fp32 + bias (vt_head_linear)."""
    M, K = x2.shape
    N = out.shape[1]
    rc = lib().vt_head_linear(_stream(), x2.data_ptr(), x2.stride(0), int(x2.dtype == BF16), wt.data_ptr(), wt.stride(0),
                              _ptr(bias), out.data_ptr(), out.stride(0), M, N, K)
    check(rc, "vt_head_linear")
    return out


def head_ln_gelu(y2, gamma, beta, eps):
    """In place on y2 [rows, N] fp32: LayerNorm (gamma / beta [groups, N], row r uses group r % groups) then the
    exact GELU (vt_head_ln_gelu)."""
    rows, N = y2.shape
    rc = lib().vt_head_ln_gelu(_stream(), y2.data_ptr(), y2.stride(0), rows, N, gamma.data_ptr(), beta.data_ptr(),
                               gamma.shape[0], float(eps))
    check(rc, "vt_head_ln_gelu")
    return y2


def soft_argmax(logits, bins, window, temperature, tracks):
    """tracks [Q, 2] = windowed soft-argmax of logits [Q, 2 * bins] per axis (vt_soft_argmax)."""
    rc = lib().vt_soft_argmax(_stream(), logits.data_ptr(), logits.stride(0), logits.shape[0], int(bins), int(window),
                              float(temperature), tracks.data_ptr(), tracks.stride(0))
    check(rc, "vt_soft_argmax")
    return tracks
