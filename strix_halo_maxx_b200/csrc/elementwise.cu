// Memory-bound kernels of the tower: LayerNorm, patch im2col (+ pixel normalisation), multi-crop
// combine and the RG-LRU recurrence.  All use 128-bit global accesses where the layout allows.
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace ew {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 load4(const void* base, long long idx, int in_bf16) {
  if (in_bf16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + idx);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
  }
  return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
}
__device__ __forceinline__ void store4(void* base, long long idx, float4 v, int out_f32) {
  if (out_f32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + idx) = v;
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(base) + idx) = make_uint2(pack_bf2(v.x, v.y), pack_bf2(v.z, v.w));
  }
}

// The per-float4 terms of the LayerNorm sums and the affine step, written with explicit roundings so the
// warp-per-row and CTA-per-row kernels below produce the same bits for a row (no compiler-chosen FMA
// contraction differs between them).
__device__ __forceinline__ float sum4(float4 v) { return __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)); }
__device__ __forceinline__ float sq4(float4 v, float mean) {
  const float a = __fsub_rn(v.x, mean), b = __fsub_rn(v.y, mean), c = __fsub_rn(v.z, mean), d = __fsub_rn(v.w, mean);
  return __fadd_rn(__fmaf_rn(a, a, __fmul_rn(b, b)), __fmaf_rn(c, c, __fmul_rn(d, d)));
}
__device__ __forceinline__ float4 norm4(float4 v, float mean, float rstd, float4 g, float4 b) {
  return make_float4(__fmaf_rn(__fmul_rn(__fsub_rn(v.x, mean), rstd), g.x, b.x),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.y, mean), rstd), g.y, b.y),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.z, mean), rstd), g.z, b.z),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.w, mean), rstd), g.w, b.w));
}

// LayerNorm over rows of N (N % 4 == 0, N <= 4096): one warp per row, the row held in registers
// (two-pass mean / variance in fp32), y = (x - mean) * rsqrt(var + eps) * gamma + beta.
// Follows F.layer_norm as md2fast.py:43-44 calls it.
// RMS = true gives RMSNorm instead: y = x * rsqrt(mean(x^2) + eps) * gamma (+ beta when given).
constexpr int LN_MAXV = 32;  // float4 per lane, upper bound (N <= 4096)
// QUANT = true: the row is also quantised per token for the int8 GEMM (vt_layernorm_quant): y rounded to bf16
// (as vt_layernorm's bf16 output), s = max(max |y|, 1e-5) / 127, q = trunc(y / s +- 0.5) -- the same numbers
// vt_quant_rows makes from vt_layernorm's output; y itself is stored only when y != null.
template <int MAXV, bool RMS, bool QUANT = false>
__global__ void __launch_bounds__(256) layernorm_kernel(const void* x, long long ldx, int in_bf16, const float* g,
                                                        const float* bta, void* y, long long ldy, int out_f32, int M,
                                                        int N, float eps, int8_t* qout, long long ldq, float* qs) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= M) return;
  const int nv = N / 4;
  float4 v[MAXV];
  // the whole row is loaded before any arithmetic (the input-type test outside the loop), so all of a
  // lane's loads are in flight together
  if (in_bf16) {
#pragma unroll
    for (int i = 0; i < MAXV; i++)
      if (i * 32 + lane < nv) v[i] = load4(x, row * ldx + 4LL * (i * 32 + lane), 1);
  } else {
#pragma unroll
    for (int i = 0; i < MAXV; i++)
      if (i * 32 + lane < nv) v[i] = load4(x, row * ldx + 4LL * (i * 32 + lane), 0);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; i++)
    if (i * 32 + lane < nv) s = __fadd_rn(s, sum4(v[i]));
  const float mean = RMS ? 0.f : warp_sum(s) / (float)N;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    const int c = (i * 32 + lane);
    if (c < nv) q = __fadd_rn(q, sq4(v[i], mean));
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)N + eps);
  // all gamma / beta loads before the first store (the compiler may not move a load past a store to y)
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    const int c = (i * 32 + lane);
    if (c < nv) {
      const float4 gg = *reinterpret_cast<const float4*>(g + 4 * c);
      const float4 bb = bta ? *reinterpret_cast<const float4*>(bta + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = norm4(v[i], mean, rstd, gg, bb);
    }
  }
  if constexpr (QUANT) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; i++) {
      if (i * 32 + lane < nv) {
        v[i] = make_float4(bfround(v[i].x), bfround(v[i].y), bfround(v[i].z), bfround(v[i].w));
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = __fdiv_rn(fmaxf(amax, 1e-5f), 127.f);
    const float rsc = __frcp_rn(sc);
    auto q8 = [sc, rsc](float xv) -> uint32_t {
      const float t = div_rn_by(xv, sc, rsc);  // == xv / sc (IEEE)
      int qi = __float2int_rz(__fadd_rn(t, t >= 0.f ? 0.5f : -0.5f));
      qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
      return (uint32_t)qi & 0xffu;
    };
#pragma unroll
    for (int i = 0; i < MAXV; i++) {
      const int c = i * 32 + lane;
      if (c < nv) {
        *reinterpret_cast<uint32_t*>(qout + row * ldq + 4LL * c) =
            q8(v[i].x) | (q8(v[i].y) << 8) | (q8(v[i].z) << 16) | (q8(v[i].w) << 24);
        if (y) store4(y, row * ldy + 4LL * c, v[i], 0);
      }
    }
    if (lane == 0) qs[row] = sc;
    return;
  }
  if (out_f32) {
#pragma unroll
    for (int i = 0; i < MAXV; i++)
      if (i * 32 + lane < nv) store4(y, row * ldy + 4LL * (i * 32 + lane), v[i], 1);
  } else {
#pragma unroll
    for (int i = 0; i < MAXV; i++)
      if (i * 32 + lane < nv) store4(y, row * ldy + 4LL * (i * 32 + lane), v[i], 0);
  }
}

// Row statistics for a folded LayerNorm: one warp per row of x (fp32, N % 32 == 0); lane l handles the
// 32-column chunks l, l+32, ...: stats[row][j] = (chunk mean, chunk sum of squared deviations), and xb
// (optional) receives the bf16 copy of x the folded GEMM reads.
__global__ void __launch_bounds__(256) rowstats_kernel(const float* __restrict__ x, long long ldx,
                                                       uint16_t* __restrict__ xb, long long ldxb,
                                                       float2* __restrict__ stats, int M, int N) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + warp;
  if (row >= M) return;
  const int nch = N / 32;
  for (int j = lane; j < nch; j += 32) {
    const float4* p = reinterpret_cast<const float4*>(x + row * ldx + 32LL * j);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 a = p[i];
      v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
    }
    float sm = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) sm += v[i];
    const float mean = sm * (1.f / 32.f);
    float m2 = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i++) m2 = fmaf(v[i] - mean, v[i] - mean, m2);
    stats[row * nch + j] = make_float2(mean, m2);
    if (xb) {
      uint4* q = reinterpret_cast<uint4*>(xb + row * ldxb + 32LL * j);
#pragma unroll
      for (int i = 0; i < 4; i++)
        q[i] = make_uint4(pack_bf2(v[8 * i], v[8 * i + 1]), pack_bf2(v[8 * i + 2], v[8 * i + 3]),
                          pack_bf2(v[8 * i + 4], v[8 * i + 5]), pack_bf2(v[8 * i + 6], v[8 * i + 7]));
    }
  }
}

// (mean, 1/sqrt(var + eps)) of every row from its nchunk per-32-column (mean, M2) pairs, merged with
// Chan's parallel formula (equal chunk counts).
// RMS = true: (0, 1 / sqrt(mean(x^2) + eps)) instead, the sum of squares merged from the same chunk statistics
// (sum over chunks of M2 + 32 mean^2) -- the RMSNorm of the TAPNext temporal block folded into its gate GEMM.
// A warp per RPW consecutive rows: lane j reads chunks j and j + 32 of each (coalesced, nchunk <= 64), all the
// warp's loads issued before the first sum (one row per warp left a warp with two loads and a long dependent
// tail, so the pass ran at ~1.2 TB/s on the tower's 94,770-row chunk), and each row's sums go through the same
// fixed shuffle tree, so a row's result does not depend on M, RPW or the other rows.
constexpr int RM_RPW = 4;
template <bool RMS>
__global__ void __launch_bounds__(256) row_moments_kernel(const float2* __restrict__ stats, int nchunk, int M,
                                                          float eps, float2* __restrict__ out) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const long long m0 = ((long long)blockIdx.x * 8 + (threadIdx.x >> 5)) * RM_RPW;
  if (m0 >= M) return;
  const float2 z = make_float2(0.f, 0.f);
  float2 v0[RM_RPW], v1[RM_RPW];
#pragma unroll
  for (int r = 0; r < RM_RPW; r++) {
    const bool in = m0 + r < M;
    const float2* st = stats + (m0 + r) * nchunk;
    v0[r] = in && lane < nchunk ? st[lane] : z;
    v1[r] = in && lane + 32 < nchunk ? st[lane + 32] : z;
  }
  const float cnt = 32.f * (float)nchunk;
  if (RMS) {
    float q[RM_RPW];
#pragma unroll
    for (int r = 0; r < RM_RPW; r++) q[r] = (v0[r].y + 32.f * v0[r].x * v0[r].x) + (v1[r].y + 32.f * v1[r].x * v1[r].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < RM_RPW; r++) q[r] += __shfl_xor_sync(0xffffffffu, q[r], o);
    if (lane < RM_RPW && m0 + lane < M) {
      float qq = q[0];
#pragma unroll
      for (int r = 1; r < RM_RPW; r++) qq = lane == r ? q[r] : qq;
      out[m0 + lane] = make_float2(0.f, rsqrtf(qq / cnt + eps));
    }
    return;
  }
  float s[RM_RPW], mu[RM_RPW], m2[RM_RPW];
#pragma unroll
  for (int r = 0; r < RM_RPW; r++) s[r] = v0[r].x + v1[r].x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RM_RPW; r++) s[r] += __shfl_xor_sync(0xffffffffu, s[r], o);
#pragma unroll
  for (int r = 0; r < RM_RPW; r++) {
    mu[r] = s[r] / (float)nchunk;
    const float d0 = v0[r].x - mu[r], d1 = v1[r].x - mu[r];
    m2[r] = (lane < nchunk ? v0[r].y + 32.f * d0 * d0 : 0.f) + (lane + 32 < nchunk ? v1[r].y + 32.f * d1 * d1 : 0.f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < RM_RPW; r++) m2[r] += __shfl_xor_sync(0xffffffffu, m2[r], o);
  if (lane < RM_RPW && m0 + lane < M) {
    float mm = mu[0], vv = m2[0];
#pragma unroll
    for (int r = 1; r < RM_RPW; r++) {
      mm = lane == r ? mu[r] : mm;
      vv = lane == r ? m2[r] : vv;
    }
    out[m0 + lane] = make_float2(mm, rsqrtf(vv / cnt + eps));
  }
}

// Patch im2col: pixels -> A[m, k] (bf16, pitch ldo) with m = crop*g*g + gy*g + gx and
// k = c*P*P + py*P + px (md2fast.py:149 permutation).  kind 0: fp32 NCHW values, 1: bf16 NCHW values,
// 2: uint8 NHWC 0..255 normalised by (u/255 - 0.5)/0.5 (md2fast.py:148).  One thread per P-pixel run.
__global__ void __launch_bounds__(256) im2col_kernel(const void* pix, int kind, int B, int C, int S, int P,
                                                     uint16_t* out, long long ldo) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int g = S / P;
  const long long total = (long long)B * g * g * C * P;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    long long r = i;
    const int py = (int)(r % P); r /= P;
    const int c = (int)(r % C); r /= C;
    const int gx = (int)(r % g); r /= g;
    const int gy = (int)(r % g); r /= g;
    const long long b = r;
    const long long m = b * g * g + (long long)gy * g + gx;
    const int y = gy * P + py;
    uint16_t* op = out + m * ldo + (long long)c * P * P + (long long)py * P;
    for (int px = 0; px < P; px++) {
      const int xx = gx * P + px;
      float val;
      if (kind == 0) {
        val = reinterpret_cast<const float*>(pix)[((b * C + c) * S + y) * (long long)S + xx];
      } else if (kind == 1) {
        val = bf2f(reinterpret_cast<const uint16_t*>(pix)[((b * C + c) * S + y) * (long long)S + xx]);
      } else {
        const float u = (float)reinterpret_cast<const uint8_t*>(pix)[((b * S + y) * (long long)S + xx) * C + c];
        val = (u / 255.0f - 0.5f) / 0.5f;
      }
      op[px] = f2bf(val);
    }
  }
}

// Multi-crop combine: out[t, :W] = f[0, t], out[t, W:2W] = mean_{i=1..n-1} f[i, t] (fp32 sum), bf16.
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* f, long long crop_stride, long long ldf,
                                                      int n_crops, int T, int W, uint16_t* out, long long ldo) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int nch = W / 8;
  const long long total = (long long)T * nch;
  const float inv = 1.0f / (float)(n_crops - 1);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / nch), c = (int)(i % nch) * 8;
    const uint4 g0 = *reinterpret_cast<const uint4*>(f + (long long)t * ldf + c);
    *reinterpret_cast<uint4*>(out + (long long)t * ldo + c) = g0;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 1; k < n_crops; k++) {
      const uint4 u = *reinterpret_cast<const uint4*>(f + k * crop_stride + (long long)t * ldf + c);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        acc[2 * e] += __uint_as_float(w[e] << 16);
        acc[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
      }
    }
    *reinterpret_cast<uint4*>(out + (long long)t * ldo + W + c) =
        make_uint4(pack_bf2(acc[0] * inv, acc[1] * inv), pack_bf2(acc[2] * inv, acc[3] * inv),
                   pack_bf2(acc[4] * inv, acc[5] * inv), pack_bf2(acc[6] * inv, acc[7] * inv));
  }
}

// RG-LRU step (tapnext/npu/r9/cpuemu.py:33-47) on the normalised input u, per element (m, n < W):
//   gx = sigmoid(G[m, n]), ga = sigmoid(G[m, W + n]), log_a = -c * ga * softplus_a[n]  (softplus(a_param))
//   h  = u * gx                                              (first frame)
//   h  = exp(log_a) * h0 + (u * gx) * sqrt(-expm1(2 log_a))   (later frames)
//   state <- h, x <- x + h     (u bf16; state and the residual stream x fp32, updated in place)

__global__ void __launch_bounds__(256) rglru_kernel(const float* G, long long ldg, const float* softplus_a,
                                                    const uint16_t* u, long long ldu, float* state, long long lds,
                                                    float* x, long long ldx, int M, int W, float c, int first) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int nv = W / 4;
  const long long total = (long long)M * nv;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / nv;
    const int n = (int)(i % nv) * 4;
    const float4 gx4 = *reinterpret_cast<const float4*>(G + m * ldg + n);
    const float4 ga4 = *reinterpret_cast<const float4*>(G + m * ldg + W + n);
    const float4 ap4 = *reinterpret_cast<const float4*>(softplus_a + n);
    float4 x4 = *reinterpret_cast<const float4*>(x + m * ldx + n);
    const uint2 u2 = *reinterpret_cast<const uint2*>(u + m * ldu + n);
    const float uv[4] = {__uint_as_float(u2.x << 16), __uint_as_float(u2.x & 0xffff0000u), __uint_as_float(u2.y << 16),
                         __uint_as_float(u2.y & 0xffff0000u)};
    float4 h4 = first ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(state + m * lds + n);
    const float gx[4] = {gx4.x, gx4.y, gx4.z, gx4.w}, ga[4] = {ga4.x, ga4.y, ga4.z, ga4.w};
    const float ap[4] = {ap4.x, ap4.y, ap4.z, ap4.w};
    float xv[4] = {x4.x, x4.y, x4.z, x4.w}, hv[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float h = rglru_elem(uv[e], gx[e], ga[e], ap[e], hv[e], c, first != 0);
      hv[e] = h;
      xv[e] += h;
    }
    *reinterpret_cast<float4*>(state + m * lds + n) = make_float4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<float4*>(x + m * ldx + n) = make_float4(xv[0], xv[1], xv[2], xv[3]);
  }
}

// The RG-LRU step with the temporal RMSNorm folded into the gate GEMM (TAPNext-style step, fold_ln): G holds
// rstd * (bf16(x) . (W gamma)^T) + b; the normed input the recurrence gates, t = bf16(x * rstd * gamma), is
// formed here from the fp32 stream.  Besides state and x += h it writes the bf16 copy of the new x and its
// per-32-column (mean, M2) statistics, the inputs of the next block's folded LayerNorm.  Thread = 4 columns;
// the 8 threads of a 32-column chunk are consecutive lanes (W % 32 == 0), so a chunk's statistics are a
// shuffle reduction over 8 lanes, and every lane of a warp runs the same number of iterations.
__global__ void __launch_bounds__(256) rglru_fold_kernel(const float* G, long long ldg, const float* softplus_a,
                                                         const float2* __restrict__ mom, const float* __restrict__ rms_g,
                                                         float* state, long long lds, float* x, long long ldx,
                                                         uint16_t* __restrict__ xb, long long ldxb,
                                                         float2* __restrict__ stats, int M, int W, float c, int first) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int nv = W / 4, nch = W / 32;
  const long long total = (long long)M * nv;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i - (threadIdx.x & 31) < total; i += stride) {
    const bool valid = i < total;  // whole 8-lane groups are valid or not (nv % 8 == 0)
    float xv[4] = {0.f, 0.f, 0.f, 0.f};
    long long m = 0;
    int n = 0;
    if (valid) {
      m = i / nv;
      n = (int)(i % nv) * 4;
      const float4 gx4 = *reinterpret_cast<const float4*>(G + m * ldg + n);
      const float4 ga4 = *reinterpret_cast<const float4*>(G + m * ldg + W + n);
      const float4 ap4 = *reinterpret_cast<const float4*>(softplus_a + n);
      const float4 rg4 = *reinterpret_cast<const float4*>(rms_g + n);
      const float4 x4 = *reinterpret_cast<const float4*>(x + m * ldx + n);
      const float4 h4 = first ? make_float4(0.f, 0.f, 0.f, 0.f) : *reinterpret_cast<const float4*>(state + m * lds + n);
      const float rstd = mom[m].y;
      const float gx[4] = {gx4.x, gx4.y, gx4.z, gx4.w}, ga[4] = {ga4.x, ga4.y, ga4.z, ga4.w};
      const float ap[4] = {ap4.x, ap4.y, ap4.z, ap4.w}, rg[4] = {rg4.x, rg4.y, rg4.z, rg4.w};
      const float hv0[4] = {h4.x, h4.y, h4.z, h4.w};
      xv[0] = x4.x, xv[1] = x4.y, xv[2] = x4.z, xv[3] = x4.w;
      float hv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float u = bfround(xv[e] * rstd * rg[e]);  // the RMSNorm output, bf16 as the unfolded path stores it
        const float h = rglru_elem(u, gx[e], ga[e], ap[e], hv0[e], c, first != 0);
        hv[e] = h;
        xv[e] += h;
      }
      *reinterpret_cast<float4*>(state + m * lds + n) = make_float4(hv[0], hv[1], hv[2], hv[3]);
      *reinterpret_cast<float4*>(x + m * ldx + n) = make_float4(xv[0], xv[1], xv[2], xv[3]);
      *reinterpret_cast<uint2*>(xb + m * ldxb + n) = make_uint2(pack_bf2(xv[0], xv[1]), pack_bf2(xv[2], xv[3]));
    }
    // chunk statistics of the new x: mean, then the sum of squared deviations, over the chunk's 8 lanes
    float sm = (xv[0] + xv[1]) + (xv[2] + xv[3]);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    const float mean = sm * (1.f / 32.f);
    float q = 0.f;
#pragma unroll
    for (int e = 0; e < 4; e++) q = fmaf(xv[e] - mean, xv[e] - mean, q);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (valid && (threadIdx.x & 7) == 0) stats[m * nch + n / 32] = make_float2(mean, q);
  }
}

// Max over the 256 threads of a CTA; every thread gets the result.  buf: 8 floats of shared memory used by
// this reduction only.
__device__ __forceinline__ float cta_max(float v, float* buf) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = buf[0];
#pragma unroll
  for (int w = 1; w < 8; w++) t = fmaxf(t, buf[w]);
  return t;
}

// Sum of the per-float4 terms part[0 .. nv) in the warp-per-row kernel's order: "lane" l adds the terms
// l, l + 32, l + 64, ... one after another, then the 32 lane sums meet in warp_sum's butterfly.  Warp 0 does
// it; the result (divided by N) is broadcast through *out.
__device__ __forceinline__ float lane_order_mean(const float* part, int nv, int N, float* out) {
  __syncthreads();  // every term is in part[]
  if (threadIdx.x < 32) {
    float a = 0.f;
    for (int c = threadIdx.x; c < nv; c += 32) a = __fadd_rn(a, part[c]);
    a = warp_sum(a) / (float)N;
    if (threadIdx.x == 0) *out = a;
  }
  __syncthreads();
  return *out;
}

// The same LayerNorm / RMSNorm (and LayerNorm + quantisation) for few rows: one CTA of 256 threads per row,
// G float4 per thread (N <= 1024 G).  The warp-per-row kernel puts 8 rows in a CTA, so a few hundred rows
// (the text decoder's 730 / 32, TAPNext's 1280) occupy a fraction of the SMs and each row waits out its
// serial load -> reduce -> gamma / beta -> store chain on one warp.  The sums are formed in that kernel's
// order (lane_order_mean), so both kernels give the same bits for a row: results do not depend on how many
// rows a call has.
template <int G, bool RMS, bool QUANT>
__global__ void __launch_bounds__(256) norm_row_kernel(const void* x, long long ldx, int in_bf16, const float* g,
                                                       const float* bta, void* y, long long ldy, int out_f32, int N,
                                                       float eps, int8_t* qout, long long ldq, float* qs) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  __shared__ float part[1024];
  __shared__ float stat[2];
  __shared__ float red[8];
  const long long row = blockIdx.x;
  const int nv = N / 4;
  float4 v[G];
#pragma unroll
  for (int i = 0; i < G; i++) {
    const int c = i * 256 + threadIdx.x;
    v[i] = c < nv ? load4(x, row * ldx + 4LL * c, in_bf16) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mean = 0.f;
  if constexpr (!RMS) {
#pragma unroll
    for (int i = 0; i < G; i++) {
      const int c = i * 256 + threadIdx.x;
      if (c < nv) part[c] = sum4(v[i]);
    }
    mean = lane_order_mean(part, nv, N, &stat[0]);
  }
#pragma unroll
  for (int i = 0; i < G; i++) {
    const int c = i * 256 + threadIdx.x;
    if (c < nv) part[c] = sq4(v[i], mean);
  }
  const float rstd = rsqrtf(lane_order_mean(part, nv, N, &stat[1]) + eps);
#pragma unroll
  for (int i = 0; i < G; i++) {
    const int c = i * 256 + threadIdx.x;
    if (c < nv) {
      const float4 gg = *reinterpret_cast<const float4*>(g + 4 * c);
      const float4 bb = bta ? *reinterpret_cast<const float4*>(bta + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = norm4(v[i], mean, rstd, gg, bb);
    }
  }
  if constexpr (QUANT) {  // the rules of layernorm_kernel<.., QUANT = true>
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < G; i++) {
      if (i * 256 + threadIdx.x < nv) {
        v[i] = make_float4(bfround(v[i].x), bfround(v[i].y), bfround(v[i].z), bfround(v[i].w));
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
      }
    }
    amax = cta_max(amax, red);
    const float sc = __fdiv_rn(fmaxf(amax, 1e-5f), 127.f);
    const float rsc = __frcp_rn(sc);
    auto q8 = [sc, rsc](float xv) -> uint32_t {
      const float t = div_rn_by(xv, sc, rsc);  // == xv / sc (IEEE)
      int qi = __float2int_rz(__fadd_rn(t, t >= 0.f ? 0.5f : -0.5f));
      qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
      return (uint32_t)qi & 0xffu;
    };
#pragma unroll
    for (int i = 0; i < G; i++) {
      const int c = i * 256 + threadIdx.x;
      if (c < nv) {
        *reinterpret_cast<uint32_t*>(qout + row * ldq + 4LL * c) =
            q8(v[i].x) | (q8(v[i].y) << 8) | (q8(v[i].z) << 16) | (q8(v[i].w) << 24);
        if (y) store4(y, row * ldy + 4LL * c, v[i], 0);
      }
    }
    if (threadIdx.x == 0) qs[row] = sc;
    return;
  }
#pragma unroll
  for (int i = 0; i < G; i++) {
    const int c = i * 256 + threadIdx.x;
    if (c < nv) store4(y, row * ldy + 4LL * c, v[i], out_f32);
  }
}

// Rows below which the CTA-per-row kernel runs (measured: 730 x 2048 rows 3.4 us against 6.4 us warp per row;
// 1280 x 768 rows 3.7 us against 3.4 us);
// VT_LN_ROW_MAX overrides it (tuning switch).
static int row_kernel_max_m() {
  static const int v = [] {
    const char* e = getenv("VT_LN_ROW_MAX");
    return e ? atoi(e) : 1024;
  }();
  return v;
}

static int grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = (long long)sm_count() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

template <bool RMS>
static int norm_launch(const char* what, cudaStream_t st, const void* x, long long ldx, int in_bf16, const float* gamma,
                       const float* beta, void* y, long long ldy, int out_f32, int M, int N, float eps) {
  if (M < 0 || N < 0) return set_error(E_SHAPE, "%s: negative shape", what);
  if (M == 0) return OK;
  if (N == 0 || N % 4 || N > 4 * 32 * LN_MAXV) return set_error(E_SHAPE, "%s: N=%d unsupported", what, N);
  if (!x || !y || !gamma || (!RMS && !beta)) return set_error(E_SHAPE, "%s: null pointer", what);
  if (ldx < N || ldy < N || ldx % 4 || ldy % 4 || !aligned16(x) || !aligned16(y) || !aligned16(gamma) ||
      (beta && !aligned16(beta)))
    return set_error(E_SHAPE, "%s: pitches / alignment invalid", what);
  const long long blocks = ((long long)M + 7) / 8;
  if (blocks > 0x7fffffffLL) return set_error(E_SHAPE, "%s: M too large", what);
  if (M < row_kernel_max_m()) {
    const int g = (N / 4 + 255) / 256;
#define VT_LNR(G)                                                                                                  \
  launch_k(norm_row_kernel<G, RMS, false>, (unsigned)M, 256, 0, st, x, ldx, in_bf16, gamma, beta, y, ldy, out_f32, N, \
           eps, (int8_t*)nullptr, 0LL, (float*)nullptr)
    if (g <= 1) VT_LNR(1);
    else if (g <= 2) VT_LNR(2);
    else VT_LNR(4);
#undef VT_LNR
    return check_launch(what);
  }
  const int per_lane = (N / 4 + 31) / 32;
#define VT_LN(V)                                                                                                  \
  launch_k(layernorm_kernel<V, RMS>, (unsigned)blocks, 256, 0, st, x, ldx, in_bf16, gamma, beta, y, ldy, out_f32, M, N, \
           eps, (int8_t*)nullptr, 0LL, (float*)nullptr)
  if (per_lane <= 4) VT_LN(4);
  else if (per_lane <= 8) VT_LN(8);
  else if (per_lane <= 12) VT_LN(12);
  else if (per_lane <= 16) VT_LN(16);
  else VT_LN(32);
#undef VT_LN
  return check_launch(what);
}

static int ln_quant_launch(cudaStream_t st, const void* x, long long ldx, int in_bf16, const float* gamma,
                           const float* beta, int M, int N, float eps, int8_t* q, long long ldq, float* s, void* y,
                           long long ldy) {
  const char* what = "vt_layernorm_quant";
  if (M < 0 || N < 0) return set_error(E_SHAPE, "%s: negative shape", what);
  if (M == 0) return OK;
  if (N == 0 || N % 4 || N > 4 * 32 * LN_MAXV) return set_error(E_SHAPE, "%s: N=%d unsupported", what, N);
  if (!x || !q || !s || !gamma || !beta) return set_error(E_SHAPE, "%s: null pointer", what);
  if (ldx < N || ldx % 4 || ldq < N || ldq % 4 || !aligned16(x) || !aligned16(gamma) || !aligned16(beta) ||
      (reinterpret_cast<uintptr_t>(q) & 3) || (y && (ldy < N || ldy % 4 || !aligned16(y))))
    return set_error(E_SHAPE, "%s: pitches / alignment invalid", what);
  const long long blocks = ((long long)M + 7) / 8;
  if (blocks > 0x7fffffffLL) return set_error(E_SHAPE, "%s: M too large", what);
  if (M < row_kernel_max_m()) {
    const int g = (N / 4 + 255) / 256;
#define VT_LNQR(G)                                                                                                  \
  launch_k(norm_row_kernel<G, false, true>, (unsigned)M, 256, 0, st, x, ldx, in_bf16, gamma, beta, y, ldy, 0, N, eps, \
           q, ldq, s)
    if (g <= 1) VT_LNQR(1);
    else if (g <= 2) VT_LNQR(2);
    else VT_LNQR(4);
#undef VT_LNQR
    return check_launch(what);
  }
  const int per_lane = (N / 4 + 31) / 32;
#define VT_LNQ(V)                                                                                                \
  launch_k(layernorm_kernel<V, false, true>, (unsigned)blocks, 256, 0, st, x, ldx, in_bf16, gamma, beta, y, ldy, 0, \
           M, N, eps, q, ldq, s)
  if (per_lane <= 4) VT_LNQ(4);
  else if (per_lane <= 8) VT_LNQ(8);
  else if (per_lane <= 16) VT_LNQ(16);
  else VT_LNQ(32);
#undef VT_LNQ
  return check_launch(what);
}
}  // namespace ew
}  // namespace vt

extern "C" {

// y[M, N] = LayerNorm(x[M, N]) * gamma + beta.  x fp32 (or bf16 when in_bf16), y bf16 (or fp32 when
// out_f32).  N % 4 == 0, N <= 4096; pitches multiples of 4 elements, 16-byte bases.
int vt_layernorm(cudaStream_t st, const void* x, long long ldx, int in_bf16, const float* gamma, const float* beta,
                 void* y, long long ldy, int out_f32, int M, int N, float eps) {
  return vt::ew::norm_launch<false>("vt_layernorm", st, x, ldx, in_bf16, gamma, beta, y, ldy, out_f32, M, N, eps);
}

// LayerNorm fused with the per-token int8 quantisation of its bf16 output (vt_quant_rows' numbers): q[M, N]
// int8 (pitch ldq bytes, a multiple of 4), s[M]; y (bf16, pitch ldy) receives the bf16 output when not null.
int vt_layernorm_quant(cudaStream_t st, const void* x, long long ldx, int in_bf16, const float* gamma,
                       const float* beta, int M, int N, float eps, int8_t* q, long long ldq, float* s, uint16_t* y,
                       long long ldy) {
  return vt::ew::ln_quant_launch(st, x, ldx, in_bf16, gamma, beta, M, N, eps, q, ldq, s, y, ldy);
}

// y = x * rsqrt(mean(x^2) + eps) * gamma (RMSNorm), same layout rules as vt_layernorm.
int vt_rmsnorm(cudaStream_t st, const void* x, long long ldx, int in_bf16, const float* gamma, void* y, long long ldy,
               int out_f32, int M, int N, float eps) {
  return vt::ew::norm_launch<true>("vt_rmsnorm", st, x, ldx, in_bf16, gamma, nullptr, y, ldy, out_f32, M, N, eps);
}

// Per-32-column chunk (mean, M2) of every row of x[M, N] (fp32, N % 32 == 0) into stats[M][N/32] (float
// pairs), and optionally the bf16 copy xb: the inputs of a LayerNorm folded into vt_gemm_fused.
int vt_rowstats(cudaStream_t st, const float* x, long long ldx, uint16_t* xb, long long ldxb, float* stats, int M,
                int N) {
  using namespace vt;
  if (M < 0 || N <= 0 || N % 32) return set_error(E_SHAPE, "vt_rowstats: N=%d must be a positive multiple of 32", N);
  if (M == 0) return OK;
  if (!x || !stats || ldx < N || ldx % 4 || !aligned16(x) || (reinterpret_cast<uintptr_t>(stats) & 7) ||
      (xb && (ldxb < N || ldxb % 8 || !aligned16(xb))))
    return set_error(E_SHAPE, "vt_rowstats: pitches / alignment invalid");
  const long long blocks = ((long long)M + 7) / 8;
  if (blocks > 0x7fffffffLL) return set_error(E_SHAPE, "vt_rowstats: M too large");
  launch_k(ew::rowstats_kernel, (unsigned)blocks, 256, 0, st, x, ldx, xb, ldxb, reinterpret_cast<float2*>(stats), M, N);
  return check_launch("vt_rowstats");
}

// Row moments for a folded LayerNorm: moments[m] = (mean, rsqrt(var + eps)) of row m (N = 32 * nchunk
// columns) from the chunk statistics vt_rowstats / vt_gemm_fused(stats_out) wrote.
int vt_row_moments(cudaStream_t st, const float* stats, int M, int nchunk, float eps, float* moments) {
  using namespace vt;
  if (M < 0 || nchunk <= 0) return set_error(E_SHAPE, "vt_row_moments: bad shape");
  if (M == 0) return OK;
  if (!stats || !moments || (reinterpret_cast<uintptr_t>(stats) & 7) || (reinterpret_cast<uintptr_t>(moments) & 7))
    return set_error(E_SHAPE, "vt_row_moments: pointers must be 8-byte aligned");
  if (nchunk > 64) return set_error(E_SHAPE, "vt_row_moments: at most 64 chunks (2048 columns)");
  launch_k(ew::row_moments_kernel<false>, (unsigned)((M + 8 * ew::RM_RPW - 1) / (8 * ew::RM_RPW)), 256, 0, st, reinterpret_cast<const float2*>(stats), nchunk, M, eps,
                                                               reinterpret_cast<float2*>(moments));
  return check_launch("vt_row_moments");
}

// Patch im2col of B square images (S x S, C channels, patch P) into A[B*(S/P)^2, C*P*P] bf16 with
// row pitch ldo (>= C*P*P, a multiple of 8).  kind: 0 fp32 NCHW, 1 bf16 NCHW, 2 uint8 NHWC (0..255).
int vt_im2col(cudaStream_t st, const void* pix, int kind, int B, int C, int S, int P, uint16_t* out, long long ldo) {
  using namespace vt;
  if (B < 0 || C <= 0 || P <= 0 || S <= 0 || S % P) return set_error(E_SHAPE, "vt_im2col: bad geometry");
  if (kind < 0 || kind > 2) return set_error(E_VARIANT, "vt_im2col: unknown pixel kind %d", kind);
  if (B == 0) return OK;
  if (!pix || !out || ldo < (long long)C * P * P) return set_error(E_SHAPE, "vt_im2col: bad output");
  const int g = S / P;
  launch_k(ew::im2col_kernel, ew::grid_for((long long)B * g * g * C * P, 256), 256, 0, st, pix, kind, B, C, S, P, out, ldo);
  return check_launch("vt_im2col");
}

// Multi-crop combine of n_crops crop features f[n][T][W] (bf16; crop n at f + n*crop_stride, row pitch
// ldf) into out[T][2W]: global crop 0, then the mean of crops 1..n-1.
int vt_crop_combine(cudaStream_t st, const uint16_t* f, long long crop_stride, long long ldf, int n_crops, int T, int W,
                    uint16_t* out, long long ldo) {
  using namespace vt;
  if (n_crops < 2 || T < 0 || W <= 0 || W % 8) return set_error(E_SHAPE, "vt_crop_combine: bad shape");
  if (T == 0) return OK;
  if (!f || !out || ldf < W || ldo < 2LL * W || ldf % 8 || ldo % 8 || crop_stride % 8 || !aligned16(f) || !aligned16(out))
    return set_error(E_SHAPE, "vt_crop_combine: pitches / alignment invalid");
  launch_k(ew::combine_kernel, ew::grid_for((long long)T * (W / 8), 256), 256, 0, st, f, crop_stride, ldf, n_crops, T, W, out, ldo);
  return check_launch("vt_crop_combine");
}

// RG-LRU step over M tokens of width W on the bf16 input u; G = [gx_pre | ga_pre] fp32 [M][ldg >= 2W];
// state and x fp32, updated in place; first != 0 starts a new sequence (state ignored and overwritten).
int vt_row_rms(cudaStream_t st, const float* stats, int M, int nchunk, float eps, float* out) {
  using namespace vt;
  if (M < 0 || nchunk <= 0) return set_error(E_SHAPE, "vt_row_rms: bad shape");
  if (M == 0) return OK;
  if (!stats || !out) return set_error(E_SHAPE, "vt_row_rms: null pointer");
  if (nchunk > 64) return set_error(E_SHAPE, "vt_row_rms: at most 64 chunks (2048 columns)");
  launch_k(ew::row_moments_kernel<true>, (unsigned)((M + 8 * ew::RM_RPW - 1) / (8 * ew::RM_RPW)), 256, 0, st, reinterpret_cast<const float2*>(stats), nchunk, M,
           eps, reinterpret_cast<float2*>(out));
  return check_launch("vt_row_rms");
}

int vt_rglru_fold(cudaStream_t st, const float* G, long long ldg, const float* softplus_a, const float* rms_moments,
                  const float* rms_gamma, float* state, long long lds, float* x, long long ldx, uint16_t* xb,
                  long long ldxb, float* stats, int M, int W, float c, int first) {
  using namespace vt;
  if (M < 0 || W <= 0 || W % 32) return set_error(E_SHAPE, "vt_rglru_fold: W must be a positive multiple of 32");
  if (M == 0) return OK;
  if (!G || !softplus_a || !rms_moments || !rms_gamma || !state || !x || !xb || !stats)
    return set_error(E_SHAPE, "vt_rglru_fold: null pointer");
  if (ldg < 2LL * W || lds < W || ldx < W || ldxb < W || ldg % 4 || lds % 4 || ldx % 4 || ldxb % 4 || !aligned16(G) ||
      !aligned16(softplus_a) || !aligned16(rms_gamma) || !aligned16(state) || !aligned16(x) ||
      (reinterpret_cast<uintptr_t>(xb) & 7) || (reinterpret_cast<uintptr_t>(rms_moments) & 7) ||
      (reinterpret_cast<uintptr_t>(stats) & 7))
    return set_error(E_SHAPE, "vt_rglru_fold: pitches / alignment invalid");
  launch_k(ew::rglru_fold_kernel, ew::grid_for((long long)M * (W / 4), 256), 256, 0, st, G, ldg, softplus_a,
           reinterpret_cast<const float2*>(rms_moments), rms_gamma, state, lds, x, ldx, xb, ldxb,
           reinterpret_cast<float2*>(stats), M, W, c, first);
  return check_launch("vt_rglru_fold");
}

int vt_rglru(cudaStream_t st, const float* G, long long ldg, const float* softplus_a, const uint16_t* u, long long ldu,
             float* state, long long lds, float* x, long long ldx, int M, int W, float c, int first) {
  using namespace vt;
  if (M < 0 || W <= 0 || W % 4) return set_error(E_SHAPE, "vt_rglru: bad shape");
  if (M == 0) return OK;
  if (!G || !softplus_a || !u || !state || !x || ldg < 2LL * W || ldu < W || lds < W || ldx < W || ldg % 4 || ldu % 4 ||
      lds % 4 || ldx % 4 || !aligned16(G) || !aligned16(state) || !aligned16(x) || !aligned16(softplus_a) ||
      (reinterpret_cast<uintptr_t>(u) & 7))
    return set_error(E_SHAPE, "vt_rglru: pitches / alignment invalid");
  launch_k(ew::rglru_kernel, ew::grid_for((long long)M * (W / 4), 256), 256, 0, st, G, ldg, softplus_a, u, ldu, state, lds, x,
                                                                             ldx, M, W, c, first);
  return check_launch("vt_rglru");
}

}  // extern "C"
