// The full TAPNext++ block's recurrent and MLP element-wise kernels (tapnext/npu/step8.py:474-485):
//   ssm_step_kernel        conv_1d (4 taps over frames) -> block-diagonal RG-LRU gates -> recurrence -> z = h * gelu(y),
//                          with the bf16 rounding points of the reference's own restatement, pack8.py:252-279 (ssm_ref)
//   gated_gelu_mul_kernel  the gated MLP's gelu_tanh(gate) * up (tapnext/npu/mm8.cc:937-960)
//   gelu_erf_kernel        the ViT MLP's exact GELU (pack8.py:246-250, gelu_erf_ref)
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace ssm {

constexpr int RB = 32, HD = 64, THREADS = 256;

__device__ __forceinline__ float bfr(float v) { return bfround(v); }

// One CTA: RB rows x one head (64 channels).  hist_old / hist_mid / hist_new hold x_(t-3) / x_(t-2) / x_(t-1)
// (zeros before the first frames); x_t is written over hist_old, so the caller rotates the three roles.
__global__ void __launch_bounds__(THREADS) ssm_step_kernel(
    const uint16_t* __restrict__ yg, const uint16_t* __restrict__ xx, long long ldi, uint16_t* hist_old,
    const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* __restrict__ h, long long ldhs,
    const float* __restrict__ conv_w, const float* __restrict__ conv_b, const float* __restrict__ sp,
    const float* __restrict__ wx, const float* __restrict__ bx, const float* __restrict__ wa,
    const float* __restrict__ ba, uint16_t* __restrict__ z, long long ldz, int R, int W, int first) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  __shared__ float xcs[RB][HD + 1];
  __shared__ float wxs[HD][HD], was[HD][HD];
  const int q = blockIdx.y, r0 = blockIdx.x * RB, tid = threadIdx.x;
  const int c0 = q * HD;
  for (int i = tid; i < HD * HD; i += THREADS) {  // [64 in][64 out] of this head, bf16 values
    wxs[i / HD][i % HD] = bfr(wx[(size_t)q * HD * HD + i]);
    was[i / HD][i % HD] = bfr(wa[(size_t)q * HD * HD + i]);
  }
  // xc = bf(bf(sum_i bf(x_(t-3+i) * bf(w_i))) + bf(b)), taps oldest .. current, summed in that order
  for (int e = tid; e < RB * HD; e += THREADS) {
    const int r = e / HD, c = e % HD, row = r0 + r, col = c0 + c;
    float xc = 0.f;
    if (row < R) {
      const size_t ih = (size_t)row * ldh + col, ii = (size_t)row * ldi + col;
      const uint16_t x0 = xx[ii];
      const float taps[4] = {bf2f(hist_old[ih]), bf2f(hist_mid[ih]), bf2f(hist_new[ih]), bf2f(x0)};
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 4; k++) s = __fadd_rn(s, bfr(__fmul_rn(taps[k], bfr(conv_w[(size_t)k * W + col]))));
      xc = bfr(__fadd_rn(bfr(s), bfr(conv_b[col])));
      hist_old[ih] = x0;
    }
    xcs[r][c] = xc;
  }
  __syncthreads();
  // gates, RG-LRU, z.  The reference sums the 64 bf16 x bf16 products in float64 and evaluates sigmoid / exp
  // in float64 before rounding to bf16; here the products are exact in fp32, the sums and transcendentals
  // are fp32, and the bf16 results differ from the float64 path only when a value falls within a few fp32
  // ulps of a bf16 rounding boundary (about 1e-4 of the elements, by one bf16 step).
  const int o = tid % HD, col = c0 + o;
  const float bxo = bfr(bx[col]), bao = bfr(ba[col]), spo = bfr(sp[col]);
  for (int r = tid / HD; r < RB; r += THREADS / HD) {
    const int row = r0 + r;
    if (row >= R) break;
    float dx = 0.f, da = 0.f;
#pragma unroll 16
    for (int i = 0; i < HD; i++) {
      const float v = xcs[r][i];
      dx = fmaf(v, wxs[i][o], dx);
      da = fmaf(v, was[i][o], da);
    }
    const float gx_pre = bfr(__fadd_rn(bfr(dx), bxo)), ga_pre = bfr(__fadd_rn(bfr(da), bao));
    const float gx = bfr(1.f / (1.f + expf(-gx_pre)));
    const float ga = bfr(1.f / (1.f + expf(-ga_pre)));
    const float log_a = bfr(__fmul_rn(bfr(-8.f * ga), spo));
    const float a = bfr(expf(log_a));
    const float xc = xcs[r][o];
    const float gated = bfr(__fmul_rn(xc, gx));
    const size_t is = (size_t)row * ldhs + col;
    float hn, hb;
    if (first) {
      hn = gated;
      hb = gated;
    } else {
      const float e2 = bfr(expf(bfr(2.f * log_a)));
      const float mult = bfr(sqrtf(bfr(__fsub_rn(1.f, e2))));
      const float nx = bfr(__fmul_rn(gated, mult));
      hn = __fadd_rn(__fmul_rn(a, h[is]), nx);
      hb = bfr(hn);
    }
    h[is] = hn;
    z[(size_t)row * ldz + col] = f2bf(__fmul_rn(hb, bf2f(yg[(size_t)row * ldi + col])));
  }
}

// out[r, j] = bf16(bf16(gelu_tanh(G[r, j])) * G[r, F + j]) for j < F: G = [gate | up] (bf16 linear outputs)
__global__ void gated_gelu_mul_kernel(const uint16_t* __restrict__ G, long long ldg, uint16_t* __restrict__ out,
                                      long long ldo, int R, int F) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int nv = F / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)R * nv;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / nv;
    const int j = (int)(i % nv) * 8;
    const uint4 g = *reinterpret_cast<const uint4*>(G + r * ldg + j);
    const uint4 u = *reinterpret_cast<const uint4*>(G + r * ldg + F + j);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float g0 = __uint_as_float(gw[k] << 16), g1 = __uint_as_float(gw[k] & 0xffff0000u);
      const float u0 = __uint_as_float(uw[k] << 16), u1 = __uint_as_float(uw[k] & 0xffff0000u);
      ow[k] = pack_bf2(__fmul_rn(bfround(gelu_tanh(g0)), u0), __fmul_rn(bfround(gelu_tanh(g1)), u1));
    }
    *reinterpret_cast<uint4*>(out + r * ldo + j) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// x = bf16(0.5 x (1 + erf(x / sqrt 2))) in place on a bf16 [R][N] matrix (N % 8 == 0)
__global__ void gelu_erf_kernel(uint16_t* __restrict__ x, long long ld, int R, int N) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int nv = N / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)R * nv;
       i += (long long)gridDim.x * blockDim.x) {
    uint4* p = reinterpret_cast<uint4*>(x + (i / nv) * ld + (int)(i % nv) * 8);
    const uint4 v = *p;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float a = __uint_as_float(w[k] << 16), b = __uint_as_float(w[k] & 0xffff0000u);
      o[k] = pack_bf2(0.5f * a * (1.f + erff(a * 0.70710678118654752f)), 0.5f * b * (1.f + erff(b * 0.70710678118654752f)));
    }
    *p = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

static int grid_for(long long n, int threads) {
  const long long b = (n + threads - 1) / threads, cap = 8LL * sm_count();
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace ssm
}  // namespace vt

extern "C" {

int vt_ssm_step(cudaStream_t st, const uint16_t* yg, const uint16_t* xx, long long ldi, uint16_t* hist_old,
                const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* h, long long ldhs,
                const float* conv_w, const float* conv_b, const float* softplus_a, const float* wx, const float* bx,
                const float* wa, const float* ba, uint16_t* z, long long ldz, int R, int W, int first) {
  using namespace vt;
  if (R < 0 || W <= 0 || W % ssm::HD) return set_error(E_SHAPE, "vt_ssm_step: W must be a positive multiple of 64");
  if (R == 0) return OK;
  if (!yg || !xx || !hist_old || !hist_mid || !hist_new || !h || !conv_w || !conv_b || !softplus_a || !wx || !bx || !wa ||
      !ba || !z || ldi < W || ldh < W || ldhs < W || ldz < W)
    return set_error(E_SHAPE, "vt_ssm_step: null pointer or row pitch below W");
  const dim3 grid((R + ssm::RB - 1) / ssm::RB, W / ssm::HD);
  launch_k(ssm::ssm_step_kernel, grid, ssm::THREADS, 0, st, yg, xx, ldi, hist_old, hist_mid, hist_new, ldh, h, ldhs, conv_w,
                                                      conv_b, softplus_a, wx, bx, wa, ba, z, ldz, R, W, first);
  return check_launch("vt_ssm_step");
}

int vt_gated_gelu_mul(cudaStream_t st, const uint16_t* G, long long ldg, uint16_t* out, long long ldo, int R, int F) {
  using namespace vt;
  if (R < 0 || F <= 0 || F % 8) return set_error(E_SHAPE, "vt_gated_gelu_mul: F must be a positive multiple of 8");
  if (R == 0) return OK;
  if (!G || !out || ldg < 2LL * F || ldo < F || ldg % 8 || ldo % 8 || !aligned16(G) || !aligned16(out))
    return set_error(E_SHAPE, "vt_gated_gelu_mul: pitches / alignment invalid");
  launch_k(ssm::gated_gelu_mul_kernel, ssm::grid_for((long long)R * (F / 8), 256), 256, 0, st, G, ldg, out, ldo, R, F);
  return check_launch("vt_gated_gelu_mul");
}

int vt_gelu_erf(cudaStream_t st, uint16_t* x, long long ld, int R, int N) {
  using namespace vt;
  if (R < 0 || N <= 0 || N % 8) return set_error(E_SHAPE, "vt_gelu_erf: N must be a positive multiple of 8");
  if (R == 0) return OK;
  if (!x || ld < N || ld % 8 || !aligned16(x)) return set_error(E_SHAPE, "vt_gelu_erf: pitch / alignment invalid");
  launch_k(ssm::gelu_erf_kernel, ssm::grid_for((long long)R * (N / 8), 256), 256, 0, st, x, ld, R, N);
  return check_launch("vt_gelu_erf");
}

}  // extern "C"
