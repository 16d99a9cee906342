// The full TAPNext++ block's recurrent and MLP element-wise kernels (tapnext/npu/step8.py:474-485):
//   ssm_step_tc_kernel     conv_1d (4 taps over frames) -> block-diagonal RG-LRU gates on tcgen05 -> recurrence ->
//                          z = h * gelu(y), with the bf16 rounding points of the reference's own restatement,
//                          pack8.py:252-279 (ssm_ref)
//   ssm_step_kernel        the same with the gates on the CUDA cores (rows or pointers that are not 16-byte aligned,
//                          and VT_SSM_TC=0)
//   gated_gelu_mul_kernel  the gated MLP's gelu_tanh(gate) * up (tapnext/npu/mm8.cc:937-960)
//   gelu_erf_kernel        the ViT MLP's exact GELU (pack8.py:246-250, gelu_erf_ref)
#include <cstdlib>
#include <mutex>

#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace ssm {

constexpr int RB = 32, HD = 64, THREADS = 256;

__device__ __forceinline__ float bfr(float v) { return bfround(v); }

// gelu_y: the y half of linear_yx arrives as the raw bf16 linear output and its GELU-tanh is taken here, with
// the GEMM epilogue's arithmetic (gelu_tanh2 on the bf16 value, rounded to bf16), so z is the same as when the
// GEMM applied the GELU.
__device__ __forceinline__ uint32_t gelu_word(uint32_t w) {
  float g0, g1;
  f2_unpack(gelu_tanh2(f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u))), g0, g1);
  return pack_bf2(g0, g1);
}

// One CTA: RB rows x one head (64 channels).  hist_old / hist_mid / hist_new hold x_(t-3) / x_(t-2) / x_(t-1)
// (zeros before the first frames); x_t is written over hist_old, so the caller rotates the three roles.
__global__ void __launch_bounds__(THREADS) ssm_step_kernel(
    const uint16_t* __restrict__ yg, const uint16_t* __restrict__ xx, long long ldi, uint16_t* hist_old,
    const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* __restrict__ h, long long ldhs,
    const float* __restrict__ conv_w, const float* __restrict__ conv_b, const float* __restrict__ sp,
    const float* __restrict__ wx, const float* __restrict__ bx, const float* __restrict__ wa,
    const float* __restrict__ ba, uint16_t* __restrict__ z, long long ldz, int R, int W, int first, int gelu_y) {
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
    uint32_t yb = yg[(size_t)row * ldi + col];
    if (gelu_y) yb = gelu_word(yb) & 0xffffu;
    z[(size_t)row * ldz + col] = f2bf(__fmul_rn(hb, bf2f((uint16_t)yb)));
  }
}

// The same step with the two block-diagonal gates on the tensor cores.  One CTA = 128 rows x one head (64
// channels), 1024 threads:
//   1. conv_1d: thread (row group, 8-channel chunk kc) builds xc for its 8 channels (the reference's bf16
//      rounding points, as above) and stores them as one 16-byte row of a core matrix of the A tile: the
//      canonical no-swizzle K-major layout [kc][row][8] (LBO 2048 B between k chunks, SBO 128 B between
//      8-row groups), so the tile is the MMA's A operand as built; x_t goes over the oldest history tap.
//   2. the head's Wx, Wa ([64 in][64 out], fp32 in global memory) become bf16 B tiles [kc][out][8] (LBO 1024 B,
//      SBO 128 B): D = A B^T sums over `in`, as the reference's x @ w.
//   3. thread 0 issues 2 x 4 tcgen05.mma (M 128, N 64, K 16) into TMEM columns [0, 64) (Wx) and [64, 128) (Wa).
//   4. warp w reads TMEM lane quarter w % 4 (its rows) and 8-channel chunk w / 4 of both accumulators; thread =
//      (row, chunk) finishes the element-wise part exactly as ssm_step_kernel does (32 warps, so the long
//      exponential / reciprocal / square-root chains of different elements overlap).
// The products of bf16 values are exact in fp32; the tensor core adds them in its own order, so a gate
// pre-activation can differ from the float64 sum of the reference by a few fp32 ulps, which changes its bf16
// rounding only within a few ulps of a bf16 boundary.  The transcendentals come from g_ssm_tab, which holds
// the reference's float64 values rounded to bf16, so they add no difference of their own.
constexpr int TC_ROWS = 128, TC_THREADS = 1024;

// The recurrence's transcendentals as functions of one bf16 value, indexed by its 16 bits, each evaluated in
// float64 and rounded to bf16 as the reference's ssm_ref does (pack8.py:264-275):
//   table 0: bf16(1 / (1 + exp(-x)))   the two gates
//   table 1: bf16(exp(x))              a = exp(log_a) and e2 = exp(2 log_a) (2 log_a of a bf16 log_a is exact)
//   table 2: bf16(sqrt(x)), the square root taken in fp32 as numpy does on float32 arrays
// 3 x 128 KB of device memory for every GPU that loads the library, filled once per device.
static __device__ uint16_t g_ssm_tab[3][65536];

__global__ void ssm_tables_kernel() {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 65536; i += gridDim.x * blockDim.x) {
    const double x = (double)__uint_as_float((uint32_t)i << 16);
    g_ssm_tab[0][i] = f2bf((float)(1.0 / (1.0 + exp(-x))));
    g_ssm_tab[1][i] = f2bf((float)exp(x));
    g_ssm_tab[2][i] = f2bf(sqrtf((float)x));
  }
}

// 8 consecutive floats (16-byte aligned) as two 128-bit loads.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

__global__ void __launch_bounds__(TC_THREADS, 1) ssm_step_tc_kernel(
    const uint16_t* __restrict__ yg, const uint16_t* __restrict__ xx, long long ldi, uint16_t* hist_old,
    const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* __restrict__ h, long long ldhs,
    const float* __restrict__ conv_w, const float* __restrict__ conv_b, const float* __restrict__ sp,
    const float* __restrict__ wx, const float* __restrict__ bx, const float* __restrict__ wa,
    const float* __restrict__ ba, uint16_t* __restrict__ z, long long ldz, int R, int W, int first, int gelu_y) {
  __shared__ __align__(1024) uint8_t a_tile[TC_ROWS * HD * 2];  // 16 KB: xc, bf16
  __shared__ __align__(1024) uint8_t b_tile[2][HD * HD * 2];    // 2 x 8 KB: Wx^T, Wa^T, bf16
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = blockIdx.y, r0 = blockIdx.x * TC_ROWS, c0 = q * HD;
  if (tid == 0) {
    mbar_init(&mma_done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 128);
    tmem_relinquish();
  }
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  // ---- 2. gate weights: thread (gate, k chunk, out n) packs w[8 kc .. 8 kc + 7][n] into the 16-byte core-matrix
  //         row (n, kc) of its gate's B tile; for each k the 64 threads of a chunk read 64 consecutive floats
  {
    const int n = tid & 63, kc = (tid >> 6) & 7, gate = tid >> 9;
    const float* w = (gate ? wa : wx) + (size_t)q * HD * HD + (size_t)(kc * 8) * HD + n;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = w[(size_t)i * HD];
    *reinterpret_cast<uint4*>(&b_tile[gate][kc * 1024 + n * 16]) =
        make_uint4(pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]), pack_bf2(v[4], v[5]), pack_bf2(v[6], v[7]));
  }
  // ---- 1. conv_1d into the A tile: thread owns 8-channel chunk kc = tid % 8 of rows tid / 8 + 64 i
  {
    const int kc = tid & 7, col = c0 + kc * 8;
    float cw[4][8], cb[8];
#pragma unroll
    for (int k = 0; k < 4; k++) load8(conv_w + (size_t)k * W + col, cw[k]);
    load8(conv_b + col, cb);
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int k = 0; k < 4; k++) cw[k][j] = bfr(cw[k][j]);
      cb[j] = bfr(cb[j]);
    }
#pragma unroll
    for (int i = 0; i < TC_ROWS / (TC_THREADS / 8); i++) {
      const int r = (tid >> 3) + (TC_THREADS / 8) * i, row = r0 + r;
      uint4 packed = make_uint4(0, 0, 0, 0);
      if (row < R) {
        const size_t ih = (size_t)row * ldh + col;
        const uint4 x0 = *reinterpret_cast<const uint4*>(xx + (size_t)row * ldi + col);
        const uint4 t0 = *reinterpret_cast<const uint4*>(hist_old + ih);
        const uint4 t1 = *reinterpret_cast<const uint4*>(hist_mid + ih);
        const uint4 t2 = *reinterpret_cast<const uint4*>(hist_new + ih);
        const uint32_t w0[4] = {t0.x, t0.y, t0.z, t0.w}, w1[4] = {t1.x, t1.y, t1.z, t1.w},
                       w2[4] = {t2.x, t2.y, t2.z, t2.w}, w3[4] = {x0.x, x0.y, x0.z, x0.w};
        uint32_t out[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
          float xc2[2];
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            const int j = 2 * p + hh;
            const float taps[4] = {hh ? __uint_as_float(w0[p] & 0xffff0000u) : __uint_as_float(w0[p] << 16),
                                   hh ? __uint_as_float(w1[p] & 0xffff0000u) : __uint_as_float(w1[p] << 16),
                                   hh ? __uint_as_float(w2[p] & 0xffff0000u) : __uint_as_float(w2[p] << 16),
                                   hh ? __uint_as_float(w3[p] & 0xffff0000u) : __uint_as_float(w3[p] << 16)};
            float sacc = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) sacc = __fadd_rn(sacc, bfr(__fmul_rn(taps[k], cw[k][j])));
            xc2[hh] = bfr(__fadd_rn(bfr(sacc), cb[j]));
          }
          out[p] = pack_bf2(xc2[0], xc2[1]);
        }
        packed = make_uint4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<uint4*>(hist_old + ih) = x0;
      }
      *reinterpret_cast<uint4*>(&a_tile[kc * 2048 + r * 16]) = packed;  // rows past R stay zero
    }
  }
  fence_proxy_async_smem();  // the generic-proxy tile writes become visible to the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // ---- 3. MMAs
  if (tid == 0) {
    constexpr uint32_t IDESC = idesc_bf16(TC_ROWS, HD);
    const uint32_t sa = smem_u32(a_tile), sb0 = smem_u32(b_tile[0]), sb1 = smem_u32(b_tile[1]);
#pragma unroll
    for (int k = 0; k < HD / 16; k++) {
      umma_f16(tmem, sdesc_noswz(sa + k * 4096, 2048, 128), sdesc_noswz(sb0 + k * 2048, 1024, 128), IDESC, k > 0 ? 1u : 0u);
      umma_f16(tmem + HD, sdesc_noswz(sa + k * 4096, 2048, 128), sdesc_noswz(sb1 + k * 2048, 1024, 128), IDESC,
               k > 0 ? 1u : 0u);
    }
    umma_commit(&mma_done);
  }
  // ---- 4. element-wise part: thread = (row, 8-channel chunk)
  const int quarter = warp & 3, cc = warp >> 2;
  const int r = quarter * 32 + lane, row = r0 + r;
  // the tcgen05.ld below are warp-collective: a warp goes on only if all its lanes saw the MMAs complete
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&mma_done, 0, &abort_flag, ST_SSM_MMA));
  tc_fence_after();
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  if (ok) {
    uint32_t dx[8], da[8];
    tmem_ld8(tmem + lane_off + cc * 8, dx);
    tmem_ld8(tmem + lane_off + HD + cc * 8, da);
    tmem_ld_wait();
    if (row < R) {
      const int col = c0 + cc * 8;
      const size_t is = (size_t)row * ldhs + col, iz = (size_t)row * ldz + col, iy = (size_t)row * ldi + col;
      float hv[8];
      if (!first) {
        const float4 t0 = *reinterpret_cast<const float4*>(h + is), t1 = *reinterpret_cast<const float4*>(h + is + 4);
        hv[0] = t0.x, hv[1] = t0.y, hv[2] = t0.z, hv[3] = t0.w, hv[4] = t1.x, hv[5] = t1.y, hv[6] = t1.z, hv[7] = t1.w;
      }
      const uint4 y0 = *reinterpret_cast<const uint4*>(yg + iy);
      uint32_t yw[4] = {y0.x, y0.y, y0.z, y0.w};
      if (gelu_y) {
#pragma unroll
        for (int k = 0; k < 4; k++) yw[k] = gelu_word(yw[k]);
      }
      const uint4 xa = *reinterpret_cast<const uint4*>(&a_tile[cc * 2048 + r * 16]);
      const uint32_t xw[4] = {xa.x, xa.y, xa.z, xa.w};
      float hn[8], bxv[8], bav[8], spv[8];
      load8(bx + col, bxv);
      load8(ba + col, bav);
      load8(sp + col, spv);
      uint32_t zw[4];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float gx_pre = bfr(__fadd_rn(bfr(__uint_as_float(dx[j])), bfr(bxv[j])));
        const float ga_pre = bfr(__fadd_rn(bfr(__uint_as_float(da[j])), bfr(bav[j])));
        const float gx = bf2f(g_ssm_tab[0][__float_as_uint(gx_pre) >> 16]);
        const float ga = bf2f(g_ssm_tab[0][__float_as_uint(ga_pre) >> 16]);
        const float log_a = bfr(__fmul_rn(bfr(-8.f * ga), bfr(spv[j])));
        const float a = bf2f(g_ssm_tab[1][__float_as_uint(log_a) >> 16]);
        const float xc = (j & 1) ? __uint_as_float(xw[j >> 1] & 0xffff0000u) : __uint_as_float(xw[j >> 1] << 16);
        const float gated = bfr(__fmul_rn(xc, gx));
        float hb;
        if (first) {
          hn[j] = gated;
          hb = gated;
        } else {
          const float e2 = bf2f(g_ssm_tab[1][__float_as_uint(2.f * log_a) >> 16]);
          const float mult = bf2f(g_ssm_tab[2][__float_as_uint(bfr(__fsub_rn(1.f, e2))) >> 16]);
          const float nx = bfr(__fmul_rn(gated, mult));
          hn[j] = __fadd_rn(__fmul_rn(a, hv[j]), nx);
          hb = bfr(hn[j]);
        }
        const float yv = (j & 1) ? __uint_as_float(yw[j >> 1] & 0xffff0000u) : __uint_as_float(yw[j >> 1] << 16);
        const uint16_t zb = f2bf(__fmul_rn(hb, yv));
        zw[j >> 1] = (j & 1) ? (zw[j >> 1] | ((uint32_t)zb << 16)) : (uint32_t)zb;
      }
      *reinterpret_cast<float4*>(h + is) = make_float4(hn[0], hn[1], hn[2], hn[3]);
      *reinterpret_cast<float4*>(h + is + 4) = make_float4(hn[4], hn[5], hn[6], hn[7]);
      *reinterpret_cast<uint4*>(z + iz) = make_uint4(zw[0], zw[1], zw[2], zw[3]);
    }
  } else if (tid == 0) {
    mbar_wait_drain(&mma_done, 0, 200000000LL);  // let the MMAs this CTA issued finish before TMEM is freed
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
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

// VT_SSM_TC=0 keeps the CUDA-core kernel (A/B switch); the tensor-core kernel is the default.
static bool ssm_use_tc_impl() {
  const char* e = getenv("VT_SSM_TC");
  return e ? atoi(e) != 0 : true;
}

static int grid_for(long long n, int threads) {
  const long long b = (n + threads - 1) / threads, cap = 8LL * sm_count();
  return (int)(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace ssm
}  // namespace vt

static bool ssm_use_tc() {
  static const bool v = vt::ssm::ssm_use_tc_impl();
  return v;
}

// Fills g_ssm_tab on the current device, once, on the caller's stream (kernels launched after it on that
// stream see the tables).  The first call on a device must not be part of a stream capture.
static int ssm_tables_ready(cudaStream_t st) {
  using namespace vt;
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return set_error(E_LAUNCH, "vt_ssm_step: no current device");
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return set_error(E_LAUNCH, "vt_ssm_step: cudaStreamIsCapturing: %s", cudaGetErrorString(e));
  if (cap != cudaStreamCaptureStatusNone)
    return set_error(E_LAUNCH, "vt_ssm_step: the first call on a device builds its tables and cannot be captured; "
                               "make one call before capturing");
  launch_k(ssm::ssm_tables_kernel, 64, 256, 0, st);
  int rc = check_launch("vt_ssm_step (tables)");
  if (rc) return rc;
  done[dev] = true;
  return OK;
}

extern "C" {

int vt_ssm_step(cudaStream_t st, const uint16_t* yg, const uint16_t* xx, long long ldi, uint16_t* hist_old,
                const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* h, long long ldhs,
                const float* conv_w, const float* conv_b, const float* softplus_a, const float* wx, const float* bx,
                const float* wa, const float* ba, uint16_t* z, long long ldz, int R, int W, int first, int gelu_y) {
  using namespace vt;
  if (R < 0 || W <= 0 || W % ssm::HD) return set_error(E_SHAPE, "vt_ssm_step: W must be a positive multiple of 64");
  if (R == 0) return OK;
  if (!yg || !xx || !hist_old || !hist_mid || !hist_new || !h || !conv_w || !conv_b || !softplus_a || !wx || !bx || !wa ||
      !ba || !z || ldi < W || ldh < W || ldhs < W || ldz < W)
    return set_error(E_SHAPE, "vt_ssm_step: null pointer or row pitch below W");
  // the tensor-core kernel reads and writes 16-byte vectors: rows and bases 16-byte aligned
  const bool vec = ldi % 8 == 0 && ldh % 8 == 0 && ldhs % 4 == 0 && ldz % 8 == 0 && W % 4 == 0 && aligned16(yg) &&
                   aligned16(xx) && aligned16(hist_old) && aligned16(hist_mid) && aligned16(hist_new) && aligned16(h) &&
                   aligned16(z) && aligned16(conv_w) && aligned16(conv_b) && aligned16(softplus_a) && aligned16(bx) &&
                   aligned16(ba);
  if (vec && ssm_use_tc()) {
    const int trc = ssm_tables_ready(st);
    if (trc) return trc;
    const dim3 grid((R + ssm::TC_ROWS - 1) / ssm::TC_ROWS, W / ssm::HD);
    launch_k(ssm::ssm_step_tc_kernel, grid, ssm::TC_THREADS, 0, st, yg, xx, ldi, hist_old, hist_mid, hist_new, ldh, h, ldhs, conv_w,
             conv_b, softplus_a, wx, bx, wa, ba, z, ldz, R, W, first, gelu_y);
    return check_launch("vt_ssm_step");
  }
  const dim3 grid((R + ssm::RB - 1) / ssm::RB, W / ssm::HD);
  launch_k(ssm::ssm_step_kernel, grid, ssm::THREADS, 0, st, yg, xx, ldi, hist_old, hist_mid, hist_new, ldh, h, ldhs, conv_w,
                                                      conv_b, softplus_a, wx, bx, wa, ba, z, ldz, R, W, first, gelu_y);
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
