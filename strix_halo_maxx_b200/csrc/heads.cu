// TAPNext++ tracking heads on the device: the reference runs them on the host after every frame
// (Step8.heads_np, tapnext/npu/step8.py:327-362, numpy fp32; Step8.heads, step8.py:364-372, torch).
//
// Each head is Linear -> LayerNorm -> erf GELU -> Linear -> LayerNorm -> erf GELU -> Linear on the
// query tokens; the coordinate head's 2 x bins logits go through a soft-argmax per axis (softmax at a
// temperature, restricted to +-window bins around the first maximum, renormalised, expectation + 0.5).
// The heads are tiny (about 0.3 GFLOP for 256 queries) and their output is compared in pixels, so they
// are computed in fp32 on the CUDA cores, with the reference's order of operations, not on the bf16
// tensor-core path:
//   head_linear_pipe_kernel  Y = X Wt + b (X bf16 or fp32, Wt fp32 [K][N]); 32 x 32 output tiles fed by a
//                          cp.async ring, each output summed over k in order with fp32 FMAs
//   head_linear_kernel     the same product for operands the ring cannot copy (unaligned rows, N % 4 != 0)
//   head_ln_gelu_kernel    in place per row: (h - mean) / sqrt(var + eps) * g + b, then 0.5 y (1 + erf(y / sqrt 2));
//                          a warp per row, the row in registers
//   soft_argmax_kernel     a warp per (query, axis)
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace heads {

constexpr int BM = 32, BN = 64, BK = 32;

template <bool IN_BF16>
__global__ void __launch_bounds__(256) head_linear_kernel(const void* __restrict__ X, long long ldx,
                                                          const float* __restrict__ Wt, long long ldw,
                                                          const float* __restrict__ bias, float* __restrict__ Y,
                                                          long long ldy, int M, int N, int K) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  __shared__ float As[BM][BK + 1];
  __shared__ float Bs[BK][BN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;  // 4 columns x 2 rows per thread
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[2][4] = {};
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int i = 0; i < (BM * BK) / 256; i++) {  // A tile, row-major, coalesced along k
      const int e = tid + i * 256, r = e / BK, c = e % BK;
      const int m = m0 + r, k = k0 + c;
      float v = 0.f;
      if (m < M && k < K) {
        if (IN_BF16) v = bf2f(static_cast<const uint16_t*>(X)[(size_t)m * ldx + k]);
        else v = static_cast<const float*>(X)[(size_t)m * ldx + k];
      }
      As[r][c] = v;
    }
#pragma unroll
    for (int i = 0; i < (BK * BN) / 256; i++) {  // B tile, coalesced along n
      const int e = tid + i * 256, r = e / BN, c = e % BN;
      const int k = k0 + r, n = n0 + c;
      Bs[r][c] = (k < K && n < N) ? Wt[(size_t)k * ldw + n] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < BK; k++) {
      const float a0 = As[ty * 2][k], a1 = As[ty * 2 + 1][k];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float b = Bs[k][tx * 4 + c];
        acc[0][c] = fmaf(a0, b, acc[0][c]);
        acc[1][c] = fmaf(a1, b, acc[1][c]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const int m = m0 + ty * 2 + r;
    if (m >= M) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int n = n0 + tx * 4 + c;
      if (n < N) Y[(size_t)m * ldy + n] = acc[r][c] + (bias ? bias[n] : 0.f);
    }
  }
}

// The same product with its operand tiles streamed through a PST-stage cp.async ring, so a CTA has PST - 1
// k-tiles in flight instead of one load -> barrier -> compute round trip per k-tile (the heads' linears are
// a few dozen CTAs with nothing else to hide that latency: 53.6 -> ~10 us for 256 x 768 -> 512).  32 x 32
// output tiles (more CTAs), each output still one fp32 FMA chain over k in order, so the results equal
// head_linear_kernel's bit for bit.  Needs 16-byte aligned X / Wt with 16-byte multiple row pitches, N % 4 == 0
// and K a multiple of 16 bytes of X (the launcher checks; other shapes take head_linear_kernel).
constexpr int PBM = 32, PBN = 32, PBK = 32, PST = 5, PTHREADS = 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {  // zero-fills past src_bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool IN_BF16>
__global__ void __launch_bounds__(PTHREADS) head_linear_pipe_kernel(const void* __restrict__ X, long long ldx,
                                                                    const float* __restrict__ Wt, long long ldw,
                                                                    const float* __restrict__ bias,
                                                                    float* __restrict__ Y, long long ldy, int M, int N,
                                                                    int K) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  constexpr int AE = IN_BF16 ? 2 : 4;       // bytes per X element
  constexpr int A_ROW = PBK * AE;           // bytes of one row's k-slice
  constexpr int A_PITCH = A_ROW + 16;       // padded: the four rows a warp reads fall in different banks
  __shared__ __align__(16) uint8_t sa[PST][PBM * A_PITCH];
  __shared__ __align__(16) float sb[PST][PBK][PBN];
  const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;  // 4 columns x 2 rows per thread
  const int m0 = blockIdx.y * PBM, n0 = blockIdx.x * PBN;
  const int nk = (K + PBK - 1) / PBK;
  const char* xb = static_cast<const char*>(X);
  auto load = [&](int kt, int st) {
    const int k0 = kt * PBK;
    for (int c = tid; c < PBM * (A_ROW / 16); c += PTHREADS) {  // X tile: rows m0.., 16-byte chunks along k
      const int r = c / (A_ROW / 16), q = c % (A_ROW / 16);
      const int m = m0 + r, k = k0 + q * (16 / AE);
      const bool in = m < M && k < K;
      cp_async16(&sa[st][r * A_PITCH + q * 16], in ? xb + ((size_t)m * ldx + k) * AE : xb, in ? 16u : 0u);
    }
    for (int c = tid; c < PBK * (PBN / 4); c += PTHREADS) {  // Wt tile: k rows, 16-byte chunks along n
      const int r = c / (PBN / 4), q = c % (PBN / 4);
      const int k = k0 + r, n = n0 + q * 4;
      const bool in = k < K && n < N;
      cp_async16(&sb[st][r][q * 4], in ? Wt + (size_t)k * ldw + n : Wt, in ? 16u : 0u);
    }
  };
#pragma unroll
  for (int s = 0; s < PST - 1; s++) {
    if (s < nk) load(s, s);
    cp_async_commit();
  }
  float acc[2][4] = {};
  for (int kt = 0; kt < nk; kt++) {
    cp_async_wait<PST - 2>();  // k-tile kt has landed (this thread's copies; the barrier makes it everyone's)
    __syncthreads();           // ... and every thread is done with the slot the next load overwrites
    if (kt + PST - 1 < nk) load(kt + PST - 1, (kt + PST - 1) % PST);
    cp_async_commit();
    const int st = kt % PST;
    const uint8_t* a0p = &sa[st][(ty * 2) * A_PITCH];
    const uint8_t* a1p = a0p + A_PITCH;
#pragma unroll 8
    for (int k = 0; k < PBK; k++) {
      float a0, a1;
      if (IN_BF16) {
        a0 = bf2f(reinterpret_cast<const uint16_t*>(a0p)[k]);
        a1 = bf2f(reinterpret_cast<const uint16_t*>(a1p)[k]);
      } else {
        a0 = reinterpret_cast<const float*>(a0p)[k];
        a1 = reinterpret_cast<const float*>(a1p)[k];
      }
      const float4 b = *reinterpret_cast<const float4*>(&sb[st][k][tx * 4]);
      acc[0][0] = fmaf(a0, b.x, acc[0][0]);
      acc[0][1] = fmaf(a0, b.y, acc[0][1]);
      acc[0][2] = fmaf(a0, b.z, acc[0][2]);
      acc[0][3] = fmaf(a0, b.w, acc[0][3]);
      acc[1][0] = fmaf(a1, b.x, acc[1][0]);
      acc[1][1] = fmaf(a1, b.y, acc[1][1]);
      acc[1][2] = fmaf(a1, b.z, acc[1][2]);
      acc[1][3] = fmaf(a1, b.w, acc[1][3]);
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const int m = m0 + ty * 2 + r;
    if (m >= M) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int n = n0 + tx * 4 + c;
      if (n < N) Y[(size_t)m * ldy + n] = acc[r][c] + (bias ? bias[n] : 0.f);
    }
  }
}

// N = 32 * V columns per row; row r uses gamma / beta group r % groups.
template <int V>
__global__ void __launch_bounds__(256) head_ln_gelu_kernel(float* __restrict__ Y, long long ldy, int rows,
                                                           const float* __restrict__ gamma,
                                                           const float* __restrict__ beta, int groups, float eps) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  constexpr int N = 32 * V;
  float* y = Y + (size_t)row * ldy;
  const float* g = gamma + (size_t)(row % groups) * N;
  const float* b = beta + (size_t)(row % groups) * N;
  float h[V];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    h[i] = y[lane + 32 * i];
    s += h[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mu = s / (float)N;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    const float d = h[i] - mu;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float sd = sqrtf(q / (float)N + eps);
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int c = lane + 32 * i;
    const float t = (h[i] - mu) / sd * g[c] + b[c];
    y[c] = 0.5f * t * (1.0f + erff(t * 0.7071067811865476f));
  }
}

// One warp per (query q, axis a): bins logits at L[q][a * bins ..]; lane l holds bins l, l + 32, ...
template <int V>
__global__ void __launch_bounds__(256) soft_argmax_kernel(const float* __restrict__ L, long long ldl, int Q,
                                                          int window, float temperature, float* __restrict__ tracks,
                                                          long long ldt) {
  griddep_wait();
  griddep_launch();
  constexpr int bins = 32 * V;
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (item >= 2 * Q) return;
  const int q = item >> 1, ax = item & 1;
  const float* h = L + (size_t)q * ldl + (size_t)ax * bins;
  float v[V];
  float best = -INFINITY;
  int arg = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < V; i++) {
    v[i] = h[lane + 32 * i];
    if (v[i] > best) {  // bins of a lane ascend, so the first maximum of the lane wins ties
      best = v[i];
      arg = lane + 32 * i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {  // the first maximum overall: largest value, then smallest index
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
    if (ob > best || (ob == best && oa < arg)) {
      best = ob;
      arg = oa;
    }
  }
  const float zmax = best * temperature;
  float e[V], s = 0.f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    e[i] = expf(v[i] * temperature - zmax);
    s += e[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    const int d = lane + 32 * i - arg;
    e[i] = (d <= window && d >= -window) ? e[i] / s : 0.f;
    s2 += e[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < V; i++) t = fmaf(e[i] / s2, (float)(lane + 32 * i), t);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (lane == 0) tracks[(size_t)q * ldt + ax] = t + 0.5f;
}

}  // namespace heads
}  // namespace vt

extern "C" {

int vt_head_linear(cudaStream_t st, const void* X, long long ldx, int x_bf16, const float* Wt, long long ldw,
                   const float* bias, float* Y, long long ldy, int M, int N, int K) {
  using namespace vt;
  if (M < 0 || N < 0 || K < 0) return set_error(E_SHAPE, "vt_head_linear: negative shape");
  if (M == 0 || N == 0) return OK;
  if (K == 0 || !X || !Wt || !Y) return set_error(E_SHAPE, "vt_head_linear: K must be >= 1 and pointers non-null");
  if (ldx < K || ldw < N || ldy < N) return set_error(E_SHAPE, "vt_head_linear: pitches smaller than the rows");
  const long long xe = x_bf16 ? 2 : 4;
  if (aligned16(X) && aligned16(Wt) && (ldx * xe) % 16 == 0 && ldw % 4 == 0 && N % 4 == 0 && (K * xe) % 16 == 0) {
    const dim3 pgrid((N + heads::PBN - 1) / heads::PBN, (M + heads::PBM - 1) / heads::PBM);
    if (pgrid.y > 65535) return set_error(E_SHAPE, "vt_head_linear: M=%d too large", M);
    if (x_bf16)
      launch_k(heads::head_linear_pipe_kernel<true>, pgrid, heads::PTHREADS, 0, st, X, ldx, Wt, ldw, bias, Y, ldy, M, N, K);
    else
      launch_k(heads::head_linear_pipe_kernel<false>, pgrid, heads::PTHREADS, 0, st, X, ldx, Wt, ldw, bias, Y, ldy, M, N, K);
    return check_launch("vt_head_linear");
  }
  const dim3 grid((N + heads::BN - 1) / heads::BN, (M + heads::BM - 1) / heads::BM);
  if (grid.y > 65535) return set_error(E_SHAPE, "vt_head_linear: M=%d too large", M);
  if (x_bf16)
    launch_k(heads::head_linear_kernel<true>, grid, 256, 0, st, X, ldx, Wt, ldw, bias, Y, ldy, M, N, K);
  else
    launch_k(heads::head_linear_kernel<false>, grid, 256, 0, st, X, ldx, Wt, ldw, bias, Y, ldy, M, N, K);
  return check_launch("vt_head_linear");
}

int vt_head_ln_gelu(cudaStream_t st, float* Y, long long ldy, int rows, int N, const float* gamma, const float* beta,
                    int groups, float eps) {
  using namespace vt;
  if (rows < 0) return set_error(E_SHAPE, "vt_head_ln_gelu: negative rows");
  if (rows == 0) return OK;
  if (!Y || !gamma || !beta || groups < 1 || ldy < N) return set_error(E_SHAPE, "vt_head_ln_gelu: bad arguments");
  const int grid = (rows + 7) / 8;
  if (N == 256) launch_k(heads::head_ln_gelu_kernel<8>, grid, 256, 0, st, Y, ldy, rows, gamma, beta, groups, eps);
  else if (N == 512) launch_k(heads::head_ln_gelu_kernel<16>, grid, 256, 0, st, Y, ldy, rows, gamma, beta, groups, eps);
  else return set_error(E_VARIANT, "vt_head_ln_gelu: N=%d unsupported (256 or 512)", N);
  return check_launch("vt_head_ln_gelu");
}

int vt_soft_argmax(cudaStream_t st, const float* logits, long long ldl, int Q, int bins, int window, float temperature,
                   float* tracks, long long ldt) {
  using namespace vt;
  if (Q < 0) return set_error(E_SHAPE, "vt_soft_argmax: negative Q");
  if (Q == 0) return OK;
  if (!logits || !tracks || ldl < 2LL * bins || ldt < 2 || window < 0)
    return set_error(E_SHAPE, "vt_soft_argmax: bad arguments");
  const int grid = (2 * Q + 7) / 8;
  if (bins == 256)
    launch_k(heads::soft_argmax_kernel<8>, grid, 256, 0, st, logits, ldl, Q, window, temperature, tracks, ldt);
  else if (bins == 512)
    launch_k(heads::soft_argmax_kernel<16>, grid, 256, 0, st, logits, ldl, Q, window, temperature, tracks, ldt);
  else return set_error(E_VARIANT, "vt_soft_argmax: %d bins unsupported (256 or 512)", bins);
  return check_launch("vt_soft_argmax");
}

}  // extern "C"
