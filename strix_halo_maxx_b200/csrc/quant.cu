// Per-token int8 activation quantisation for the W8A8 GEMM (vt_gemm_i8): the replacement of the
// reference's quant_rows (moondream/gpu/tgemm.py:81-91 `_quant_rows`, called through hgemm.py:10-16 and
// HI8Lin.quant, hgemm.py:116-117).  Row m of x (bf16) becomes
//     s[m] = max(max_k |x[m,k]|, 1e-5) / 127
//     q[m,k] = trunc(x[m,k] / s[m] + (x / s >= 0 ? 0.5 : -0.5))      (round half away from zero)
// with IEEE fp32 division (div_rn_by: the correctly rounded quotient from one reciprocal per row) and
// addition, clamped to [-127, 127] (a no-op: |x / s| <= 127 within rounding).
// One CTA of 256 threads per row; the row stays in registers between the max and the quantisation pass
// (16-byte loads of 8 bf16 values, G of them per thread, K <= 2048 * G).
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace quant {

constexpr int QT = 256;

template <int G>
__global__ void __launch_bounds__(QT) quant_rows_kernel(const uint16_t* __restrict__ x, long long ldx, int K,
                                                        int8_t* __restrict__ q, long long ldq, float* __restrict__ s) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  __shared__ float red[QT / 32];
  const long long row = blockIdx.x;
  const int ng = K / 8;
  const uint16_t* xr = x + row * ldx;
  uint4 u[G];
  float amax = 0.f;
#pragma unroll
  for (int g = 0; g < G; g++) {
    const int idx = g * QT + threadIdx.x;
    if (idx < ng) {
      u[g] = *reinterpret_cast<const uint4*>(xr + 8LL * idx);
      const uint32_t w[4] = {u[g].x, u[g].y, u[g].z, u[g].w};
#pragma unroll
      for (int e = 0; e < 4; e++)
        amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(w[e] << 16)), fabsf(__uint_as_float(w[e] & 0xffff0000u))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < QT / 32; i++) amax = fmaxf(amax, red[i]);
  const float sc = __fdiv_rn(fmaxf(amax, 1e-5f), 127.f);
  const float rsc = __frcp_rn(sc);
  int8_t* qr = q + row * ldq;
#pragma unroll
  for (int g = 0; g < G; g++) {
    const int idx = g * QT + threadIdx.x;
    if (idx < ng) {
      const uint32_t w[4] = {u[g].x, u[g].y, u[g].z, u[g].w};
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const float xv = (e & 1) ? __uint_as_float(w[e >> 1] & 0xffff0000u) : __uint_as_float(w[e >> 1] << 16);
        const float v = div_rn_by(xv, sc, rsc);  // == xv / sc (IEEE)
        int qi = __float2int_rz(__fadd_rn(v, v >= 0.f ? 0.5f : -0.5f));
        qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
        packed[e >> 2] |= ((uint32_t)qi & 0xffu) << (8 * (e & 3));
      }
      *reinterpret_cast<uint2*>(qr + 8LL * idx) = make_uint2(packed[0], packed[1]);
    }
  }
  if (threadIdx.x == 0) s[row] = sc;
}

}  // namespace quant
}  // namespace vt

extern "C" {

// q[M, K] int8 (pitch ldq bytes) and s[M] fp32 from x[M, K] bf16 (pitch ldx elements); K % 8 == 0,
// K <= 16384, x 16-byte aligned with ldx % 8 == 0, q 8-byte aligned with ldq % 8 == 0.
int vt_quant_rows(cudaStream_t st, const uint16_t* x, long long ldx, int M, int K, int8_t* q, long long ldq,
                  float* s) {
  using namespace vt;
  if (M < 0 || K <= 0 || K % 8 || K > 16384)
    return set_error(E_SHAPE, "vt_quant_rows: M=%d K=%d (K a multiple of 8, at most 16384)", M, K);
  if (M == 0) return OK;
  if (!x || !q || !s || !aligned16(x) || ldx < K || ldx % 8 || ldq < K || ldq % 8 ||
      (reinterpret_cast<uintptr_t>(q) & 7))
    return set_error(E_SHAPE, "vt_quant_rows: x / q alignment or pitch (ldx=%lld ldq=%lld)", ldx, ldq);
  const int ng = K / 8;
  const dim3 grid((unsigned)M);
  if (ng <= 1 * quant::QT) launch_k(quant::quant_rows_kernel<1>, grid, quant::QT, 0, st, x, ldx, K, q, ldq, s);
  else if (ng <= 2 * quant::QT) launch_k(quant::quant_rows_kernel<2>, grid, quant::QT, 0, st, x, ldx, K, q, ldq, s);
  else if (ng <= 4 * quant::QT) launch_k(quant::quant_rows_kernel<4>, grid, quant::QT, 0, st, x, ldx, K, q, ldq, s);
  else launch_k(quant::quant_rows_kernel<8>, grid, quant::QT, 0, st, x, ldx, K, q, ldq, s);
  return check_launch("vt_quant_rows");
}

}  // extern "C"
