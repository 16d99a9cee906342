// Mask-free, non-causal flash attention:  O = softmax(Q K^T * scale) V  per (crop, head),
// the replacement of the reference's attn_fwd2 / vtranspose (moondream/gpu/hip/attn.hip:142-288,
// 433-462) behind hattn.Attn (moondream/gpu/hattn.py:17-37).
//
// Q, K, V are read in place from any [batch][token][head][d] strides -- for the tower that is the
// fused QKV GEMM output [T, 3*H*D] -- so no transposed copy of V is made.  head_dim D (a multiple of 8,
// <= 80) is zero-padded in shared memory to DP = 64 or 80, the tensor-core K granularity; pad lanes are
// exact zeros (cp.async zero fill).  Online softmax in base 2; P is rounded to bf16 and the row sum is
// taken over the rounded P (as attn.hip:225-226 does), accumulation in fp32.
//
// CTA = 8 warps x 16 query rows = 128 queries of one (crop, head); K/V stream through a double-
// buffered 64-key shared-memory ring filled by cp.async.
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace attn {

constexpr int BQ = 128, BKV = 64, THREADS = 256;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Args {
  const uint16_t *q, *k, *v;
  uint16_t* o;
  int T, D;
  long long sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h, so_b, so_t, so_h;
  float scale_log2;
  int b0;  // first crop of this launch
};

template <int DP>
__global__ void __launch_bounds__(THREADS) attn_fwd_mma_kernel(Args a) {
  constexpr int LD = DP + 8;  // row pitch in elements: an odd number of 16-byte chunks (conflict-free ldmatrix)
  constexpr int NCH = DP / 8;
  extern __shared__ uint8_t smraw[];
  uint16_t* Qs = reinterpret_cast<uint16_t*>(smraw);
  uint16_t* Ks = Qs + BQ * LD;        // [2][BKV][LD]
  uint16_t* Vs = Ks + 2 * BKV * LD;   // [2][BKV][LD]

  const int b = a.b0 + blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * BQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, dch = a.D / 8;
  const uint16_t* Qb = a.q + b * a.sq_b + h * a.sq_h;
  const uint16_t* Kb = a.k + b * a.sk_b + h * a.sk_h;
  const uint16_t* Vb = a.v + b * a.sv_b + h * a.sv_h;

  for (int i = tid; i < BQ * NCH; i += THREADS) {
    const int r = i / NCH, c = i % NCH, t = q0 + r;
    const bool ok = (t < T) && (c < dch);
    cp_async16(Qs + r * LD + c * 8, ok ? (const void*)(Qb + (long long)t * a.sq_t + c * 8) : (const void*)Qb, ok);
  }
  auto load_kv = [&](int j, int buf) {
    const int k0 = j * BKV;
    uint16_t* kd = Ks + buf * BKV * LD;
    uint16_t* vd = Vs + buf * BKV * LD;
    for (int i = tid; i < BKV * NCH; i += THREADS) {
      const int r = i / NCH, c = i % NCH, t = k0 + r;
      const bool ok = (t < T) && (c < dch);
      cp_async16(kd + r * LD + c * 8, ok ? (const void*)(Kb + (long long)t * a.sk_t + c * 8) : (const void*)Kb, ok);
      cp_async16(vd + r * LD + c * 8, ok ? (const void*)(Vb + (long long)t * a.sv_t + c * 8) : (const void*)Vb, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int nkv = (T + BKV - 1) / BKV;
  uint32_t qf[DP / 16][4];
  float o[DP / 8][4];
#pragma unroll
  for (int i = 0; i < DP / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int quad = lane & 3;

  for (int j = 0; j < nkv; j++) {
    if (j + 1 < nkv) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; kk++)
        ldsm_x4(qf[kk], Qs + (warp * 16 + (lane & 15)) * LD + kk * 16 + (lane >> 4) * 8);
    }
    const uint16_t* Kt = Ks + (j & 1) * BKV * LD;
    const uint16_t* Vt = Vs + (j & 1) * BKV * LD;

    float s[BKV / 8][4];
#pragma unroll
    for (int i = 0; i < BKV / 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; kk++) {
#pragma unroll
      for (int np = 0; np < BKV / 16; np++) {
        uint32_t kb[4];
        ldsm_x4(kb, Kt + (np * 16 + (lane >> 4) * 8 + (lane & 7)) * LD + kk * 16 + ((lane >> 3) & 1) * 8);
        mma16816(s[2 * np], qf[kk], kb[0], kb[1]);
        mma16816(s[2 * np + 1], qf[kk], kb[2], kb[3]);
      }
    }
    // scale, mask the key tail, online softmax (rows lane/4 and lane/4 + 8 of this warp's 16)
    const int kbase = j * BKV;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < BKV / 8; nt++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int key = kbase + nt * 8 + 2 * quad + (e & 1);
        const float val = key < T ? s[nt][e] * a.scale_log2 : -INFINITY;
        s[nt][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      mnew[r] = fmaxf(mrow[r], mx[r]);
      alpha[r] = exp2f(mrow[r] - mnew[r]);
      mrow[r] = mnew[r];
    }
    uint32_t pk[BKV / 8][2];
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < BKV / 8; nt++) {
      const float p0 = bfround(exp2f(s[nt][0] - mnew[0])), p1 = bfround(exp2f(s[nt][1] - mnew[0]));
      const float p2 = bfround(exp2f(s[nt][2] - mnew[1])), p3 = bfround(exp2f(s[nt][3] - mnew[1]));
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pk[nt][0] = pack_bf2(p0, p1);
      pk[nt][1] = pack_bf2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      lrow[r] = lrow[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < DP / 8; i++) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kk = 0; kk < BKV / 16; kk++) {
      const uint32_t pa[4] = {pk[2 * kk][0], pk[2 * kk][1], pk[2 * kk + 1][0], pk[2 * kk + 1][1]};
#pragma unroll
      for (int dp = 0; dp < DP / 16; dp++) {
        uint32_t vb[4];
        ldsm_x4_t(vb, Vt + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + dp * 16 + (lane >> 4) * 8);
        mma16816(o[2 * dp], pa, vb[0], vb[1]);
        mma16816(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();
  }
  const float inv0 = 1.f / lrow[0], inv1 = 1.f / lrow[1];
  const int t0 = q0 + warp * 16 + (lane >> 2), t1 = t0 + 8;
  uint16_t* Ob = a.o + b * a.so_b + h * a.so_h;
#pragma unroll
  for (int nt = 0; nt < DP / 8; nt++) {
    const int d = nt * 8 + 2 * quad;
    if (d < a.D) {
      if (t0 < T) *reinterpret_cast<uint32_t*>(Ob + (long long)t0 * a.so_t + d) = pack_bf2(o[nt][0] * inv0, o[nt][1] * inv0);
      if (t1 < T) *reinterpret_cast<uint32_t*>(Ob + (long long)t1 * a.so_t + d) = pack_bf2(o[nt][2] * inv1, o[nt][3] * inv1);
    }
  }
}

template <int DP>
static int launch_dp(cudaStream_t st, Args a, int B, int H) {
  constexpr int LD = DP + 8;
  constexpr int SMEM = (BQ + 4 * BKV) * LD * 2;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(attn_fwd_mma_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    attr_done[dev] = true;
  }
  for (int b0 = 0; b0 < B; b0 += 65535) {
    a.b0 = b0;
    const int nb = (B - b0) < 65535 ? (B - b0) : 65535;
    dim3 grid((a.T + BQ - 1) / BQ, H, nb);
    attn_fwd_mma_kernel<DP><<<grid, THREADS, SMEM, st>>>(a);
    int rc = check_launch("vt_attn_fwd");
    if (rc) return rc;
  }
  return OK;
}

}  // namespace attn
}  // namespace vt

extern "C" {

// O[b, t, h, :D] = softmax(Q[b, :, h] K[b, :, h]^T * scale) V[b, :, h] for every crop b < B and head h < H.
// Element (b, t, h, d) of X lives at X + b*sx_b + t*sx_t + h*sx_h + d.  D must be a multiple of 8 and
// <= 80; all strides of Q/K/V multiples of 8 elements, bases 16-byte aligned; O strides even.
int vt_attn_fwd(cudaStream_t st, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int B, int T,
                int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b, long long sk_t,
                long long sk_h, long long sv_b, long long sv_t, long long sv_h, long long so_b, long long so_t,
                long long so_h, float scale) {
  using namespace vt;
  if (B < 0 || T < 0 || H < 0 || D < 0) return set_error(E_SHAPE, "vt_attn_fwd: negative shape");
  if (B == 0 || T == 0 || H == 0) return OK;
  if (H > 65535) return set_error(E_SHAPE, "vt_attn_fwd: H=%d too large", H);
  if (D == 0 || D % 8 || D > 80) return set_error(E_VARIANT, "vt_attn_fwd: head_dim %d unsupported (multiple of 8, <= 80)", D);
  if (!Q || !K || !V || !O) return set_error(E_SHAPE, "vt_attn_fwd: null pointer");
  const long long s16[] = {sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h};
  for (long long s : s16)
    if (s % 8) return set_error(E_SHAPE, "vt_attn_fwd: Q/K/V strides must be multiples of 8 elements");
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V)) return set_error(E_SHAPE, "vt_attn_fwd: Q/K/V must be 16-byte aligned");
  if ((so_b | so_t | so_h) & 1 || (reinterpret_cast<uintptr_t>(O) & 3))
    return set_error(E_SHAPE, "vt_attn_fwd: O strides must be even and O 4-byte aligned");
  attn::Args a{Q, K, V, O, T, D, sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h, so_b, so_t, so_h,
               scale * 1.4426950408889634f, 0};
  if (D <= 64) return attn::launch_dp<64>(st, a, B, H);
  return attn::launch_dp<80>(st, a, B, H);
}

}  // extern "C"
