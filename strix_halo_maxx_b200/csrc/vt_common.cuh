// Shared device helpers for the sm_100a kernels of libvt_b200.so: bf16 conversion, bounded
// mbarrier waits, TMA tile loads, tcgen05 (UMMA / TMEM) wrappers and the shared-memory matrix
// descriptors they consume.  Everything here is hand-written inline PTX for sm_100a.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vt {

// ---------------------------------------------------------------- status word
// Kernels never trap.  A wait that runs out of budget ORs a site bit into this word, the kernel
// unwinds (draining its own copies and MMAs) and the host reads the word with vt_device_status().
// Defined here: libvt_b200.so is one translation unit (vt_b200.cu includes every .cu file).
__device__ unsigned int g_status = 0;
enum : unsigned int {
  ST_GEMM_PRODUCER = 1u << 0,
  ST_GEMM_MMA = 1u << 1,
  ST_GEMM_EPILOGUE = 1u << 2,
  ST_GEMM_DRAIN = 1u << 3,
  ST_ATTN_PRODUCER = 1u << 4,
  ST_ATTN_MMA = 1u << 5,
  ST_ATTN_SOFTMAX = 1u << 6,
  ST_SSM_MMA = 1u << 7,
  ST_SELFTEST = 1u << 8,  // vt_wait_selftest
};
// A wait gives up after this many SM clock cycles (~2 s at 1.9 GHz); legitimate waits are microseconds.
constexpr long long kSpinCycles = 4000000000LL;

// ---------------------------------------------------------------- bf16
// fp32 -> bf16 with round-to-nearest-even (the cvt instruction; one instruction per pair for pack_bf2).
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
}
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ float bfround(float f) { return bf2f(f2bf(f)); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {  // lo -> bits 0..15, hi -> bits 16..31
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Hardware approximations (single MUFU instructions): 2^x and tanh(x).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Blackwell three-input max and packed fp32x2 arithmetic (one instruction for two lanes of work).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), with the hardware tanh
// (max relative error about 2^-11, below the bf16 rounding the GEMM epilogue applies next).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.0f + tanh_approx(u));
}
// The same on two lanes: u = x (k0 + k1 x^2), gelu = h + h tanh(u) with h = x / 2.
__device__ __forceinline__ unsigned long long gelu_tanh2(unsigned long long x) {
  const unsigned long long k0 = f2_pack(0.7978845608028654f, 0.7978845608028654f);
  const unsigned long long k1 = f2_pack(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f);
  const unsigned long long half = f2_pack(0.5f, 0.5f);
  const unsigned long long u = f2_mul(x, f2_fma(k1, f2_mul(x, x), k0));
  float u0, u1;
  f2_unpack(u, u0, u1);
  const unsigned long long h = f2_mul(half, x);
  return f2_fma(h, f2_pack(tanh_approx(u0), tanh_approx(u1)), h);
}

// x / d rounded to nearest even, for many x and one d > 0 (normal) whose correctly rounded reciprocal
// rd = __frcp_rn(d) the caller computed once.  q = x * rd is within 1.5 ulp of x / d; a first correction
// q + (x - q d) rd (the residual formed in one FMA) brings it within one ulp, and by Markstein's theorem
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990: with rd within half an ulp of 1/d and q within one ulp of
// x / d, the FMA residual is exact and q + r rd rounds to the correctly rounded quotient) the second
// correction returns exactly the IEEE quotient.  Five FP operations instead of a full division; valid
// while the residual does not underflow (|x| above ~1e-30 here, far below any quotient whose rounding
// matters to the int8 result).
__device__ __forceinline__ float div_rn_by(float x, float d, float rd) {
  float q = __fmul_rn(x, rd);
  q = __fmaf_rn(__fmaf_rn(-q, d, x), rd, q);
  return __fmaf_rn(__fmaf_rn(-q, d, x), rd, q);
}

// GELU-tanh as x * sigmoid(2u) = x / (1 + e^(-2u)), u = sqrt(2/pi) (x + 0.044715 x^3): the function of
// 0.5 x (1 + tanh u) (the int8 epilogue's GELU, i8gemm.hip:11, there with tanh u = 1 - 2 / (1 + e^(2u)))
// without the cancellation of 1 + tanh u in the negative tail, so the relative error stays near 1e-6
// everywhere (tanh.approx leaves an absolute error near 1e-3 there); two MUFU operations (ex2, rcp).
// e^(-2u) = inf gives -0, e^(-2u) = 0 gives x.
__device__ __forceinline__ float gelu_sigmoid(float x) {
  constexpr float k = -2.0f * 1.4426950408889634f * 0.7978845608028654f;  // -2 log2(e) sqrt(2/pi)
  const float z = k * x * fmaf(0.044715f, x * x, 1.0f);                     // -2u log2(e)
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(z));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return x * r;
}

// RG-LRU element step (tapnext/npu/r9/cpuemu.py:33-47) in fp32: u the normed input, gx_pre / ga_pre the gate
// pre-activations, sp = softplus(a_param) of the channel (computed once per channel by the caller), h0 the state
// (unused when first).  h = u sigmoid(gx) on a sequence's first frame, else a h0 + u sigmoid(gx) sqrt(1 - a^2)
// with log a = -c sigmoid(ga) sp.  The sigmoids and a = exp(log a) take the hardware exponential and division
// (__expf, __fdividef: a few ulp, far inside the RG-LRU's tolerances); 1 - a^2 keeps expm1f, which a near 1
// needs.  Shared by vt_rglru and vt_rglru_fold, so both give the same numbers.
__device__ __forceinline__ float rglru_elem(float u, float gx_pre, float ga_pre, float sp, float h0, float c,
                                            bool first) {
  const float gated = u * __fdividef(1.0f, 1.0f + __expf(-gx_pre));
  if (first) return gated;
  const float log_a = -c * __fdividef(1.0f, 1.0f + __expf(-ga_pre)) * sp;
  return __expf(log_a) * h0 + gated * sqrtf(-expm1f(2.0f * log_a));
}

// Attention-tile layout: offset (bf16 elements) of row t, 8-element d chunk c of operand w (0 q, 1 k, 2 v)
// within one (crop, operand, head) block of ceil(T/128) tiles of NC * 1024 elements.  A Q tile is
// [c][128 rows][8]; a K or V tile is two 64-row halves [half][c][64 rows][8], so each 64-key tile the
// attention kernel streams is one contiguous NC KB copy.  Both are the canonical no-swizzle layout of
// 8-row x 16-byte core matrices that tcgen05 descriptors address.
__device__ __forceinline__ size_t attn_tile_off(int w, int t, int c, int NC) {
  const size_t tile = (size_t)(t >> 7) * NC * 1024;
  if (w == 0) return tile + (size_t)c * 1024 + (size_t)(t & 127) * 8;
  return tile + (size_t)((t >> 6) & 1) * NC * 512 + (size_t)c * 512 + (size_t)(t & 63) * 8;
}

// Programmatic dependent launch (see launch_k in vt_host.h): griddep_wait blocks until the previous kernel
// in the stream has completed and its memory is visible (a no-op when launched without the attribute);
// griddep_launch lets the next kernel start launching once every CTA of this one has called it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of `parity` to complete.  Returns false if another role of this CTA has
// aborted (flag set) or if the wait outlives `limit` cycles (kSpinCycles for mbar_wait), in which case
// it sets the flag and records `site` in g_status.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              unsigned int site, long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255u) == 0) {
      if (*abort_flag) return false;
      if (clock64() - t0 > limit) {
        *abort_flag = 1;
        atomicOr(&g_status, site);
        return false;
      }
    }
  }
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int site) {
  return mbar_wait_for(bar, parity, abort_flag, site, kSpinCycles);
}
// Bounded wait used while unwinding: ignores the abort flag, gives up after `cycles`.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, long long cycles) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > cycles) {
      atomicOr(&g_status, (unsigned int)ST_GEMM_DRAIN);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA (every load reads this GPU and fills one CTA)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)m) : "memory");
}
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* m, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)m), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// TMA store of a shared-memory box to global memory (bulk-group completion), and the bulk-group waits:
// wait_read<N> returns once at most N groups still read shared memory, wait_all<N> once at most N are
// incomplete.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)m),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same for signed 8-bit operands (kind::i8, K = 32 per instruction, s32 accumulators in TMEM).
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier gets one arrive once every tcgen05 op this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
// The same with A in tensor memory (rows = lanes, two bf16 per 32-bit column, K-major).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Non-tensor bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completion
// counted on the mbarrier; it fills only the issuing CTA.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (tensor core reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- CTA pairs (cluster of 2, cta_group::2)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// 16-byte store into the shared memory of a CTA of this cluster (a shared::cluster address from mapa_shared).
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load issued by either CTA of a pair; completion is counted on the mbarrier at `bar_addr`, a
// shared::cluster address (the leader CTA's barrier); it fills only the issuing CTA.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* m, uint32_t bar_addr, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)m), "r"(bar_addr), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {  // one warp of each CTA
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs] * B[smem of both CTAs]^T, M = 256 across the pair.
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// One arrive on the mbarrier at shared::cluster address `bar_addr` (this or the peer CTA) once every
// tcgen05 op this thread issued before has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_addr)
               : "memory");
}

// Shared-memory matrix descriptor without swizzle (canonical "interleave" layout of 8-row x 16-byte core
// matrices): lbo / sbo are the byte distances between core matrices along the leading / strided
// dimension, as tcgen05 defines them for the operand's major-ness.
__device__ __forceinline__ uint64_t sdesc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version; layout type 0 = SWIZZLE_NONE
  return d;
}

// Shared-memory matrix descriptor, K-major operand written by TMA with 128-byte swizzle: rows of
// 64 bf16 (128 B), 8-row groups 1024 B apart (SBO), version 1 (sm_100), layout SWIZZLE_128B.
// The tile base must be 1024-byte aligned; stepping K by 16 elements adds 32 B to the start.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // LBO: unused for swizzled K-major layouts
  d |= (uint64_t)(1024 >> 4) << 32;   // SBO
  d |= (uint64_t)1 << 46;             // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// kind::i8: s32 accumulator (bits 4-5 = 2), signed 8-bit A and B (bits 7-9, 10-12 = 1), both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace vt
