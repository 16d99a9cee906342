// bf16 and W8A8 int8 GEMMs on the 5th-generation tensor cores (tcgen05 / TMEM, operands staged by TMA):
//     C[M, N] = epilogue( A[M, K] . W[N, K]^T )
// the replacement of the reference's bf16gemm_kernel / bf16gemm_launch
// (moondream/gpu/hip/i8gemm.hip:286-385, 534-552) that HLin calls (moondream/gpu/hgemm.py:139-178), and, with
// I8 = true (signed int8 operands, kind::i8, s32 accumulators scaled in the epilogue), of the int8 kernels
// i8gemm_launch / i8gemm_small_launch (i8gemm.hip:91-204, 480-593) that HI8Lin calls (hgemm.py:95-137).
//
// Design (one CTA per SM, persistent over output tiles):
//   * tile 128 x 256 x 64, 4-stage shared-memory ring (48 KB per stage), 128-byte swizzle;
//   * warp 0 lane 0 issues the TMA loads (each fills only its own CTA), warp 1 lane 0 issues tcgen05.mma
//     (M=128, N=256, K=16 each, fp32 accumulators in TMEM), warps 2-9 run the epilogue (two warps per
//     TMEM lane quarter, each on half of the tile's columns, so one warp's loads hide behind the other's);
//   * two 256-column TMEM accumulators, so the epilogue of tile i overlaps the MMAs of tile i+1;
//   * tiles are walked N-fastest, so the CTAs resident at one time share A rows and the whole of W
//     through L2;
//   * epilogue: + bias, then either bf16 output (optionally GELU-tanh applied after rounding to bf16,
//     as i8gemm.hip:378 does) or fp32 output with a residual / periodic addend (fp32 or bf16) and an
//     optional bf16 copy.  M, N and K tails are handled by TMA zero fill and masked stores.
// The CTA-pair kernel below (256 x 256 or 256 x 128 tiles, cta_group::2) runs every GEMM with enough rows
// to give the SM pairs work; the single-CTA kernel takes the rest (128 x 256, or 128 x 64 with split K).
#include <cstdlib>

#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace gemm {

// Tile shape: BM x BN x BK with BN 256 (default) or 192.
constexpr int BM = 128, BK = 64;
constexpr int EPI_WARPS = 8;                 // two warps per TMEM lane quarter, each owning half the columns
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr long long kDrainCycles = 200000000LL;
template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 192) ? 5 : 8;  // BN 64: 24 KB stages
  static constexpr uint32_t TMEM_COLS = 512;  // two BN-column accumulators, rounded to a power of two
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
};

struct Epi {
  const float* bias;  // [N] fp32 or null
  void* out;          // [M][ldo], bf16 or fp32
  long long ldo;
  const void* res;    // addend [rows][ldr] or null; row = m % res_period when res_period > 0
  long long ldr;
  int res_period;
  int res_bf16;
  int out_f32;
  int gelu;
  uint16_t* out2;     // optional bf16 copy of an fp32 output, [M][ldo2]
  long long ldo2;
  // attention-tile output (pk_T > 0): the bf16 result [M = crops*T][3*H*D] is scattered into the tile
  // layout vt_attn_tiles_fwd reads: element (b, w, h, t, d) at ((b*3 + w)*H + h)*Tt*NC*1024 +
  // attn_tile_off(w, t, d/8, NC) + d%8
  int pk_T, pk_H, pk_D, pk_NC, pk_Tt;
  // row statistics of an fp32 output (stats_out != null, N % 32 == 0): for every 32-column chunk j of
  // row m, stats_out[m * N/32 + j] = (chunk mean, chunk sum of squared deviations)
  float2* stats_out;
  // LayerNorm folded into this GEMM (ln_moments != null): A holds bf16 x, W holds W * diag(gamma), and
  // the accumulator becomes rstd * (acc - mean * ln_c[n]) (+ bias = b + W beta), with (mean, rstd) of
  // row m read from ln_moments[m] (written by vt_row_moments from the chunk statistics)
  const float2* ln_moments;
  const float* ln_c;
  // all row-major outputs / the residual are 32-byte aligned with 32-byte multiple pitches: full chunks
  // use 256-bit accesses (set by the launcher)
  int wide;
  // split-K (128 x 64 tiles only, ksplit > 1; set by the launcher when the caller passes a workspace): the
  // K range of a tile is cut into ksplit slices computed by different CTAs.  Slice s stores its fp32
  // partial into sk_ws + s * M * sk_pitch ([M][sk_pitch]) and counts itself in sk_cnt [M][sk_pitch / 32]
  // per 32-column chunk of a row; the slice that arrives last adds the ksplit partials in slice order
  // (so the result does not depend on which CTA finished first), runs the epilogue above on the sum and
  // puts the counter back to zero for the next call.
  float* sk_ws;
  int* sk_cnt;
  int sk_pitch;
  int ksplit;
  // W8A8 int8 operands (the I8 kernel instantiations, vt_gemm_i8): the accumulator is the exact int32 dot
  // product of the int8 rows, scaled as ((float)acc * i8_sa[m]) * i8_sw[n] before the bias, the order of
  // the reference's int8 epilogue (moondream/gpu/hip/i8gemm.hip:183-197); gelu = 2 there applies GELU-tanh to
  // the fp32 value in the sigmoid form (gelu_sigmoid; gelu = 1: tanh.approx on the bf16-rounded value, the
  // bf16 GEMM's rule)
  const float* i8_sa;
  const float* i8_sw;
  // The same LayerNorm / RMSNorm fold with the row factors merged here from chunk statistics (ln_stats != null
  // instead of ln_moments; vt_gemm_fused_lnstats): ln_stats[m * ln_nchunk + j] = (mean, M2) of 32-column chunk
  // j of row m, merged as vt_row_moments / vt_row_rms do (ln_rms: mean 0, rstd from the mean square); the
  // tiles of column block 0 also store (mean, rstd) of their rows in ln_mom_out when it is set
  const float2* ln_stats;
  int ln_nchunk;
  float ln_eps;
  int ln_rms;
  float2* ln_mom_out;
};

__host__ __device__ __forceinline__ bool ln_folded(const Epi& ep) { return ep.ln_moments || ep.ln_stats; }

// (mean, rstd) of A row m for a folded norm (left as (0, 1) without one); issued by the epilogue threads before
// they wait for the tile's accumulator, so the loads overlap the MMAs.  The merge is vt_row_moments' (mean of
// the chunk means, M2 = sum of chunk M2 + 32 (chunk mean - mean)^2) summed in chunk order by one thread.
__device__ __forceinline__ void ln_row_factors(const Epi& ep, int m, int M, bool store, float& mu, float& rstd) {
  if (m >= M) return;
  if (ep.ln_moments) {
    const float2 mr = ep.ln_moments[m];
    mu = mr.x;
    rstd = mr.y;
    return;
  }
  if (!ep.ln_stats) return;
  const float2* st = ep.ln_stats + (size_t)m * ep.ln_nchunk;
  const int n = ep.ln_nchunk;
  const float inv = 1.f / (32.f * (float)n);
  if (ep.ln_rms) {
    float q = 0.f;
#pragma unroll 4
    for (int i = 0; i < n; i++) {
      const float2 v = st[i];
      q += v.y + 32.f * v.x * v.x;
    }
    mu = 0.f;
    rstd = rsqrtf(q * inv + ep.ln_eps);
  } else {
    float sum = 0.f;
#pragma unroll 4
    for (int i = 0; i < n; i++) sum += st[i].x;
    mu = sum / (float)n;
    float m2 = 0.f;
#pragma unroll 4
    for (int i = 0; i < n; i++) {
      const float2 v = st[i];
      const float d = v.x - mu;
      m2 += v.y + 32.f * d * d;
    }
    rstd = rsqrtf(m2 * inv + ep.ln_eps);
  }
  if (store && ep.ln_mom_out) ep.ln_mom_out[m] = make_float2(mu, rstd);
}

// Split-K slices of one launch (the workspace holds this many partial planes).
constexpr int kMaxSplit = 16;

// 32 consecutive 32-bit words at p: 256-bit accesses (one full 32-byte sector each, p 32-byte aligned) when
// wide, else 128-bit ones.
__device__ __forceinline__ void ld_words32(const void* p, uint32_t (&w)[32], bool wide) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
  if (wide) {
#pragma unroll
    for (int i = 0; i < 4; i++)
      asm volatile("ld.global.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(w[8 * i]), "=r"(w[8 * i + 1]), "=r"(w[8 * i + 2]), "=r"(w[8 * i + 3]), "=r"(w[8 * i + 4]),
                     "=r"(w[8 * i + 5]), "=r"(w[8 * i + 6]), "=r"(w[8 * i + 7])
                   : "l"(q + 8 * i));
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint4 u = *reinterpret_cast<const uint4*>(q + 4 * i);
      w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
    }
  }
}
template <int NW>  // NW = 8, 16 or 32 words (32-byte aligned when wide)
__device__ __forceinline__ void st_words(void* p, const uint32_t* w, bool wide) {
  uint32_t* q = reinterpret_cast<uint32_t*>(p);
  if (wide) {
#pragma unroll
    for (int i = 0; i < NW / 8; i++)
      asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(q + 8 * i), "r"(w[8 * i]), "r"(w[8 * i + 1]),
                   "r"(w[8 * i + 2]), "r"(w[8 * i + 3]), "r"(w[8 * i + 4]), "r"(w[8 * i + 5]), "r"(w[8 * i + 6]),
                   "r"(w[8 * i + 7])
                   : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < NW / 4; i++)
      *reinterpret_cast<uint4*>(q + 4 * i) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

// The scalar path for a chunk that crosses N (only the last column tile of a launch).
__device__ __forceinline__ void epilogue_chunk_partial(const uint32_t (&r)[32], int m, int n0, int N, const Epi& ep, float mu,
                                               float rstd) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
  const bool full = (n0 + 32 <= N);
  if (ep.i8_sw) {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (n0 + j < N) v[j] = __fmul_rn(v[j], ep.i8_sw[n0 + j]);
  }
  if (ln_folded(ep)) {
    if (full) {
      const float4* c4 = reinterpret_cast<const float4*>(ep.ln_c + n0);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float4 c = __ldg(c4 + j);
        v[4 * j] = rstd * fmaf(-mu, c.x, v[4 * j]);
        v[4 * j + 1] = rstd * fmaf(-mu, c.y, v[4 * j + 1]);
        v[4 * j + 2] = rstd * fmaf(-mu, c.z, v[4 * j + 2]);
        v[4 * j + 3] = rstd * fmaf(-mu, c.w, v[4 * j + 3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n0 + j < N) v[j] = rstd * fmaf(-mu, ep.ln_c[n0 + j], v[j]);
    }
  }
  if (ep.bias) {
    if (full) {
      const float4* b4 = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float4 b = __ldg(b4 + j);
        v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n0 + j < N) v[j] += ep.bias[n0 + j];
    }
  }
  if (ep.res) {
    const long long rr = ep.res_period > 0 ? (long long)(m % ep.res_period) : (long long)m;
    if (ep.res_bf16) {
      const uint16_t* rp = reinterpret_cast<const uint16_t*>(ep.res) + rr * ep.ldr + n0;
      if (full) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const uint4 u = *reinterpret_cast<const uint4*>(rp + 8 * j);
          w[4 * j] = u.x; w[4 * j + 1] = u.y; w[4 * j + 2] = u.z; w[4 * j + 3] = u.w;
        }
#pragma unroll
        for (int e = 0; e < 16; e++) {
          v[2 * e] += __uint_as_float(w[e] << 16);
          v[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (n0 + j < N) v[j] += bf2f(rp[j]);
      }
    } else {
      const float* rp = reinterpret_cast<const float*>(ep.res) + rr * ep.ldr + n0;
      if (full) {
        uint32_t w[32];
        ld_words32(rp, w, ep.wide != 0);
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] += __uint_as_float(w[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (n0 + j < N) v[j] += rp[j];
      }
    }
  }
  if (ep.out_f32) {
    if (ep.stats_out) {  // N % 32 == 0, so the chunk is full; 4 independent partial sums per pass
      float sm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 32; j++) sm[j & 3] += v[j];
      const float mean = ((sm[0] + sm[1]) + (sm[2] + sm[3])) * (1.f / 32.f);
      float q[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 32; j++) q[j & 3] = fmaf(v[j] - mean, v[j] - mean, q[j & 3]);
      ep.stats_out[(long long)m * (N / 32) + n0 / 32] = make_float2(mean, (q[0] + q[1]) + (q[2] + q[3]));
    }
    float* op = reinterpret_cast<float*>(ep.out) + (long long)m * ep.ldo + n0;
    if (full) {
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 32; j++) w[j] = __float_as_uint(v[j]);
      st_words<32>(op, w, ep.wide != 0);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n0 + j < N) op[j] = v[j];
    }
    if (ep.out2) {
      uint16_t* o2 = ep.out2 + (long long)m * ep.ldo2 + n0;
      if (full) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; j++) w[j] = pack_bf2(v[2 * j], v[2 * j + 1]);
        st_words<16>(o2, w, ep.wide != 0);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (n0 + j < N) o2[j] = f2bf(v[j]);
      }
    }
  } else if (ep.pk_T > 0) {
    const int HD = ep.pk_H * ep.pk_D;
    const long long crop = m / ep.pk_T;
    const int t = m % ep.pk_T;
    const size_t tile_elems = (size_t)ep.pk_NC * 1024;
    uint16_t* base = reinterpret_cast<uint16_t*>(ep.out);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + 8 * j;
      if (n < N) {
        const int w = n / HD, rem = n % HD, hh = rem / ep.pk_D, d = rem % ep.pk_D;
        const size_t off = (((size_t)crop * 3 + w) * ep.pk_H + hh) * ep.pk_Tt * tile_elems +
                           attn_tile_off(w, t, d / 8, ep.pk_NC);
        *reinterpret_cast<uint4*>(base + off) =
            make_uint4(pack_bf2(v[8 * j], v[8 * j + 1]), pack_bf2(v[8 * j + 2], v[8 * j + 3]),
                       pack_bf2(v[8 * j + 4], v[8 * j + 5]), pack_bf2(v[8 * j + 6], v[8 * j + 7]));
      }
    }
  } else {
    if (ep.gelu == 1) {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = gelu_tanh(bfround(v[j]));
    } else if (ep.gelu == 2) {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = gelu_sigmoid(v[j]);
    }
    uint16_t* op = reinterpret_cast<uint16_t*>(ep.out) + (long long)m * ep.ldo + n0;
    if (full) {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; j++) w[j] = pack_bf2(v[2 * j], v[2 * j + 1]);
      st_words<16>(op, w, ep.wide != 0);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (n0 + j < N) op[j] = f2bf(v[j]);
    }
  }
}

// The residual words of one full 32-column chunk of row m (fp32: 32 words; bf16: the first 16), loaded
// ahead of the chunk's epilogue so that the loads overlap other work.  Nothing is loaded without a
// residual, for rows past M or for a chunk that crosses N (the scalar path loads its own).
__device__ __forceinline__ void res_load(uint32_t (&w)[32], int m, int n0, int M, int N, const Epi& ep) {
  if (!ep.res || m >= M || n0 + 32 > N) return;
  const long long rr = ep.res_period > 0 ? (long long)(m % ep.res_period) : (long long)m;
  if (ep.res_bf16) {
    const uint16_t* rp = reinterpret_cast<const uint16_t*>(ep.res) + rr * ep.ldr + n0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint4 u = *reinterpret_cast<const uint4*>(rp + 8 * j);
      w[4 * j] = u.x; w[4 * j + 1] = u.y; w[4 * j + 2] = u.z; w[4 * j + 3] = u.w;
    }
  } else {
    ld_words32(reinterpret_cast<const float*>(ep.res) + rr * ep.ldr + n0, w, ep.wide != 0);
  }
}

// Applies the epilogue to one 32-column chunk of row m (columns n0 .. n0+31) held in r.  PRE: the chunk's
// residual words are already in rw (res_load, issued earlier); otherwise they are loaded here, where they
// are added.  Full chunks (every column < N) do their arithmetic two columns at a time with the packed
// fp32x2 instructions.
template <bool PRE>
__device__ __forceinline__ void epilogue_chunk_rw(const uint32_t (&r)[32], const uint32_t (&rw_in)[32], int m, int M,
                                                  int n0, int N, const Epi& ep, float mu, float rstd) {
  if (n0 + 32 > N) {
    epilogue_chunk_partial(r, m, n0, N, ep, mu, rstd);
    return;
  }
  unsigned long long v[16];
#pragma unroll
  for (int j = 0; j < 16; j++) v[j] = f2_pack(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
  if (ep.i8_sw) {  // int8 path: the column scale (the row scale is already in)
    const float4* s4 = reinterpret_cast<const float4*>(ep.i8_sw + n0);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float4 sw = __ldg(s4 + j);
      v[2 * j] = f2_mul(v[2 * j], f2_pack(sw.x, sw.y));
      v[2 * j + 1] = f2_mul(v[2 * j + 1], f2_pack(sw.z, sw.w));
    }
  }
  if (ln_folded(ep)) {  // rstd * (acc - mean * c) + bias = rstd * acc + (bias - rstd * mean * c)
    const unsigned long long rs = f2_pack(rstd, rstd), nrm = f2_pack(-rstd * mu, -rstd * mu);
    const float4* c4 = reinterpret_cast<const float4*>(ep.ln_c + n0);
    const float4* b4 = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float4 c = __ldg(c4 + j);
      const float4 b = ep.bias ? __ldg(b4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[2 * j] = f2_fma(rs, v[2 * j], f2_fma(nrm, f2_pack(c.x, c.y), f2_pack(b.x, b.y)));
      v[2 * j + 1] = f2_fma(rs, v[2 * j + 1], f2_fma(nrm, f2_pack(c.z, c.w), f2_pack(b.z, b.w)));
    }
  } else if (ep.bias) {
    const float4* b4 = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float4 b = __ldg(b4 + j);
      v[2 * j] = f2_add(v[2 * j], f2_pack(b.x, b.y));
      v[2 * j + 1] = f2_add(v[2 * j + 1], f2_pack(b.z, b.w));
    }
  }
  if (ep.res) {
    uint32_t rw_local[32];
    if constexpr (!PRE) res_load(rw_local, m, n0, M, N, ep);
    const uint32_t* rw = PRE ? rw_in : rw_local;
    if (ep.res_bf16) {
#pragma unroll
      for (int e = 0; e < 16; e++)
        v[e] = f2_add(v[e], f2_pack(__uint_as_float(rw[e] << 16), __uint_as_float(rw[e] & 0xffff0000u)));
    } else {
#pragma unroll
      for (int j = 0; j < 16; j++) v[j] = f2_add(v[j], f2_pack(__uint_as_float(rw[2 * j]), __uint_as_float(rw[2 * j + 1])));
    }
  }
  uint32_t w[32];
  if (ep.out_f32) {
    if (ep.stats_out) {  // N % 32 == 0; four independent fp32x2 partial sums per pass
      unsigned long long a[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int j = 0; j < 16; j++) a[j & 3] = f2_add(a[j & 3], v[j]);
      float s0, s1;
      f2_unpack(f2_add(f2_add(a[0], a[1]), f2_add(a[2], a[3])), s0, s1);
      const float mean = (s0 + s1) * (1.f / 32.f);
      const unsigned long long nm = f2_pack(-mean, -mean);
#pragma unroll
      for (int j = 0; j < 4; j++) a[j] = 0ull;
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const unsigned long long d = f2_add(v[j], nm);
        a[j & 3] = f2_fma(d, d, a[j & 3]);
      }
      f2_unpack(f2_add(f2_add(a[0], a[1]), f2_add(a[2], a[3])), s0, s1);
      ep.stats_out[(long long)m * (N / 32) + n0 / 32] = make_float2(mean, s0 + s1);
    }
#pragma unroll
    for (int j = 0; j < 16; j++) {
      float x0, x1;
      f2_unpack(v[j], x0, x1);
      w[2 * j] = __float_as_uint(x0);
      w[2 * j + 1] = __float_as_uint(x1);
    }
    st_words<32>(reinterpret_cast<float*>(ep.out) + (long long)m * ep.ldo + n0, w, ep.wide != 0);
    if (ep.out2) {
#pragma unroll
      for (int j = 0; j < 16; j++) w[j] = pack_bf2(__uint_as_float(w[2 * j]), __uint_as_float(w[2 * j + 1]));
      st_words<16>(ep.out2 + (long long)m * ep.ldo2 + n0, w, ep.wide != 0);
    }
    return;
  }
  // bf16 outputs: round to bf16 first (GELU is applied to the bf16 linear output), except for the int8
  // epilogue's GELU on the fp32 value
  if (ep.gelu == 2) {
#pragma unroll
    for (int j = 0; j < 16; j++) {
      float g0, g1;
      f2_unpack(v[j], g0, g1);
      v[j] = f2_pack(gelu_sigmoid(g0), gelu_sigmoid(g1));
    }
  }
#pragma unroll
  for (int j = 0; j < 16; j++) {
    float x0, x1;
    f2_unpack(v[j], x0, x1);
    w[j] = pack_bf2(x0, x1);
  }
  if (ep.gelu == 1) {
#pragma unroll
    for (int j = 0; j < 16; j++) {
      float g0, g1;
      f2_unpack(gelu_tanh2(f2_pack(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xffff0000u))), g0, g1);
      w[j] = pack_bf2(g0, g1);
    }
  }
  if (ep.gelu == 3) {
    // gated: the chunk holds gate columns 16c .. 16c+15 (words 0-7) and the matching up columns (words 8-15) of a
    // weight whose gate / up rows are interleaved in blocks of 16; out column 16c + i = bf16(bf16(gelu_tanh(gate))
    // * up), 16 bf16 outputs at n0 / 2
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float g0, g1;
      f2_unpack(gelu_tanh2(f2_pack(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xffff0000u))), g0, g1);
      o[j] = pack_bf2(__fmul_rn(bfround(g0), __uint_as_float(w[8 + j] << 16)),
                      __fmul_rn(bfround(g1), __uint_as_float(w[8 + j] & 0xffff0000u)));
    }
    st_words<8>(reinterpret_cast<uint16_t*>(ep.out) + (long long)m * ep.ldo + n0 / 2, o, ep.wide != 0);
    return;
  }
  if (ep.pk_T > 0) {
    // attention tiles: the chunk's four 8-column groups each lie in one head (D % 8 == 0); the head and
    // d offset advance incrementally from the chunk's first column instead of being divided out per group
    const int HD = ep.pk_H * ep.pk_D;
    const int crop = m / ep.pk_T, t = m - crop * ep.pk_T;
    int wsel = n0 / HD;
    const int rem = n0 - wsel * HD;
    int hh = rem / ep.pk_D, d = rem - hh * ep.pk_D;
    const size_t tile_elems = (size_t)ep.pk_NC * 1024;
    uint16_t* base = reinterpret_cast<uint16_t*>(ep.out);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const size_t off = (((size_t)crop * 3 + wsel) * ep.pk_H + hh) * (size_t)ep.pk_Tt * tile_elems +
                         attn_tile_off(wsel, t, d >> 3, ep.pk_NC);
      *reinterpret_cast<uint4*>(base + off) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      d += 8;
      if (d >= ep.pk_D) {
        d = 0;
        if (++hh == ep.pk_H) { hh = 0; ++wsel; }
      }
    }
    return;
  }
  st_words<16>(reinterpret_cast<uint16_t*>(ep.out) + (long long)m * ep.ldo + n0, w, ep.wide != 0);
}

// int8 path: the s32 accumulator words of a chunk become fp32 (float)acc * sa, sa the row's activation scale.
__device__ __forceinline__ void i8_row_scale(uint32_t (&r)[32], float sa) {
#pragma unroll
  for (int j = 0; j < 32; j++) r[j] = __float_as_uint(__fmul_rn(__int2float_rn((int)r[j]), sa));
}

// The same with the residual loaded where it is added.
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], int m, int M, int n0, int N, const Epi& ep,
                                               float mu, float rstd) {
  epilogue_chunk_rw<false>(r, r, m, M, n0, N, ep, mu, rstd);
}

// I8: signed int8 operands (kind::i8, 128-element k-blocks: the same 128-byte swizzled rows), s32
// accumulators converted in the epilogue (Epi::i8_sa / i8_sw).
template <int BN, bool I8>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                        int K, Epi ep) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES, STAGE_BYTES = C::STAGE_BYTES, A_BYTES = C::A_BYTES;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nN = (N + BN - 1) / BN;
  const int ntiles = ((M + BM - 1) / BM) * nN;
  constexpr int BKE = I8 ? 2 * BK : BK;  // k-block width in elements (128 bytes)
  const int nk = (K + BKE - 1) / BKE;
  // work unit u = (tile u / ks_n, K slice u % ks_n); slice s covers k-blocks [nk*s/ks_n, nk*(s+1)/ks_n)
  const int ks_n = ep.ksplit > 1 ? ep.ksplit : 1;
  const int nunits = ntiles * ks_n;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // programmatic dependent launch: the operands' producer has completed
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
        const int t = u / ks_n, ks = u % ks_n;
        const int mt = t / nN, nt = t % nN;
        const int kb1 = (int)((long long)nk * (ks + 1) / ks_n);
        for (int kb = (int)((long long)nk * ks / ks_n); kb < kb1; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, ST_GEMM_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = smem + stage * STAGE_BYTES;
          tma_load_2d(&tmA, &full[stage], sa, kb * BKE, mt * BM);
          tma_load_2d(&tmB, &full[stage], sa + A_BYTES, kb * BKE, nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // unwinding: let the loads this thread issued land before the CTA exits
        uint32_t s = stage, p = phase;
        for (int j = 0; j < STAGES && j < issued; j++) {
          if (s == 0) {
            s = STAGES - 1;
            p ^= 1;
          } else {
            s--;
          }
          mbar_wait_drain(&full[s], p, kDrainCycles);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC = I8 ? idesc_i8(BM, BN) : idesc_bf16(BM, BN);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
        const int ks = u % ks_n;
        const int kb0 = (int)((long long)nk * ks / ks_n), kb1 = (int)((long long)nk * (ks + 1) / ks_n);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, ST_GEMM_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; kb++) {
          if (!mbar_wait(&full[stage], phase, abort_flag, ST_GEMM_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t ad = sdesc_k_sw128(sa), bd = sdesc_k_sw128(sa + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {  // 32 bytes of K per instruction (16 bf16 / 32 int8)
            if constexpr (I8)
              umma_i8(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_f16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      // no MMA may still be writing TMEM when it is freed
      umma_commit(drain);
      mbar_wait_drain(drain, 0, kDrainCycles);
    }
  } else {
    // ---------------- epilogue: warps 2..9; warp w reads TMEM lanes 32*(w%4) .. +31 (the hardware's
    // lane-quarter rule) and the chunks [half * BN/64, (half + 1) * BN/64) of the tile's columns
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int CH = BN / 64;  // 32-column chunks per warp
    const int row = q * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
      const int t = u / ks_n;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int mt = t / nN, nt = t % nN;
      const int m = mt * BM + row;
      float mu = 0.f, rstd = 1.f, sa = 1.f;
      ln_row_factors(ep, m, M, nt == 0 && half == 0, mu, rstd);  // before the wait: overlaps the tile's MMAs
      if (I8 && m < M) sa = ep.i8_sa[m];
      // 64-wide tiles without split K (one 32-column chunk per warp and tile; the small-M GEMMs, often one tile
      // per CTA): the chunk's residual is loaded before the accumulator wait, so its latency overlaps the MMAs
      // instead of following them
      const bool pre = CH == 1 && ks_n == 1;
      uint32_t rw[32];
      if (pre) res_load(rw, m, nt * BN + half * 32, M, N, ep);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ST_GEMM_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = half * CH; c < (half + 1) * CH; c++) {
        const int n0 = nt * BN + c * 32;
        if (n0 >= N) break;  // uniform across the CTA
        uint32_t r[32];
        tmem_ld32(tb + (uint32_t)(c * 32), r);
        tmem_ld_wait();
        if (m >= M) continue;
        if (ks_n > 1) {  // split-K: store this slice's partial; the slice that completes the row chunk sums them
          const size_t plane = (size_t)M * ep.sk_pitch;
          float* w = ep.sk_ws + (size_t)m * ep.sk_pitch + n0;
          const int ks = u % ks_n;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            __stcg(reinterpret_cast<float4*>(w + ks * plane + e),
                   make_float4(__uint_as_float(r[e]), __uint_as_float(r[e + 1]), __uint_as_float(r[e + 2]),
                               __uint_as_float(r[e + 3])));
          __threadfence();
          int* cnt = ep.sk_cnt + (size_t)m * (ep.sk_pitch / 32) + n0 / 32;
          if (atomicAdd(cnt, 1) != ks_n - 1) continue;
          __threadfence();
          if constexpr (I8) {  // int32 partials: the sum is exact in any order
            int acc[32];
#pragma unroll
            for (int e = 0; e < 32; e++) acc[e] = 0;
            for (int sl = 0; sl < ks_n; sl++) {
#pragma unroll
              for (int e = 0; e < 32; e += 4) {
                const int4 v = __ldcg(reinterpret_cast<const int4*>(w + sl * plane + e));
                acc[e] += v.x;
                acc[e + 1] += v.y;
                acc[e + 2] += v.z;
                acc[e + 3] += v.w;
              }
            }
#pragma unroll
            for (int e = 0; e < 32; e++) r[e] = (uint32_t)acc[e];
          } else {
            float acc[32];
#pragma unroll
            for (int e = 0; e < 32; e++) acc[e] = 0.f;
            for (int sl = 0; sl < ks_n; sl++) {
#pragma unroll
              for (int e = 0; e < 32; e += 4) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(w + sl * plane + e));
                acc[e] += v.x;
                acc[e + 1] += v.y;
                acc[e + 2] += v.z;
                acc[e + 3] += v.w;
              }
            }
#pragma unroll
            for (int e = 0; e < 32; e++) r[e] = __float_as_uint(acc[e]);
          }
          *cnt = 0;
        }
        if constexpr (I8) i8_row_scale(r, sa);
        if (pre) epilogue_chunk_rw<true>(r, rw, m, M, n0, N, ep, mu, rstd);
        else epilogue_chunk(r, m, M, n0, N, ep, mu, rstd);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a cluster of 2 CTAs computes 256 x 256 output tiles.  Each CTA stages
// its 128 rows of A and its 128 rows of B (B rows = output columns n0 + rank*128 ..) per 64-wide k-block;
// the leader (rank 0) issues tcgen05.mma.cta_group::2 (M 256, N 256), which reads A and B from both CTAs'
// shared memory and writes each CTA's 128 output rows into that CTA's TMEM.  Per SM the L2 -> shared
// traffic is 32 KB per k-block instead of 48 KB for the single-CTA 128 x 256 tile.
//   * TMA loads of both CTAs complete on the leader's full[s] (armed by the leader for both CTAs' bytes);
//   * the leader's commits arrive on empty[s] / tfull[a] of each CTA (two commits, one per CTA);
//   * the epilogue warps of both CTAs arrive on the leader's tempty[a] (one arrive per warp).
// Epilogue modes of the pair kernel (one instantiation each, so that each keeps its own register budget):
//   0  no residual: the accumulator chunk goes straight through epilogue_chunk;
//   1  residual in registers: the residual of the next 32-column chunk is loaded while this one is done;
//   2  staged fp32 residual epilogue (out = acc + bias + res in fp32, optional bf16 copy and row
//      statistics; the proj GEMM): each epilogue warp TMA-loads its 32 x 32 residual box into shared
//      memory one chunk ahead, adds in place and TMA-stores the fp32 box (and a bf16 box), so every
//      global access is a whole-line bulk copy instead of one 32-byte sector in each of 32 rows.  It
//      trades two of the six mainloop stages for the 96 KB of staging buffers.
// PBN: the pair tile's width, 256 (each CTA stages 128 rows of B) or 128 (64 rows; for GEMMs whose 256-wide
// tiles would leave most SM pairs idle, e.g. the text prefill's 730 x 2048 proj / fc2 with 24 tiles).
template <int MODE, int PBN = 256>
struct PairCfg {
  static constexpr int B_ROWS = PBN / 2;
  static constexpr int STAGES = PBN == 256 ? (MODE == 2 ? 4 : 6) : (MODE == 2 ? 5 : 8);
  static constexpr int STAGE_BYTES = (128 + B_ROWS) * BK * 2;  // this CTA's 128 rows of A and B_ROWS of B
  static constexpr int EPI_WARP_BYTES = MODE == 2 ? 2 * 4096 + 2 * 2048 : 0;  // 2 fp32 + 2 bf16 32x32 boxes
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + EPI_WARPS * EPI_WARP_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 1024 + 512;
};
constexpr int P_A_BYTES = 128 * BK * 2;

template <int MODE, bool I8, int PBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_bf16_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO,
                             const __grid_constant__ CUtensorMap tmO2, int M, int N, int K, Epi ep) {
  using C = PairCfg<MODE, PBN>;
  constexpr int P_STAGES = C::STAGES, P_STAGE_BYTES = C::STAGE_BYTES;
  constexpr int BN = PBN;
  constexpr uint32_t TMEM_COLS = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* rbar = drain + 1;  // [EPI_WARPS][2] residual-box barriers (mode 2)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int nN = (N + BN - 1) / BN;
  const int ntiles = ((M + 255) / 256) * nN;
  constexpr int BKE = I8 ? 2 * BK : BK;  // k-block width in elements (128 bytes)
  const int nk = (K + BKE - 1) / BKE;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (MODE == 2) {
      tma_prefetch_desc(&tmR);
      tma_prefetch_desc(&tmO);
      if (ep.out2) tma_prefetch_desc(&tmO2);
    }
    for (int s = 0; s < P_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);  // one arrive per epilogue warp of each CTA
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * EPI_WARPS; i++) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();  // programmatic dependent launch: the operands' producer has completed
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs): this CTA's 128 rows of A and of B per stage
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters) {
        const int mt = t / nN, nt = t % nN;
        // (256-wide tiles) a column tile with at most 128 valid columns runs as N = 128: each CTA then holds
        // 64 B rows; 128-wide tiles always hold 64
        const int bhalf = (PBN == 128 || N - nt * BN <= 128) ? 64 : 128;
        for (int kb = 0; kb < nk; kb++) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, ST_GEMM_PRODUCER)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          const uint32_t fb = full_leader0 + stage * 8;
          tma_load_2d_pair(&tmA, fb, sa, kb * BKE, mt * 256 + (int)rank * 128);
          tma_load_2d_pair(&tmB, fb, sa + P_A_BYTES, kb * BKE, nt * BN + (int)rank * bhalf);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // no drain here: loads complete on the leader's barriers, which the leader's MMA thread (or its
      // own unwinding below) observes before the final cluster barrier
      if (!ok) {
        const long long t0 = clock64();
        while (clock64() - t0 < 200000) {
        }  // ~0.1 ms: in-flight tile loads land long before this
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (leader CTA only)
      constexpr uint32_t IDESC = I8 ? idesc_i8(256, BN) : idesc_bf16(256, BN);
      constexpr uint32_t IDESC_HALF = I8 ? idesc_i8(256, BN / 2) : idesc_bf16(256, BN / 2);
      const uint32_t empty0_self = smem_u32(&empty[0]), empty0_peer = mapa_shared(smem_u32(&empty[0]), 1);
      const uint32_t tfull0_self = smem_u32(&tfull[0]), tfull0_peer = mapa_shared(smem_u32(&tfull[0]), 1);
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, ST_GEMM_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        const uint32_t idesc = (PBN == 256 && N - (t % nN) * BN <= 128) ? IDESC_HALF : IDESC;  // see the producer
        for (int kb = 0; kb < nk; kb++) {
          if (!mbar_wait(&full[stage], phase, abort_flag, ST_GEMM_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint64_t ad = sdesc_k_sw128(sa), bd = sdesc_k_sw128(sa + P_A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {  // 32 bytes of K per instruction (16 bf16 / 32 int8)
            if constexpr (I8)
              umma_i8_pair(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16_pair(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty0_self + stage * 8);
          umma_commit_pair(empty0_peer + stage * 8);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          umma_commit_pair(tfull0_self + acc * 8);
          umma_commit_pair(tfull0_peer + acc * 8);
        }
      }
      umma_commit_pair(smem_u32(drain));
      mbar_wait_drain(drain, 0, kDrainCycles);
      if (!ok) {  // let every armed stage's loads (both CTAs') land before the pair exits
        for (int j = 0; j < P_STAGES; j++) mbar_wait_drain(&full[j], 0, 20000000LL);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of each 256 x 256 tile; warp w reads TMEM
    // lanes 32*(w%4) .. +31 and the columns [half * 128, half * 128 + 128) of the tile
    const int q = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;
    constexpr int CH = BN / 64;
    const int row = q * 32 + lane;
    const uint32_t tempty0_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    // mode 2: this warp's staging buffers and residual barriers, the chunk counter g (buffer g & 1, use
    // g >> 1 of it) and which buffers have a load in flight
    uint8_t* stg = smem + C::EPI_OFF + ew * C::EPI_WARP_BYTES;
    uint64_t* rb = rbar + 2 * ew;
    uint32_t g = 0;
    bool pend[2] = {false, false};
    bool ok = true;
    int it = 0;
    for (int t = cluster; t < ntiles; t += nclusters, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int mt = t / nN, nt = t % nN;
      const int m = mt * 256 + (int)rank * 128 + row;
      float mu = 0.f, rstd = 1.f, sa = 1.f;
      ln_row_factors(ep, m, M, nt == 0 && half == 0, mu, rstd);
      if (I8 && m < M) sa = ep.i8_sa[m];
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + half * CH * 32);
      const int nbase = nt * BN + half * CH * 32;
      if constexpr (MODE == 2) {
        const int mw = mt * 256 + (int)rank * 128 + q * 32;  // the warp's first row
        const bool rows_in = mw < M;                          // uniform across the warp
        auto issue_load = [&](int n0, uint32_t gg) {          // lane 0: residual box of chunk gg
          const int b = gg & 1;
          bulk_wait_read<0>();  // the store that last read buffer b has finished reading it
          mbar_arrive_expect_tx(&rb[b], 4096);
          tma_load_2d(&tmR, &rb[b], stg + b * 4096, n0, mw);
          pend[b] = true;
        };
        if (rows_in && nbase < N && lane == 0) issue_load(nbase, g);
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ST_GEMM_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (rows_in) {
#pragma unroll 1
          for (int i = 0; i < CH; i++) {
            const int n0 = nbase + i * 32;
            if (n0 >= N) break;  // uniform across the warp
            const int b = g & 1;
            if (i + 1 < CH && n0 + 32 < N && lane == 0) issue_load(n0 + 32, g + 1);
            uint32_t r[32];
            tmem_ld32(tb + (uint32_t)(i * 32), r);
            tmem_ld_wait();
            if (!mbar_wait(&rb[b], (g >> 1) & 1, abort_flag, ST_GEMM_EPILOGUE)) {
              ok = false;
              break;
            }
            if (lane == 0) pend[b] = false;
            // row `lane` of the 32 x 32 fp32 box: 16-byte chunk c lives at chunk c ^ (lane & 7) (128-byte
            // swizzle); the bf16 box's row is 64 bytes with chunk c at c ^ ((lane >> 1) & 3) (64-byte swizzle)
            uint8_t* fr = stg + b * 4096 + lane * 128;
            uint8_t* br = stg + 8192 + b * 2048 + lane * 64;
            unsigned long long v[16];
            if constexpr (I8) {  // ((acc * sa) * sw + bias) + res, the int8 epilogue's order
              i8_row_scale(r, sa);
              const float4* s4 = reinterpret_cast<const float4*>(ep.i8_sw + n0);
#pragma unroll
              for (int c = 0; c < 8; c++) {
                const float4 sw = __ldg(s4 + c);
                const float4 bb = ep.bias ? __ldg(reinterpret_cast<const float4*>(ep.bias + n0) + c)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 x = *reinterpret_cast<const float4*>(fr + ((c ^ (lane & 7)) << 4));
                unsigned long long a0 = f2_mul(f2_pack(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1])),
                                               f2_pack(sw.x, sw.y));
                unsigned long long a1 = f2_mul(f2_pack(__uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3])),
                                               f2_pack(sw.z, sw.w));
                if (ep.bias) {
                  a0 = f2_add(a0, f2_pack(bb.x, bb.y));
                  a1 = f2_add(a1, f2_pack(bb.z, bb.w));
                }
                v[2 * c] = f2_add(a0, f2_pack(x.x, x.y));
                v[2 * c + 1] = f2_add(a1, f2_pack(x.z, x.w));
              }
            } else {
#pragma unroll
              for (int c = 0; c < 8; c++) {
                const float4 x = *reinterpret_cast<const float4*>(fr + ((c ^ (lane & 7)) << 4));
                v[2 * c] =
                    f2_add(f2_pack(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1])), f2_pack(x.x, x.y));
                v[2 * c + 1] =
                    f2_add(f2_pack(__uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3])), f2_pack(x.z, x.w));
              }
              if (ep.bias) {
                const float4* b4 = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                  const float4 bb = __ldg(b4 + j);
                  v[2 * j] = f2_add(v[2 * j], f2_pack(bb.x, bb.y));
                  v[2 * j + 1] = f2_add(v[2 * j + 1], f2_pack(bb.z, bb.w));
                }
              }
            }
            if (ep.stats_out && m < M) {  // four independent fp32x2 partial sums per pass
              unsigned long long a4[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
              for (int j = 0; j < 16; j++) a4[j & 3] = f2_add(a4[j & 3], v[j]);
              float s0, s1;
              f2_unpack(f2_add(f2_add(a4[0], a4[1]), f2_add(a4[2], a4[3])), s0, s1);
              const float mean = (s0 + s1) * (1.f / 32.f);
              const unsigned long long nm = f2_pack(-mean, -mean);
#pragma unroll
              for (int j = 0; j < 4; j++) a4[j] = 0ull;
#pragma unroll
              for (int j = 0; j < 16; j++) {
                const unsigned long long dd = f2_add(v[j], nm);
                a4[j & 3] = f2_fma(dd, dd, a4[j & 3]);
              }
              f2_unpack(f2_add(f2_add(a4[0], a4[1]), f2_add(a4[2], a4[3])), s0, s1);
              ep.stats_out[(long long)m * (N / 32) + n0 / 32] = make_float2(mean, s0 + s1);
            }
#pragma unroll
            for (int c = 0; c < 8; c++) {
              float x0, x1, x2, x3;
              f2_unpack(v[2 * c], x0, x1);
              f2_unpack(v[2 * c + 1], x2, x3);
              *reinterpret_cast<float4*>(fr + ((c ^ (lane & 7)) << 4)) = make_float4(x0, x1, x2, x3);
              if (ep.out2 && (c & 1)) {  // two fp32 chunks = one 16-byte bf16 chunk
                float y0, y1, y2, y3;
                f2_unpack(v[2 * c - 2], y0, y1);
                f2_unpack(v[2 * c - 1], y2, y3);
                const int bc = c >> 1;
                *reinterpret_cast<uint4*>(br + ((bc ^ ((lane >> 1) & 3)) << 4)) =
                    make_uint4(pack_bf2(y0, y1), pack_bf2(y2, y3), pack_bf2(x0, x1), pack_bf2(x2, x3));
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmO, stg + b * 4096, n0, mw);
              if (ep.out2) tma_store_2d(&tmO2, stg + 8192 + b * 2048, n0, mw);
              bulk_commit();
            }
            ++g;
          }
          if (!ok) break;
        }
      } else if constexpr (MODE == 1) {
        // the residual of chunk i+1 is loaded while chunk i is processed, the first chunk's before the
        // accumulator wait (the residual does not depend on the MMAs)
        uint32_t rw[2][32];
        res_load(rw[0], m, nbase, M, N, ep);
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ST_GEMM_EPILOGUE)) break;
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < CH; i++) {
          const int n0 = nbase + i * 32;
          if (n0 >= N) break;  // uniform across the warp
          if (i + 1 < CH) res_load(rw[(i + 1) & 1], m, n0 + 32, M, N, ep);
          uint32_t r[32];
          tmem_ld32(tb + (uint32_t)(i * 32), r);
          tmem_ld_wait();
          if constexpr (I8) i8_row_scale(r, sa);
          if (m < M) epilogue_chunk_rw<true>(r, rw[i & 1], m, M, n0, N, ep, mu, rstd);
        }
      } else {
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, ST_GEMM_EPILOGUE)) break;
        tc_fence_after();
#pragma unroll 1
        for (int i = 0; i < CH; i++) {
          const int n0 = nbase + i * 32;
          if (n0 >= N) break;
          uint32_t r[32];
          tmem_ld32(tb + (uint32_t)(i * 32), r);
          tmem_ld_wait();
          if constexpr (I8) i8_row_scale(r, sa);
          if (m < M) epilogue_chunk(r, m, M, n0, N, ep, mu, rstd);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0_leader + acc * 8);
    }
    if constexpr (MODE == 2) {
      if (lane == 0) {
        // unwinding: residual loads still in flight land before the CTA exits; every store completes
        for (int b = 0; b < 2; b++)
          if (pend[b]) mbar_wait_drain(&rb[b], ((g + (uint32_t)((b - (int)(g & 1)) & 1)) >> 1) & 1, kDrainCycles);
        bulk_wait_all<0>();
      }
      __syncwarp();
    }
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into the peer's TMEM / smem are complete before either CTA exits
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// The staged epilogue (mode 2) applies to fp32 out = acc (+ bias) + fp32 residual (+ bf16 copy, + row
// statistics) with N % 32 == 0 and 16-byte pitches, when K <= 2048: there a tile's mainloop is shorter
// than its register epilogue (proj, K 1152: 0.49 -> 0.33 ms per 130-crop launch), while a long mainloop
// (fc2, K 4304) already hides that epilogue and would only lose the two mainloop stages.
// VT_GEMM_TMA_EPI=0 turns it off.
static bool pair_mode2_ok(const Epi& ep, int N, int K) {
  static const int enabled = [] {
    const char* e = getenv("VT_GEMM_TMA_EPI");
    return e ? atoi(e) : 1;
  }();
  return enabled && K <= 2048 && ep.res && !ep.res_bf16 && ep.res_period == 0 && ep.out_f32 && !ep.gelu &&
         ep.pk_T == 0 && !ln_folded(ep) && N % 32 == 0 && ep.ldr % 4 == 0 && ep.ldo % 4 == 0 &&
         (!ep.out2 || ep.ldo2 % 8 == 0);
}


// K-major operand tensor maps: bf16 with 64-element boxes, or int8 with 128-element ones (128 bytes either way).
static int make_tmap_op(CUtensorMap* m, const void* p, int K, int rows, long long ld, int box_rows, bool i8) {
  return i8 ? make_tmap_i8(m, p, (uint64_t)K, (uint64_t)rows, (uint64_t)ld, 2 * BK, box_rows)
            : make_tmap_bf16(m, p, (uint64_t)K, (uint64_t)rows, (uint64_t)ld, BK, box_rows);
}

template <int MODE, bool I8, int PBN>
static void launch_pair_mode(cudaStream_t st, int clusters, const CUtensorMap& ta, const CUtensorMap& tb,
                             const CUtensorMap& tr, const CUtensorMap& to, const CUtensorMap& to2, int M, int N, int K,
                             const Epi& ep) {
  // a failure here leaves the kernel's default shared-memory limit, so the launch below fails and check_launch
  // reports it
  smem_attr_once((const void*)gemm_bf16_tc_pair_kernel<MODE, I8, PBN>, PairCfg<MODE, PBN>::SMEM_BYTES, "vt_gemm");
  launch_k(gemm_bf16_tc_pair_kernel<MODE, I8, PBN>, 2 * clusters, THREADS, PairCfg<MODE, PBN>::SMEM_BYTES, st, ta, tb,
           tr, to, to2, M, N, K, ep);
}

template <bool I8, int PBN>
static void launch_pair_width(cudaStream_t st, int mode, int clusters, const CUtensorMap& ta, const CUtensorMap& tb,
                              const CUtensorMap& tr, const CUtensorMap& to, const CUtensorMap& to2, int M, int N, int K,
                              const Epi& ep) {
  if (mode == 2) launch_pair_mode<2, I8, PBN>(st, clusters, ta, tb, tr, to, to2, M, N, K, ep);
  else if (mode == 1) launch_pair_mode<1, I8, PBN>(st, clusters, ta, tb, tr, to, to2, M, N, K, ep);
  else launch_pair_mode<0, I8, PBN>(st, clusters, ta, tb, tr, to, to2, M, N, K, ep);
}

static int launch_pair(cudaStream_t st, const void* A, long long lda, const void* W, long long ldw, int M, int N,
                       int K, const Epi& ep, bool i8, int pbn) {
  CUtensorMap ta, tb, tr, to, to2;
  memset(&tr, 0, sizeof(tr));
  memset(&to, 0, sizeof(to));
  memset(&to2, 0, sizeof(to2));
  int rc = make_tmap_op(&ta, A, K, M, lda, 128, i8);
  if (rc) return rc;
  rc = make_tmap_op(&tb, W, K, N, ldw, pbn / 2, i8);
  if (rc) return rc;
  const int mode = !ep.res ? 0 : pair_mode2_ok(ep, N, K) ? 2 : 1;
  if (mode == 2) {
    rc = make_tmap_epi(&tr, ep.res, 4, (uint64_t)N, (uint64_t)M, (uint64_t)ep.ldr, 32, 32, 128);
    if (!rc) rc = make_tmap_epi(&to, ep.out, 4, (uint64_t)N, (uint64_t)M, (uint64_t)ep.ldo, 32, 32, 128);
    if (!rc && ep.out2) rc = make_tmap_epi(&to2, ep.out2, 2, (uint64_t)N, (uint64_t)M, (uint64_t)ep.ldo2, 32, 32, 64);
    if (rc) return rc;
  }
  const long long ntiles = (long long)((M + 255) / 256) * ((N + pbn - 1) / pbn);
  if (ntiles > 0x7fffffffLL) return set_error(E_SHAPE, "vt_gemm: too many tiles");
  const int max_clusters = sm_count() / 2;
  const int clusters = (int)(ntiles < max_clusters ? ntiles : max_clusters);
  if (i8) {
    if (pbn == 128) launch_pair_width<true, 128>(st, mode, clusters, ta, tb, tr, to, to2, M, N, K, ep);
    else launch_pair_width<true, 256>(st, mode, clusters, ta, tb, tr, to, to2, M, N, K, ep);
  } else {
    if (pbn == 128) launch_pair_width<false, 128>(st, mode, clusters, ta, tb, tr, to, to2, M, N, K, ep);
    else launch_pair_width<false, 256>(st, mode, clusters, ta, tb, tr, to, to2, M, N, K, ep);
  }
  return check_launch("vt_gemm (CTA pair)");
}

// Split-K factor for a 128 x 64 tile launch with a workspace: 1 unless the tiles leave two thirds of the
// SMs idle, else the s in 1..16 that minimises the busiest CTA's work, ceil(tiles * s / SMs) work units of
// ceil(nk / s) k-blocks plus a fixed cost of 2 k-blocks each (accumulator hand-off, partial store), plus 2
// k-blocks' worth for the partial-sum pass.  Measured on the text question (M 32): a CTA of this kernel
// streams about one 8 KB weight block per 0.3 us, so the 32-tile proj / fc2 run 13 -> 10 us and
// 39 -> 16 us split 4 ways, while the 96- / 128-tile qkv / fc1 got slower split (the atomic partial sums of
// their wide outputs cost more than the idle third of the SMs).  Without the per-unit cost fc2 chose 9
// (bf16) or 13 (int8) slices, several units per CTA: the whole question took 2.48 / 2.91 ms instead of
// 2.32 / 2.34 ms.  VT_SPLITK_UNIT overrides the per-unit cost (tuning switch).
static int split_k(long long ntiles, int K, int bke) {
  static const int unit = [] {
    const char* e = getenv("VT_SPLITK_UNIT");
    return e ? atoi(e) : 2;
  }();
  const int nk = (K + bke - 1) / bke, sms = sm_count();
  if (ntiles * 3 > sms) return 1;
  int best_s = 1;
  long long best = -1;
  for (int s = 1; s <= kMaxSplit && s <= nk; s++) {
    const long long cost = (ntiles * s + sms - 1) / sms * ((nk + s - 1) / s + unit) + (s > 1 ? 2 : 0);
    if (best < 0 || cost < best) {
      best = cost;
      best_s = s;
    }
  }
  return best_s;
}

template <int BN, bool I8>
static int launch_bn(cudaStream_t st, const void* A, long long lda, const void* W, long long ldw, int M, int N, int K,
                     Epi ep) {
  CUtensorMap ta, tb;
  int rc = make_tmap_op(&ta, A, K, M, lda, BM, I8);
  if (rc) return rc;
  rc = make_tmap_op(&tb, W, K, N, ldw, BN, I8);
  if (rc) return rc;
  rc = smem_attr_once((const void*)gemm_bf16_tc_kernel<BN, I8>, Cfg<BN>::SMEM_BYTES, "vt_gemm");
  if (rc) return rc;
  const long long ntiles = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  ep.ksplit = (BN == 64 && ep.sk_ws) ? split_k(ntiles, K, I8 ? 2 * BK : BK) : 1;  // <= kMaxSplit
  const long long units = ntiles * ep.ksplit;
  if (units > 0x7fffffffLL) return set_error(E_SHAPE, "vt_gemm: too many tiles");
  const int grid = (int)(units < sm_count() ? units : sm_count());
  launch_k(gemm_bf16_tc_kernel<BN, I8>, grid, THREADS, Cfg<BN>::SMEM_BYTES, st, ta, tb, M, N, K, ep);
  return check_launch("vt_gemm");
}

// i8: A and W are int8 (pitches in bytes, multiples of 16) and ep carries the int8 scales.
static int launch(cudaStream_t st, const void* A, long long lda, const void* W, long long ldw, int M, int N, int K,
                  Epi ep, bool i8 = false) {
  if (M < 0 || N < 0 || K < 0) return set_error(E_SHAPE, "vt_gemm: negative shape M=%d N=%d K=%d", M, N, K);
  if (M == 0 || N == 0) return OK;
  if (K == 0) return set_error(E_SHAPE, "vt_gemm: K must be >= 1");
  if (!A || !W || !ep.out) return set_error(E_SHAPE, "vt_gemm: null operand");
  const int pal = i8 ? 16 : 8;  // pitch alignment in elements: 16 bytes
  if (lda < K || ldw < K || lda % pal || ldw % pal || !aligned16(A) || !aligned16(W))
    return set_error(E_SHAPE, "vt_gemm: A/W need 16-byte aligned bases and row pitches (lda=%lld ldw=%lld K=%d)", lda,
                     ldw, K);
  const int n_out = ep.gelu == 3 ? N / 2 : N;  // the gated GELU writes one column per gate / up pair
  if (ep.pk_T <= 0 && (ep.ldo < n_out || ep.ldo % 8 || !aligned16(ep.out)))
    return set_error(E_SHAPE, "vt_gemm: output pitch %lld must be >= %d columns, a multiple of 8, 16-byte aligned",
                     ep.ldo, n_out);
  if (ep.res && (ep.ldr < N || ep.ldr % 8 || !aligned16(ep.res) || ep.res_period < 0))
    return set_error(E_SHAPE, "vt_gemm: residual pitch %lld / period %d invalid", ep.ldr, ep.res_period);
  if (ep.out2 && (ep.ldo2 < N || ep.ldo2 % 8 || !aligned16(ep.out2)))
    return set_error(E_SHAPE, "vt_gemm: bf16 copy pitch %lld invalid", ep.ldo2);
  if (ep.bias && !aligned16(ep.bias)) return set_error(E_SHAPE, "vt_gemm: bias must be 16-byte aligned");
  if (ep.gelu && ep.out_f32) return set_error(E_VARIANT, "vt_gemm: GELU is only fused for bf16 output");
  if (ep.gelu == 3 && (N % 32 || ep.res || ep.pk_T > 0 || ep.stats_out || ep.out2 || ep.i8_sw))
    return set_error(E_VARIANT, "vt_gemm: the gated GELU epilogue needs N %% 32 == 0 and no residual, tiles, "
                                "statistics or second output");
  {
    auto a32 = [](const void* p, long long ld, int es) {
      return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 31) == 0 && (ld * es) % 32 == 0);
    };
    ep.wide = (ep.pk_T > 0 || a32(ep.out, ep.ldo, ep.out_f32 ? 4 : 2)) && a32(ep.res, ep.ldr, ep.res_bf16 ? 2 : 4) &&
             a32(ep.out2, ep.ldo2, 2);
  }
  if (ep.stats_out && (!ep.out_f32 || N % 32 || (reinterpret_cast<uintptr_t>(ep.stats_out) & 7)))
    return set_error(E_VARIANT, "vt_gemm: row statistics need an fp32 output with N %% 32 == 0");
  if (ep.ln_moments && (!ep.ln_c || !aligned16(ep.ln_c) || (reinterpret_cast<uintptr_t>(ep.ln_moments) & 7)))
    return set_error(E_VARIANT, "vt_gemm: folded LayerNorm needs ln_c (16-byte aligned) and 8-byte aligned moments");
  if (ep.ln_stats && (ep.ln_moments || !ep.ln_c || !aligned16(ep.ln_c) || ep.ln_nchunk < 1 ||
                      (reinterpret_cast<uintptr_t>(ep.ln_stats) & 7) || (reinterpret_cast<uintptr_t>(ep.ln_mom_out) & 7)))
    return set_error(E_VARIANT, "vt_gemm: folded norm from chunk statistics needs ln_c (16-byte aligned), nchunk >= 1, "
                                "8-byte aligned statistics / moments and no ln_moments");

  // 256-wide tiles by default: measured on B200 they beat 192-wide ones on every tower shape, even where
  // 192 divides N exactly (N = 1152, 3456).  VT_GEMM_BN=192 selects the 192-wide tile (tuning switch,
  // like the reference's HGEMM_* variables, hgemm.py:56, 85-86).
  static const int forced = [] {
    const char* e = getenv("VT_GEMM_BN");
    return e ? atoi(e) : 0;
  }();
  if (forced == 192 && !i8) return launch_bn<192, false>(st, A, lda, W, ldw, M, N, K, ep);
  // CTA-pair 256 x 256 tiles unless VT_GEMM_2SM=0 (A/B switch) or the problem is a single small tile row
  static const int pair = [] {
    const char* e = getenv("VT_GEMM_2SM");
    return e ? atoi(e) : 1;
  }();
  // Tile shape by how many tiles keep the GPU busy: CTA-pair 256 x 256 tiles when a quarter of the SM pairs
  // get one (measured: the text prefill's 24-tile proj / fc2 still run faster as pairs); 128 x 256 tiles when
  // half of the SMs get one; else 128 x 64 tiles (small-M or narrow GEMMs: the text decoder's 32-token
  // question, the TAPNext 768-wide GEMMs with 15 pair tiles), which spread the weights over 4x more SMs.
  // VT_GEMM_BN=256 keeps the 128 x 256 tile for those.
  const int sms = sm_count();
  const long long tiles_pair = (long long)((M + 255) / 256) * ((N + 255) / 256);
  const long long tiles_256 = (long long)((M + 127) / 128) * ((N + 255) / 256);
  // 256 x 128 pair tiles where 256-wide ones would occupy fewer than half of the SM pairs (the text prefill's
  // 730 x 2048 proj / fc2: 24 -> 48 tiles); VT_GEMM_PAIR_BN=256 / 128 forces one width (A/B switch)
  static const int pair_bn = [] {
    const char* e = getenv("VT_GEMM_PAIR_BN");
    return e ? atoi(e) : 0;
  }();
  if (pair && M > 128 && tiles_pair >= sms / 8) {
    const int pbn = pair_bn == 256 ? 256 : (pair_bn == 128 || tiles_pair * 4 < sms) ? 128 : 256;
    return launch_pair(st, A, lda, W, ldw, M, N, K, ep, i8, pbn);
  }
  if (forced == 256 || tiles_256 >= sms / 2)
    return i8 ? launch_bn<256, true>(st, A, lda, W, ldw, M, N, K, ep)
              : launch_bn<256, false>(st, A, lda, W, ldw, M, N, K, ep);
  return i8 ? launch_bn<64, true>(st, A, lda, W, ldw, M, N, K, ep)
            : launch_bn<64, false>(st, A, lda, W, ldw, M, N, K, ep);
}

}  // namespace gemm
}  // namespace vt

extern "C" long long vt_gemm_ws_bytes(int M, int N);

namespace vt {
namespace gemm {
// Points ep's split-K state into the caller's workspace (null: no split-K).
static int set_workspace(Epi& ep, void* ws, long long ws_bytes, int M, int N) {
  if (!ws || M <= 0 || N <= 0) return OK;
  if (!aligned16(ws) || ws_bytes < vt_gemm_ws_bytes(M, N))
    return set_error(E_SHAPE, "vt_gemm: workspace of %lld bytes (needs %lld, 16-byte aligned)", ws_bytes,
                     vt_gemm_ws_bytes(M, N));
  const int p = (N + 31) / 32 * 32;
  const size_t planes = (size_t)kMaxSplit * M * p * 4;
  ep.sk_cnt = static_cast<int*>(ws);
  ep.sk_ws = reinterpret_cast<float*>(static_cast<char*>(ws) + ((size_t)ws_bytes / 16 * 16 - planes));
  ep.sk_pitch = p;
  return OK;
}
}  // namespace gemm
}  // namespace vt

extern "C" {

int vt_gemm_fused_ws(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M, int N,
                     int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
                     long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2, float* stats_out,
                     const float* ln_moments, const float* ln_c, int tiles_T, int tiles_H, int tiles_D, void* ws,
                     long long ws_bytes);

// C[M,N] (bf16, pitch ldc) = A[M,K] . W[N,K]^T + bias, optionally GELU-tanh (after bf16 rounding).
int vt_gemm_bf16(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw,
                 const float* bias, uint16_t* C, long long ldc, int M, int N, int K, int gelu) {
  vt::gemm::Epi ep{bias, C, ldc, nullptr, 0, 0, 0, 0, gelu ? 1 : 0, nullptr, 0, 0, 0, 0, 0, 0, nullptr, nullptr, nullptr, 0};
  return vt::gemm::launch(st, A, lda, W, ldw, M, N, K, ep);
}

// General form.  out_f32 selects fp32 output (no GELU); res (fp32, or bf16 when res_bf16) is added
// after the bias, read at row (m % res_period) when res_period > 0; out2 receives a bf16 copy of an
// fp32 output.  res may alias out (in-place residual update).
int vt_gemm_ex(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M, int N, int K,
               const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res, long long ldr,
               int res_period, int res_bf16, uint16_t* out2, long long ldo2) {
  vt::gemm::Epi ep{bias, out, ldo, res, ldr, res_period, res_bf16 ? 1 : 0, out_f32 ? 1 : 0, gelu ? 1 : 0, out2, ldo2,
                   0, 0, 0, 0, 0, nullptr, nullptr, nullptr, 0};
  return vt::gemm::launch(st, A, lda, W, ldw, M, N, K, ep);
}

// Superset of vt_gemm_ex with the LayerNorm fusions of the tower (see include/vt_b200.h):
//   stats_out  (fp32 output only): per-32-column chunk (mean, M2) of every output row;
//   ln_moments / ln_c: LayerNorm of the A rows folded into the epilogue;
//   tiles_T > 0: bf16 output scattered into the attention-tile layout (N = 3*tiles_H*tiles_D).
int vt_gemm_fused(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M, int N,
                  int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
                  long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2, float* stats_out,
                  const float* ln_moments, const float* ln_c, int tiles_T, int tiles_H, int tiles_D) {
  return vt_gemm_fused_ws(st, A, lda, W, ldw, M, N, K, bias, out, ldo, out_f32, gelu, res, ldr, res_period, res_bf16,
                          out2, ldo2, stats_out, ln_moments, ln_c, tiles_T, tiles_H, tiles_D, nullptr, 0);
}

// Workspace of vt_gemm_fused_ws for an M x N output: int arrival counters [M][P/32] at its start and up to
// 16 fp32 partial-sum planes [M][P] at its end, P = N rounded up to 32.  Calls of other shapes sharing a
// workspace sized for the largest keep the same two ends, so one call's partial sums never land on
// another's counters (which must read zero when a call starts).
long long vt_gemm_ws_bytes(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  const long long p = ((long long)N + 31) / 32 * 32;
  return ((long long)M * (p / 32) * 4 + 15) / 16 * 16 + (long long)vt::gemm::kMaxSplit * M * p * 4;
}

// vt_gemm_fused with a workspace (ws_bytes >= vt_gemm_ws_bytes(M, N), zero-filled when allocated) that lets
// the small-tile path split K across CTAs; every call leaves the counters at zero again.  ws may be null.
int vt_gemm_fused_ws(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M, int N,
                     int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
                     long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2, float* stats_out,
                     const float* ln_moments, const float* ln_c, int tiles_T, int tiles_H, int tiles_D, void* ws,
                     long long ws_bytes) {
  using namespace vt;
  if (tiles_T > 0) {
    if (tiles_H <= 0 || tiles_D <= 0 || tiles_D % 8 || tiles_D > 80 || M % tiles_T || N != 3 * tiles_H * tiles_D ||
        out_f32 || gelu || res || out2 || stats_out || !aligned16(out))
      return set_error(E_SHAPE, "vt_gemm_fused: attention-tile output needs bf16, N = 3*H*D, M a multiple of T");
  }
  vt::gemm::Epi ep{bias, out, ldo, res, ldr, res_period, res_bf16 ? 1 : 0, out_f32 ? 1 : 0, gelu == 2 ? 3 : gelu ? 1 : 0,
                   out2, ldo2, tiles_T > 0 ? tiles_T : 0, tiles_H, tiles_D, tiles_D <= 64 ? 8 : 10,
                   tiles_T > 0 ? (tiles_T + 127) / 128 : 0, reinterpret_cast<float2*>(stats_out),
                   reinterpret_cast<const float2*>(ln_moments), ln_c, 0};
  const int rc = vt::gemm::set_workspace(ep, ws, ws_bytes, M, N);
  if (rc) return rc;
  return vt::gemm::launch(st, A, lda, W, ldw, M, N, K, ep);
}

// vt_gemm_fused_ws with the folded norm's row factors merged in the epilogue from the chunk statistics that
// the last writer of the A rows left (ln_stats [M][ln_nchunk] float pairs; ln_rms selects RMSNorm) instead of
// a vt_row_moments / vt_row_rms pass; ln_mom_out (may be null) receives the (mean, rstd) pairs.
int vt_gemm_fused_lnstats(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M,
                          int N, int K, const float* bias, void* out, long long ldo, int out_f32, int gelu,
                          const void* res, long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2,
                          float* stats_out, const float* ln_stats, int ln_nchunk, float ln_eps, int ln_rms,
                          const float* ln_c, float* ln_mom_out, int tiles_T, int tiles_H, int tiles_D, void* ws,
                          long long ws_bytes) {
  using namespace vt;
  if (!ln_stats) return set_error(E_SHAPE, "vt_gemm_fused_lnstats: ln_stats is required");
  if (tiles_T > 0) {
    if (tiles_H <= 0 || tiles_D <= 0 || tiles_D % 8 || tiles_D > 80 || M % tiles_T || N != 3 * tiles_H * tiles_D ||
        out_f32 || gelu || res || out2 || stats_out || !aligned16(out))
      return set_error(E_SHAPE, "vt_gemm_fused_lnstats: attention-tile output needs bf16, N = 3*H*D, M a multiple of T");
  }
  vt::gemm::Epi ep{bias, out, ldo, res, ldr, res_period, res_bf16 ? 1 : 0, out_f32 ? 1 : 0, gelu == 2 ? 3 : gelu ? 1 : 0,
                   out2, ldo2, tiles_T > 0 ? tiles_T : 0, tiles_H, tiles_D, tiles_D <= 64 ? 8 : 10,
                   tiles_T > 0 ? (tiles_T + 127) / 128 : 0, reinterpret_cast<float2*>(stats_out), nullptr, ln_c, 0};
  ep.ln_stats = reinterpret_cast<const float2*>(ln_stats);
  ep.ln_nchunk = ln_nchunk;
  ep.ln_eps = ln_eps;
  ep.ln_rms = ln_rms ? 1 : 0;
  ep.ln_mom_out = reinterpret_cast<float2*>(ln_mom_out);
  const int rc = vt::gemm::set_workspace(ep, ws, ws_bytes, M, N);
  if (rc) return rc;
  return vt::gemm::launch(st, A, lda, W, ldw, M, N, K, ep);
}

// W8A8 int8 GEMM: out[M,N] = epilogue(((float)(A[M,K] . W[N,K]^T) * sa[m]) * sw[n] + bias[n]), the int32
// dot products exact, GELU-tanh on the fp32 value when gelu; A / W signed int8 with pitches in bytes
// (multiples of 16).  Same output / residual / workspace rules as vt_gemm_fused_ws.
int vt_gemm_i8(cudaStream_t st, const int8_t* A, long long lda, const int8_t* W, long long ldw, const float* sa,
               const float* sw, int M, int N, int K, const float* bias, void* out, long long ldo, int out_f32, int gelu,
               const void* res, long long ldr, int res_bf16, void* ws, long long ws_bytes) {
  using namespace vt;
  if ((M > 0 && N > 0) && (!sa || !sw || !aligned16(sw)))
    return set_error(E_SHAPE, "vt_gemm_i8: row scales sa and 16-byte aligned column scales sw are required");
  vt::gemm::Epi ep{bias, out, ldo, res, ldr, 0, res_bf16 ? 1 : 0, out_f32 ? 1 : 0, gelu ? 2 : 0, nullptr, 0,
                   0, 0, 0, 0, 0, nullptr, nullptr, nullptr, 0};
  ep.i8_sa = sa;
  ep.i8_sw = sw;
  const int rc = vt::gemm::set_workspace(ep, ws, ws_bytes, M, N);
  if (rc) return rc;
  return vt::gemm::launch(st, A, lda, W, ldw, M, N, K, ep, true);
}

// Fused QKV projection for attention: A[M = crops*T, K] . W[3*H*D, K]^T + bias, written as bf16 straight
// into the attention-tile layout of vt_attn_tiles_fwd (`tiles` holds vt_attn_tiles_bytes(M/T, T, H, D)
// bytes, zero-filled once when allocated; its pad rows and lanes are never written).
int vt_gemm_qkv_tiles(cudaStream_t st, const uint16_t* A, long long lda, const uint16_t* W, long long ldw,
                      const float* bias, uint16_t* tiles, int M, int K, int T, int H, int D) {
  using namespace vt;
  if (T <= 0 || H <= 0 || D <= 0 || D % 8 || D > 80 || M < 0 || M % T)
    return set_error(E_SHAPE, "vt_gemm_qkv_tiles: M=%d T=%d H=%d D=%d invalid (M a multiple of T, D%%8 == 0, D <= 80)", M,
                     T, H, D);
  if (!aligned16(tiles)) return set_error(E_SHAPE, "vt_gemm_qkv_tiles: tiles must be 16-byte aligned");
  vt::gemm::Epi ep{bias, tiles, 0, nullptr, 0, 0, 0, 0, 0, nullptr, 0, T, H, D, D <= 64 ? 8 : 10, (T + 127) / 128,
                   nullptr, nullptr, nullptr, 0};
  return vt::gemm::launch(st, A, lda, W, ldw, M, 3 * H * D, K, ep);
}

}  // extern "C"
