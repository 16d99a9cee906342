// Flash attention on the 5th-generation tensor cores (tcgen05 / TMEM), the B200 replacement of the
// reference's attn_fwd2 (moondream/gpu/hip/attn.hip:142-272, 442) and its V^T copy (vtranspose,
// attn.hip:275-288) behind hattn.Attn (moondream/gpu/hattn.py:17-37).
//
// Operand layout ("attention tiles"): for crop b, operand w (0 q, 1 k, 2 v), head h, token t, 8-element d
// chunk c:  tiles[((b*3 + w)*H + h)*Tt*NC*1024 + attn_tile_off(w, t, c, NC) + e]  (vt_common.cuh), with
// Tt = ceil(T/128), NC = DP/8, DP = 64 or 80 (head_dim padded to the tensor-core K granularity).  A
// 128-token Q tile is [c][128][8] and each 64-token half of a K or V tile [c][64][8], NC*2 KB and NC KB
// contiguous in exactly the canonical no-swizzle layout tcgen05 reads (8-row x 16-byte core matrices), so
// each arrives with one cp.async.bulk.  Rows t >= T and lanes d >= D are zero (the buffer is zeroed once at
// allocation and never written there).  The tower's QKV GEMM writes this layout from its epilogue;
// vt_attn_pack builds it from any strided Q/K/V.
//
// CTA = one 128-query tile of one (crop, head), or one 64-query half of it (QR = 64, M = 64 MMAs, for grids of
// fewer than two 128-query CTAs per SM and fewer than 16 key tiles: the accumulator rows then sit in lanes 0-15
// of each TMEM lane quarter, lanes 16-31 of every warp carry no row; with 16 or more key tiles such grids split
// the keys instead, KS = 2 below), 2 CTAs per SM; 6 warps:
//   warp 4 lane 0: bulk loads (Q once, then K_j and V_j per 64-key tile, KVS-stage rings);
//   warp 5 lane 0: tcgen05.mma  S_j = Q K_j^T (M 128, N 64, K DP) into one of two TMEM S buffers, then
//                  O += P_j V_j (M 128, N DP, K 64; P read from TMEM, V an MN-major B operand in shared
//                  memory) into a TMEM accumulator;
//   warps 0-3: softmax, thread i owns query row i (TMEM lane i): row max, P = 2^(s*scale*log2e - m) as
//              bf16 pairs written back over S, row sums in fp32.
// O is rescaled only when a row max grows by more than 2^8 (P <= 256 otherwise, exact in fp32
// accumulation), so TMEM round trips of O are rare.  tcgen05 ops of one thread complete in issue order.
#include <mutex>

#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace attn_tc {

constexpr int BQ = 128, BKV = 64, THREADS = 192;
#ifndef VT_ATTN_KVS
#define VT_ATTN_KVS 3
#endif
constexpr int KVS = VT_ATTN_KVS;  // K and V ring stages (two CTAs share an SM's 228 KB)
constexpr uint32_t TMEM_COLS = 256;  // S buffers: columns [0, 64) and [64, 128); O: [128, 128 + DP)
constexpr long long kDrainCycles = 200000000LL;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int NC>
struct Smem {
  static constexpr int QT = NC * 2048;  // bytes of the 128-row Q tile
  static constexpr int KT = NC * 1024;  // bytes of a 64-row K or V tile
  static constexpr int Q = 0;
  static constexpr int K = QT;                      // KVS stages
  static constexpr int V = QT + KVS * KT;           // KVS stages
  // P lives in tensor memory, over the S buffer it was computed from (bf16 pairs in its first 32 columns)
  static constexpr int BAR = QT + 2 * KVS * KT;
  static constexpr int BYTES = BAR + 256;
};

struct Args {
  const uint16_t* tiles;
  uint16_t* o;
  int T, H, D, Tt;
  long long so_b, so_t, so_h;
  float scale_log2;
  int b0;
};

// Pipeline per CTA (one 128-query tile), key tiles of 64, j = 0 .. nkv-1:
//   MMA thread:  S_0;  then for each j: S_(j+1) into the other S buffer, wait P_j, O += P_j V_j.
//                So the tensor core computes S_(j+1) while the softmax warps work on S_j.
//   softmax:     wait S_j, row max, (rare) O rescale after PV_(j-1) is done, P_j = 2^(s - m) as bf16 pairs
//                into the first 32 columns of S buffer j%2 (tcgen05.st), arrive.  The MMA reads P_j from tensor
//                memory (A operand); S_(j+2), the next writer of that buffer, is issued after PV_j and the
//                tensor core runs them in order.
//
// KS = 2 (grids of fewer than two query-tile CTAs per SM and 16 or more key tiles: a TAPNext frame): the keys
// of a query tile are split over a cluster of two CTAs, each running the pipeline above on its half of the key
// tiles, so a CTA's chain of key tiles is half as long.  At the end rank 1 sends its unnormalised O rows with
// their row max and row sum into rank 0's shared memory (over its then idle K / V ring) and rank 0 merges the
// two halves (flash-decoding's rescale by 2^(m_i - max m)) and stores the output.
template <int NC, int QR, int KS>
__global__ void __launch_bounds__(THREADS, 2) attn_tc_kernel(Args a) {
  using L = Smem<NC>;
  constexpr int DP = NC * 8;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;            // [KVS]
  uint64_t* k_empty = bar + 1 + KVS;     // [KVS]
  uint64_t* v_full = bar + 1 + 2 * KVS;  // [KVS]
  uint64_t* v_empty = bar + 1 + 3 * KVS; // [KVS]
  uint64_t* s_full = bar + 1 + 4 * KVS;  // [2]
  uint64_t* p_full = s_full + 2;         // [2], one arrival per softmax warp
  uint64_t* o_full = s_full + 4;
  uint64_t* drain = s_full + 5;
  constexpr int NBAR = 1 + 4 * KVS + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  static_assert(KS == 1 || QR == 128, "the key split runs 128-query tiles");
  const int tt = (QR == 128 && KS == 1) ? blockIdx.x : blockIdx.x >> 1, hq = QR == 128 ? 0 : blockIdx.x & 1;
  const int ks = KS == 2 ? (int)(blockIdx.x & 1) : 0;  // the cluster rank: blockIdx.x pairs form the clusters
  const int h = blockIdx.y, b = a.b0 + blockIdx.z;
  const int T = a.T, H = a.H, Tt = a.Tt;
  const int nkv_all = (T + BKV - 1) / BKV;
  const int kt0 = nkv_all * ks / KS;                    // this CTA's key tiles: [kt0, kt0 + nkv)
  const int nkv = nkv_all * (ks + 1) / KS - kt0;
  const size_t tile_elems = (size_t)NC * 1024;  // one 128-row tile of one operand
  const uint16_t* q_src = a.tiles + ((((size_t)b * 3 + 0) * H + h) * Tt + tt) * tile_elems;
  const uint16_t* k_base = a.tiles + ((((size_t)b * 3 + 1) * H + h) * Tt) * tile_elems;
  const uint16_t* v_base = a.tiles + ((((size_t)b * 3 + 2) * H + h) * Tt) * tile_elems;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBAR; i++) mbar_init(&bar[i], 1);
    mbar_init(&p_full[0], 4);  // one arrival per softmax warp
    mbar_init(&p_full[1], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 128;
  griddep_wait();  // programmatic dependent launch: the tiles' producer has completed
  griddep_launch();
  float m_used = -INFINITY, l = 0.f;  // softmax threads: the row's running max (log2 units) and sum
  bool have_o = false;                // (KS = 2) softmax threads: O complete

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- bulk loads: Q once (NC * 2 KB); per 64-key tile one NC KB copy each for K and V.
      // The MMA thread needs K_(j+1) (for S_(j+1)) before V_j (for PV_j), and K_(j+1)'s stage frees when
      // S_(j+1-KVS) completes while V_j's frees only when PV_(j-KVS) does: so K is issued one tile ahead
      // of V and never queues behind a V wait.
      bool ok = true;
      int last_k = 0, last_v = -1;  // last key tiles whose K / V copies were issued
      auto load_kv = [&](uint64_t* full, const uint16_t* base, int j, int off) {
        const int g = kt0 + j;  // the key tile's index in the head
        const uint16_t* src = base + (size_t)(g >> 1) * tile_elems + (size_t)(g & 1) * NC * 512;
        mbar_arrive_expect_tx(full, L::KT);
        bulk_load(sm + off + (j % KVS) * L::KT, src, L::KT, full);
      };
      mbar_arrive_expect_tx(q_full, L::QT);
      bulk_load(sm + L::Q, q_src, L::QT, q_full);
      load_kv(&k_full[0], k_base, 0, L::K);
      for (int j = 0; j < nkv && ok; j++) {
        const int k1 = j + 1;
        if (k1 < nkv) {
          if (k1 >= KVS && !mbar_wait(&k_empty[k1 % KVS], (k1 / KVS - 1) & 1, abort_flag, ST_ATTN_PRODUCER)) { ok = false; break; }
          load_kv(&k_full[k1 % KVS], k_base, k1, L::K);
          last_k = k1;
        }
        if (j >= KVS && !mbar_wait(&v_empty[j % KVS], (j / KVS - 1) & 1, abort_flag, ST_ATTN_PRODUCER)) { ok = false; break; }
        load_kv(&v_full[j % KVS], v_base, j, L::V);
        last_v = j;
      }
      if (!ok) {  // unwinding: let the copies this thread issued land before the CTA exits
        mbar_wait_drain(q_full, 0, kDrainCycles);
        for (int j = last_k >= KVS ? last_k - KVS + 1 : 0; j <= last_k; j++)
          mbar_wait_drain(&k_full[j % KVS], (j / KVS) & 1, kDrainCycles);
        for (int j = last_v >= KVS ? last_v - KVS + 1 : 0; j <= last_v; j++)
          mbar_wait_drain(&v_full[j % KVS], (j / KVS) & 1, kDrainCycles);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC_S = idesc_bf16(QR, BKV);
      constexpr uint32_t IDESC_O = idesc_bf16(QR, DP) | (1u << 16);  // B (= V) MN-major
      const uint32_t sq = smem_u32(sm + L::Q), sk = smem_u32(sm + L::K), sv = smem_u32(sm + L::V);
      // S_j = Q K_j^T into S buffer j%2; k_ready: K_j is known to have landed (checked off the S chain)
      auto issue_s = [&](int j, bool k_ready) -> bool {
        const int s = j & 1;
        const int ks = j % KVS;
        if (!k_ready && !mbar_wait(&k_full[ks], (j / KVS) & 1, abort_flag, ST_ATTN_MMA)) return false;
        tc_fence_after();
        const uint32_t kb = sk + ks * L::KT;
#pragma unroll
        for (int k = 0; k < NC / 2; k++)  // K = 16 per MMA: Q chunks 2k, 2k+1 (2048 B apart), K chunks (1024 B apart)
          umma_f16(tmem + s * BKV, sdesc_noswz(sq + hq * 1024 + k * 4096, 2048, 128), sdesc_noswz(kb + k * 2048, 1024, 128),
                   IDESC_S, k > 0 ? 1u : 0u);
        umma_commit(&s_full[s]);  // first: the softmax warps wait on this one
        umma_commit(&k_empty[ks]);
        return true;
      };
      // The chain that sets the tile rate runs P_j -> PV_j -> S_(j+2) (issued at the top of the next
      // iteration) -> softmax of tile j+2, and one thread issues a tcgen05.mma every ~48 cycles and a commit
      // every ~44 (measured): so the chain carries one commit per MMA group (O's rescale waits on v_empty, there
      // is no separate PV barrier), and every wait that can be settled before P_j arrives is settled then (V_j,
      // and a non-blocking look at K_(j+2), which usually has landed; its phase cannot alias: K_(j+2-KVS) was
      // waited for and K_(j+2+KVS) needs S_(j+2)).
      bool ok = mbar_wait(q_full, 0, abort_flag, ST_ATTN_MMA) && issue_s(0, false);
      bool k_next = false;  // K_(j+1) seen landed during iteration j-1
      for (int j = 0; j < nkv && ok; j++) {
        const int s = j & 1;
        if (j + 1 < nkv && !issue_s(j + 1, k_next)) { ok = false; break; }
        if (!mbar_wait(&v_full[j % KVS], (j / KVS) & 1, abort_flag, ST_ATTN_MMA)) { ok = false; break; }
        k_next = j + 2 < nkv && mbar_try_wait(&k_full[(j + 2) % KVS], ((j + 2) / KVS) & 1);
        if (!mbar_wait(&p_full[s], (j >> 1) & 1, abort_flag, ST_ATTN_MMA)) { ok = false; break; }
        tc_fence_after();
        const uint32_t vb = sv + (j % KVS) * L::KT;
#pragma unroll
        for (int k = 0; k < BKV / 16; k++)  // 16 keys per MMA: P columns 8k .. 8k+7 of S buffer s; V rows 16k ..
          umma_f16_ts(t_o, tmem + s * BKV + k * 8, sdesc_noswz(vb + k * 256, 128, 1024), IDESC_O,
                      (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(&v_empty[j % KVS]);
      }
      if (ok) umma_commit(o_full);
      umma_commit(drain);
      mbar_wait_drain(drain, 0, kDrainCycles);
    }
  } else {
    // ---------------- softmax warps 0-3: thread = query row
    const bool has_row = QR == 128 || lane < 16;  // M = 64: rows 16w .. 16w+15 in lanes 0-15 of quarter w
    const int row = QR == 128 ? warp * 32 + lane : warp * 16 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    for (int j = 0; j < nkv; j++) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, abort_flag, ST_ATTN_SOFTMAX)) { ok = false; break; }
      tc_fence_after();
      const uint32_t t_s = tmem + s * BKV + lane_off;
      const int kbase = (kt0 + j) * BKV;
      const bool tail = kbase + BKV > T;  // only the last key tile has keys past T (zero rows, masked)
      uint32_t r0[32], r1[32];
      tmem_ld32(t_s, r0);
      tmem_ld32(t_s + 32, r1);
      tmem_ld_wait();
      // keys past T only exist in the last tile: their scores become -inf in place, so the max below ignores
      // them and the exponentials give exactly 0 (ex2.approx(-inf) = +0) with no per-key test in the loop
      if (tail) {
#pragma unroll
        for (int e = 0; e < 32; e++) {
          if (kbase + e >= T) r0[e] = 0xff800000u;
          if (kbase + 32 + e >= T) r1[e] = 0xff800000u;
        }
      }
      // row max as a tree of three-input maxima (64 -> 22 -> 8 -> 3 -> 1)
      float t[64];
#pragma unroll
      for (int e = 0; e < 32; e++) {
        t[e] = __uint_as_float(r0[e]);
        t[32 + e] = __uint_as_float(r1[e]);
      }
#pragma unroll
      for (int e = 0; e < 21; e++) t[e] = max3f(t[3 * e], t[3 * e + 1], t[3 * e + 2]);
      t[21] = t[63];
#pragma unroll
      for (int e = 0; e < 7; e++) t[e] = max3f(t[3 * e], t[3 * e + 1], t[3 * e + 2]);
      t[7] = t[21];
      t[0] = max3f(t[0], t[1], t[2]);
      t[1] = max3f(t[3], t[4], t[5]);
      t[2] = fmaxf(t[6], t[7]);
      float mx = max3f(t[0], t[1], t[2]);
      mx *= a.scale_log2;
      if (j == 0) {
        m_used = mx;
      } else {
        const bool need = has_row && mx > m_used + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {  // O round trip through registers (warp-collective), rare
          // O must hold every P.V up to j-1: wait for PV_(j-1) on its V stage's barrier.  S_j is complete, so
          // PV_(j-2) and everything before it are too, and PV_(j-1+KVS), the next arrival on that barrier, needs P_j
          if (!mbar_wait(&v_empty[(j - 1) % KVS], ((j - 1) / KVS) & 1, abort_flag, ST_ATTN_SOFTMAX)) { ok = false; break; }
          tc_fence_after();
          const float m_new = need ? mx : m_used;
          const float alpha = exp2f(m_used - m_new);
          m_used = m_new;
          l *= alpha;
#pragma unroll
          for (int c = 0; c < DP / 16; c++) {
            uint32_t r[16];
            tmem_ld16(t_o + lane_off + c * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; e++) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st16(t_o + lane_off + c * 16, r);
          }
          tmem_st_wait();
        }
      }
      // P = 2^(s * scale_log2 - m) with the scale and shift done two lanes at a time (fma.rn.f32x2); the
      // row sum accumulates in four independent fp32x2 partial sums
      const unsigned long long sl2 = f2_pack(a.scale_log2, a.scale_log2), neg_m = f2_pack(-m_used, -m_used);
      unsigned long long sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const uint32_t* r = c ? r1 : r0;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; e++) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1])), sl2, neg_m), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          sum2[e & 3] = f2_add(sum2[e & 3], f2_pack(p0, p1));
          pk[e] = pack_bf2(p0, p1);
        }
        tmem_st16(t_s + c * 16, pk);  // keys 32c .. 32c+31 as bf16 pairs: S columns 16c .. 16c+15 (S is in r0 / r1)
      }
      {
        const unsigned long long s01 = f2_add(sum2[0], sum2[1]), s23 = f2_add(sum2[2], sum2[3]);
        float lo, hi;
        f2_unpack(f2_add(s01, s23), lo, hi);
        l += lo + hi;
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    if (KS == 2) {
      have_o = __all_sync(0xffffffffu, ok && mbar_wait(o_full, 0, abort_flag, ST_ATTN_SOFTMAX));
      if (have_o) tc_fence_after();
    } else if (ok && mbar_wait(o_full, 0, abort_flag, ST_ATTN_SOFTMAX)) {
      tc_fence_after();
      const int t = tt * BQ + hq * QR + row;
      const float inv = 1.f / l;
      uint16_t* orow = a.o + (size_t)b * a.so_b + (size_t)t * a.so_t + (size_t)h * a.so_h;
#pragma unroll
      for (int c = 0; c < DP / 16; c++) {
        uint32_t r[16];
        tmem_ld16(t_o + lane_off + c * 16, r);
        tmem_ld_wait();
        if (has_row && t < T) {
#pragma unroll
          for (int half = 0; half < 2; half++) {
            const int d0 = c * 16 + half * 8;
            if (d0 < a.D)
              *reinterpret_cast<uint4*>(orow + d0) =
                  make_uint4(pack_bf2(__uint_as_float(r[8 * half]) * inv, __uint_as_float(r[8 * half + 1]) * inv),
                             pack_bf2(__uint_as_float(r[8 * half + 2]) * inv, __uint_as_float(r[8 * half + 3]) * inv),
                             pack_bf2(__uint_as_float(r[8 * half + 4]) * inv, __uint_as_float(r[8 * half + 5]) * inv),
                             pack_bf2(__uint_as_float(r[8 * half + 6]) * inv, __uint_as_float(r[8 * half + 7]) * inv));
          }
        }
      }
    }
  }
  if constexpr (KS == 2) {
    // every MMA of both CTAs is complete and every load has landed: rank 0's K / V ring takes rank 1's rows
    // while rank 0 still holds its own O in tensor memory.  16-byte chunk q of row i (O columns 4q .. 4q+3; chunk
    // DP/4 = m, l, a valid flag) sits at (q * 128 + i) * 16 bytes, so a warp's 32 rows fill 512 consecutive bytes
    // (no bank conflicts on either side)
    constexpr int NQ = DP / 4 + 1;  // 16-byte chunks per row
    static_assert(NQ * 128 * 16 <= L::BAR - L::K, "the merge buffer must fit in the K / V ring");
    const uint32_t rx = smem_u32(sm + L::K);
    const int row = warp * 32 + lane;
    const uint32_t t_row = t_o + ((uint32_t)(warp * 32) << 16);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp < 4 && ks == 1) {
      const uint32_t dst = mapa_shared(rx + (uint32_t)(row * 16), 0);
      if (have_o) {
#pragma unroll
        for (int c = 0; c < DP / 16; c++) {
          uint32_t r[16];
          tmem_ld16(t_row + c * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            st_cluster_v4(dst + (uint32_t)((c * 4 + e / 4) * 2048), r[e], r[e + 1], r[e + 2], r[e + 3]);
        }
      }
      st_cluster_v4(dst + (uint32_t)((NQ - 1) * 2048), __float_as_uint(m_used), __float_as_uint(l), have_o ? 1u : 0u, 0u);
    }
    __syncwarp();
    cluster_sync();  // release / acquire: rank 1's rows are visible in rank 0's shared memory
    if (warp < 4 && ks == 0) {
      const float4* prow = reinterpret_cast<const float4*>(sm + L::K) + row;  // chunk q at prow[q * 128]
      const int t = tt * BQ + row;
      const float4 ml = prow[(NQ - 1) * 128];
      const float m1 = ml.x, l1 = ml.y;
      const bool both = have_o && __float_as_uint(ml.z) == 1u;
      const float mx = fmaxf(m_used, m1);
      const float a0 = exp2f(m_used - mx), a1 = exp2f(m1 - mx);
      const float inv = 1.f / (l * a0 + l1 * a1);
      const float s0 = a0 * inv, s1 = a1 * inv;
      uint16_t* orow = a.o + (size_t)b * a.so_b + (size_t)t * a.so_t + (size_t)h * a.so_h;
#pragma unroll
      for (int c = 0; c < DP / 16; c++) {
        uint32_t r[16];
        tmem_ld16(t_row + c * 16, r);
        tmem_ld_wait();
        if (both && t < T) {
#pragma unroll
          for (int half = 0; half < 2; half++) {
            const int d0 = c * 16 + half * 8;
            if (d0 < a.D) {
              const float4 p0 = prow[(d0 / 4) * 128], p1 = prow[(d0 / 4 + 1) * 128];
              const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; e++) v[e] = __uint_as_float(r[8 * half + e]) * s0 + pv[e] * s1;
              *reinterpret_cast<uint4*>(orow + d0) = make_uint4(pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]),
                                                                pack_bf2(v[4], v[5]), pack_bf2(v[6], v[7]));
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Strided Q/K/V -> attention tiles.  One thread per 16-byte chunk (8 elements of d); rows t < T and
// chunks c < D/8 only (the pads keep their zeros).
__global__ void __launch_bounds__(256) pack_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                   const uint16_t* __restrict__ v, uint16_t* __restrict__ tiles, int B,
                                                   int T, int H, int D, int NC, int Tt, long long sq_b, long long sq_t,
                                                   long long sq_h, long long sk_b, long long sk_t, long long sk_h,
                                                   long long sv_b, long long sv_t, long long sv_h) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int dch = D / 8;
  const long long per_tok = 3LL * H * dch;
  const long long total = (long long)B * T * per_tok;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    long long r = i;
    const int c = (int)(r % dch); r /= dch;
    const int hh = (int)(r % H); r /= H;
    const int w = (int)(r % 3); r /= 3;
    const int t = (int)(r % T);
    const long long bb = r / T;
    const uint16_t* src = w == 0 ? q + bb * sq_b + t * sq_t + hh * sq_h
                        : w == 1 ? k + bb * sk_b + t * sk_t + hh * sk_h
                                 : v + bb * sv_b + t * sv_t + hh * sv_h;
    const size_t dst = (((size_t)bb * 3 + w) * H + hh) * Tt * ((size_t)NC * 1024) + attn_tile_off(w, t, c, NC);
    *reinterpret_cast<uint4*>(tiles + dst) = *reinterpret_cast<const uint4*>(src + c * 8);
  }
}

// Once per device, with that device current: the dynamic shared-memory size and carveout of both
// instantiations (head_dim <= 64 and <= 80).  std::call_once keeps first calls from several host threads safe.
int prepare_device() {
  static std::once_flag once[64];
  static cudaError_t status[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(E_LAUNCH, "attention: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(E_LAUNCH, "attention: device %d out of range", dev);
  std::call_once(once[dev], [dev] {
    // two CTAs per SM need (almost) the whole 228 KB as shared memory
    auto set = [](auto kernel, int bytes) {
      cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      return r == cudaSuccess ? cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) : r;
    };
    cudaError_t r = set(attn_tc_kernel<8, 128, 1>, Smem<8>::BYTES);
    if (r == cudaSuccess) r = set(attn_tc_kernel<8, 64, 1>, Smem<8>::BYTES);
    if (r == cudaSuccess) r = set(attn_tc_kernel<8, 128, 2>, Smem<8>::BYTES);
    if (r == cudaSuccess) r = set(attn_tc_kernel<10, 128, 1>, Smem<10>::BYTES);
    if (r == cudaSuccess) r = set(attn_tc_kernel<10, 64, 1>, Smem<10>::BYTES);
    if (r == cudaSuccess) r = set(attn_tc_kernel<10, 128, 2>, Smem<10>::BYTES);
    status[dev] = r;
  });
  if (status[dev] != cudaSuccess)
    return set_error(E_LAUNCH, "attention: setting the kernel attributes: %s", cudaGetErrorString(status[dev]));
  return OK;
}

// launch_k with clusters of two CTAs along x (the key split)
template <typename... KArgs, typename... Args>
static cudaError_t launch_pairs(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

template <int NC, int QR, int KS>
static int launch_nc(cudaStream_t st, Args a, int B) {
  int rc = prepare_device();
  if (rc) return rc;
  for (int b0 = 0; b0 < B; b0 += 65535) {
    a.b0 = b0;
    const int nb = (B - b0) < 65535 ? (B - b0) : 65535;
    const dim3 grid(a.Tt * (128 / QR) * KS, a.H, nb);
    if (KS == 2) launch_pairs(attn_tc_kernel<NC, QR, KS>, grid, THREADS, Smem<NC>::BYTES, st, a);
    else launch_k(attn_tc_kernel<NC, QR, KS>, grid, THREADS, Smem<NC>::BYTES, st, a);
    rc = check_launch("vt_attn_tiles_fwd");
    if (rc) return rc;
  }
  return OK;
}

static int dp_chunks(int D) { return D <= 64 ? 8 : 10; }

}  // namespace attn_tc
}  // namespace vt

extern "C" {

// Bytes of the attention-tile buffer for B crops x H heads x T tokens, head_dim D (0 if unsupported).
long long vt_attn_tiles_bytes(int B, int T, int H, int D) {
  if (B < 0 || T < 0 || H < 0 || D <= 0 || D % 8 || D > 80) return 0;
  const long long Tt = (T + 127) / 128;
  return (long long)B * 3 * H * Tt * vt::attn_tc::dp_chunks(D) * 1024 * 2;
}

// Strided Q/K/V (element (b,t,h,d) at X + b*sx_b + t*sx_t + h*sx_h + d) -> attention tiles.  `tiles`
// must hold vt_attn_tiles_bytes(B, T, H, D) bytes and be zero-filled once when allocated.
int vt_attn_pack(cudaStream_t st, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* tiles, int B,
                 int T, int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b, long long sk_t,
                 long long sk_h, long long sv_b, long long sv_t, long long sv_h) {
  using namespace vt;
  if (B < 0 || T < 0 || H < 0) return set_error(E_SHAPE, "vt_attn_pack: negative shape");
  if (B == 0 || T == 0 || H == 0) return OK;
  if (D <= 0 || D % 8 || D > 80) return set_error(E_VARIANT, "vt_attn_pack: head_dim %d unsupported", D);
  const long long s16[] = {sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h};
  for (long long s : s16)
    if (s % 8) return set_error(E_SHAPE, "vt_attn_pack: strides must be multiples of 8 elements");
  if (!Q || !K || !V || !tiles || !aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(tiles))
    return set_error(E_SHAPE, "vt_attn_pack: pointers must be 16-byte aligned");
  const int NC = attn_tc::dp_chunks(D), Tt = (T + 127) / 128;
  const long long total = (long long)B * T * 3 * H * (D / 8);
  long long g = (total + 255) / 256;
  const long long cap = (long long)sm_count() * 16;
  launch_k(attn_tc::pack_kernel, (int)(g < cap ? (g < 1 ? 1 : g) : cap), 256, 0, st, Q, K, V, tiles, B, T, H, D, NC, Tt, sq_b,
                                                                               sq_t, sq_h, sk_b, sk_t, sk_h, sv_b,
                                                                               sv_t, sv_h);
  return check_launch("vt_attn_pack");
}

// O[b, t, h, :D] = softmax(Q K^T * scale) V from attention tiles (tcgen05).  O element (b,t,h,d) at
// O + b*so_b + t*so_t + h*so_h + d; so_* multiples of 8, O 16-byte aligned.
int vt_attn_tiles_fwd(cudaStream_t st, const uint16_t* tiles, uint16_t* O, int B, int T, int H, int D, long long so_b,
                      long long so_t, long long so_h, float scale) {
  using namespace vt;
  if (B < 0 || T < 0 || H < 0) return set_error(E_SHAPE, "vt_attn_tiles_fwd: negative shape");
  if (B == 0 || T == 0 || H == 0) return OK;
  if (H > 65535) return set_error(E_SHAPE, "vt_attn_tiles_fwd: H=%d too large", H);
  if (D <= 0 || D % 8 || D > 80) return set_error(E_VARIANT, "vt_attn_tiles_fwd: head_dim %d unsupported", D);
  if (!tiles || !O || !aligned16(tiles) || !aligned16(O) || (so_b | so_t | so_h) % 8)
    return set_error(E_SHAPE, "vt_attn_tiles_fwd: pointers / strides not 16-byte aligned");
  attn_tc::Args a{tiles, O, T, H, D, (T + 127) / 128, so_b, so_t, so_h, scale * 1.4426950408889634f, 0};
  // Fewer 128-query CTAs than two per SM: with 16 or more key tiles (a TAPNext frame: 10 query tiles x 12 heads,
  // 20 key tiles) the keys of each query tile split over a cluster of two CTAs (14.3 against 19.7 us per launch);
  // else, or with VT_ATTN_KSPLIT=0 (A/B switch), 64-query CTAs (M = 64 MMAs), so that two share each SM (config 3
  // 1.220 -> 1.211 ms per frame against 128-query CTAs).  The split would also be faster for one or two tower crops
  // (13.2 / 21.3 against 13.6 / 23.5 us) and the text prefill (18.9 against 22.0 us), but it sums a row in another
  // order than the unsplit kernel, and tower crops (12 key tiles) must give the same bits whatever batch they run
  // in (a 130-crop chunk, a 13-crop frame, a frame sharded over GPUs), so the choice never splits them
  static const int ksplit = [] {
    const char* e = getenv("VT_ATTN_KSPLIT");
    return e ? atoi(e) : 1;
  }();
  const bool few = (long long)a.Tt * H * B < 2LL * sm_count();
  const bool split = few && ksplit && (T + 63) / 64 >= 16;
  if (attn_tc::dp_chunks(D) == 8)
    return split ? attn_tc::launch_nc<8, 128, 2>(st, a, B)
                 : few ? attn_tc::launch_nc<8, 64, 1>(st, a, B) : attn_tc::launch_nc<8, 128, 1>(st, a, B);
  return split ? attn_tc::launch_nc<10, 128, 2>(st, a, B)
               : few ? attn_tc::launch_nc<10, 64, 1>(st, a, B) : attn_tc::launch_nc<10, 128, 1>(st, a, B);
}

}  // extern "C"
