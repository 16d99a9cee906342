// Text-decoder kernels for the tower's consumer (FastMD2._text_layers, moondream/gpu/md2fast.py:169-199):
//   rope_qkv_kernel     rotary embedding of q and k (md2fast.py:162-167) and the KV-cache write of k and v
//                       (md2fast.py:190-191): the unfused equivalent of the reference's fused rope_cache
//   attn_causal_kernel  attention of n new tokens at positions pos0 .. pos0+n-1 over the cache with the
//                       question mask (md2fast.py:132-136: position p sees keys 0 .. p), for the question prefill;
//                       one CTA per (head, 8 new tokens), so each cache row is read once per group
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace text {

constexpr int HD = 64, ROT = 32, MAX_CTX = 2048;  // moondream2 context: 2048 positions

// qkv [n][3*H*64] bf16 (q | k | v, head-major); thread = (token r, head h, pair i < 32):
//   i < 16: q / k dims i and 16 + i rotate into the interleaved pair 2i, 2i+1; i >= 16: dims 2i, 2i+1 pass.
//   v dims 2i, 2i+1 are copied.  q -> qo[h][r][64]; k, v -> kc / vc[h][pos0 + r][64].
__global__ void rope_qkv_kernel(const uint16_t* __restrict__ qkv, long long ld, int n, int H, int pos0,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t, uint16_t* __restrict__ qo,
                                uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int ctx) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= (long long)n * H * 32) return;
  const int i = (int)(t % 32), h = (int)((t / 32) % H), r = (int)(t / (32LL * H));
  const uint16_t* row = qkv + (size_t)r * ld;
  const int pos = pos0 + r;
  const size_t oq = ((size_t)h * n + r) * HD + 2 * i, oc = ((size_t)h * ctx + pos) * HD + 2 * i;
  for (int w = 0; w < 2; w++) {  // q, k
    const uint16_t* x = row + (size_t)w * H * HD + (size_t)h * HD;
    uint32_t o;
    if (i < ROT / 2) {
      const float a = bf2f(x[i]), b = bf2f(x[ROT / 2 + i]);
      const float c = cos_t[pos * (ROT / 2) + i], s = sin_t[pos * (ROT / 2) + i];
      o = pack_bf2(a * c - b * s, a * s + b * c);
    } else {
      o = *reinterpret_cast<const uint32_t*>(x + 2 * i);
    }
    *reinterpret_cast<uint32_t*>((w == 0 ? qo + oq : kc + oc)) = o;
  }
  *reinterpret_cast<uint32_t*>(vc + oc) = *reinterpret_cast<const uint32_t*>(row + (size_t)2 * H * HD + (size_t)h * HD + 2 * i);
}

// CTA = (head h, group of QG consecutive new tokens), 8 warps.  The group's tokens share the cache rows, so
// each K and V row is read once per CTA:
//   scores   thread = key j (stride CT): its K row (128 B) against the QG scaled q rows (shared memory,
//            broadcast reads); token i sees keys 0 .. pos0 + i, later keys get -inf;
//   softmax  warp w = token w of the group: max and exp over its keys in fp32 (expf), row sum;
//   P.V      thread = (key slice w = warp, dim pair 2*lane): every 8th key, QG x 2 accumulators; the 8
//            slices are summed through shared memory and scaled by 1 / sum.
// Dynamic shared memory: qs [QG][64] | ps [QG][nkp] | red [8][QG][64] | lsum [QG] (fp32).
constexpr int QG = 8, CT = 256;
__host__ __device__ constexpr int causal_smem_floats(int nkp) { return QG * HD + QG * nkp + 8 * QG * HD + QG; }

__global__ void __launch_bounds__(CT) attn_causal_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                                                         const uint16_t* __restrict__ vc, int n, int H, int pos0, int ctx,
                                                         int nkp, float scale, uint16_t* __restrict__ out,
                                                         long long ldo) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  extern __shared__ float smf[];
  const int h = blockIdx.x, g0 = blockIdx.y * QG;
  const int nq = min(QG, n - g0);
  const int nk = pos0 + g0 + nq;  // keys the group's last token sees
  float* qs = smf;
  float* ps = qs + QG * HD;
  float* red = ps + QG * nkp;
  float* lsum = red + 8 * QG * HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < QG * HD; e += CT) {
    const int qi = e / HD;
    qs[e] = qi < nq ? bf2f(q[((size_t)h * n + g0 + qi) * HD + e % HD]) * scale : 0.f;
  }
  __syncthreads();
  for (int j = tid; j < nk; j += CT) {
    const uint16_t* kr = kc + ((size_t)h * ctx + j) * HD;
    float sc[QG];
#pragma unroll
    for (int qi = 0; qi < QG; qi++) sc[qi] = 0.f;
#pragma unroll
    for (int d = 0; d < HD; d += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      float kv[8];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        kv[2 * e] = __uint_as_float(w[e] << 16);
        kv[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
      }
#pragma unroll
      for (int qi = 0; qi < QG; qi++) {
        const float4 qa = *reinterpret_cast<const float4*>(qs + qi * HD + d);
        const float4 qb = *reinterpret_cast<const float4*>(qs + qi * HD + d + 4);
        float t = sc[qi];
        t = fmaf(qa.x, kv[0], t);
        t = fmaf(qa.y, kv[1], t);
        t = fmaf(qa.z, kv[2], t);
        t = fmaf(qa.w, kv[3], t);
        t = fmaf(qb.x, kv[4], t);
        t = fmaf(qb.y, kv[5], t);
        t = fmaf(qb.z, kv[6], t);
        t = fmaf(qb.w, kv[7], t);
        sc[qi] = t;
      }
    }
#pragma unroll
    for (int qi = 0; qi < QG; qi++) ps[qi * nkp + j] = j <= pos0 + g0 + qi ? sc[qi] : -INFINITY;
  }
  __syncthreads();
  {  // softmax of token `warp` of the group (rows past nq see keys up to nk too; they are never stored)
    float* pr = ps + warp * nkp;
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, pr[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < nk; j += 32) {
      const float p = expf(pr[j] - mx);
      pr[j] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) lsum[warp] = sum;
  }
  __syncthreads();
  float acc[QG][2];
#pragma unroll
  for (int qi = 0; qi < QG; qi++) acc[qi][0] = acc[qi][1] = 0.f;
  // 8 of this slice's keys per round: their V loads are issued together, then consumed
  for (int j0 = warp; j0 < nk; j0 += 64) {
    uint32_t v2[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int j = j0 + 8 * u;
      v2[u] = j < nk ? *reinterpret_cast<const uint32_t*>(vc + ((size_t)h * ctx + j) * HD + 2 * lane) : 0u;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int j = j0 + 8 * u;
      if (j >= nk) break;
      const float vx = __uint_as_float(v2[u] << 16), vy = __uint_as_float(v2[u] & 0xffff0000u);
#pragma unroll
      for (int qi = 0; qi < QG; qi++) {
        const float p = ps[qi * nkp + j];
        acc[qi][0] = fmaf(p, vx, acc[qi][0]);
        acc[qi][1] = fmaf(p, vy, acc[qi][1]);
      }
    }
  }
#pragma unroll
  for (int qi = 0; qi < QG; qi++)
    *reinterpret_cast<float2*>(red + (warp * QG + qi) * HD + 2 * lane) = make_float2(acc[qi][0], acc[qi][1]);
  __syncthreads();
  if (warp < nq) {  // token g0 + warp, dims 2*lane, 2*lane+1
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int sl = 0; sl < 8; sl++) {
      const float2 r = *reinterpret_cast<const float2*>(red + (sl * QG + warp) * HD + 2 * lane);
      o0 += r.x;
      o1 += r.y;
    }
    const float inv = 1.f / lsum[warp];
    *reinterpret_cast<uint32_t*>(out + (size_t)(g0 + warp) * ldo + (size_t)h * HD + 2 * lane) =
        pack_bf2(o0 * inv, o1 * inv);
  }
}

}  // namespace text
}  // namespace vt

extern "C" {

int vt_rope_qkv(cudaStream_t st, const uint16_t* qkv, long long ld, int n, int H, int pos0, const float* cos_t,
                const float* sin_t, uint16_t* q, uint16_t* kc, uint16_t* vc, int ctx) {
  using namespace vt;
  if (n < 0 || H <= 0 || pos0 < 0 || ctx <= 0 || pos0 + n > ctx)
    return set_error(E_SHAPE, "vt_rope_qkv: n=%d H=%d pos0=%d ctx=%d", n, H, pos0, ctx);
  if (n == 0) return OK;
  if (!qkv || !cos_t || !sin_t || !q || !kc || !vc || ld < 3LL * H * text::HD || ld % 2 ||
      (reinterpret_cast<uintptr_t>(qkv) & 3) || (reinterpret_cast<uintptr_t>(q) & 3) ||
      (reinterpret_cast<uintptr_t>(kc) & 3) || (reinterpret_cast<uintptr_t>(vc) & 3))
    return set_error(E_SHAPE, "vt_rope_qkv: null pointer, pitch or alignment invalid");
  const long long threads = (long long)n * H * 32;
  launch_k(text::rope_qkv_kernel, (unsigned)((threads + 255) / 256), 256, 0, st, qkv, ld, n, H, pos0, cos_t, sin_t, q, kc,
                                                                          vc, ctx);
  return check_launch("vt_rope_qkv");
}

int vt_attn_causal(cudaStream_t st, const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int n, int H, int pos0,
                   int ctx, float scale, uint16_t* out, long long ldo) {
  using namespace vt;
  if (n < 0 || H <= 0 || pos0 < 0 || ctx <= 0 || pos0 + n > ctx || ctx > text::MAX_CTX)
    return set_error(E_SHAPE, "vt_attn_causal: n=%d H=%d pos0=%d ctx=%d (ctx <= %d)", n, H, pos0, ctx, text::MAX_CTX);
  if (n == 0) return OK;
  if (!q || !kc || !vc || !out || ldo < (long long)H * text::HD || ldo % 2 || !aligned16(q) || !aligned16(kc) ||
      !aligned16(vc) || (reinterpret_cast<uintptr_t>(out) & 3))
    return set_error(E_SHAPE, "vt_attn_causal: null pointer, pitch or alignment invalid");
  if (H > 65535 || (n + text::QG - 1) / text::QG > 65535)
    return set_error(E_SHAPE, "vt_attn_causal: grid too large (H=%d, n=%d)", H, n);
  const int arc = smem_attr_once((const void*)text::attn_causal_kernel, text::causal_smem_floats(text::MAX_CTX) * 4,
                                 "vt_attn_causal");
  if (arc) return arc;
  const int nkp = (pos0 + n + 3) & ~3;  // row pitch of the score rows (floats), 16-byte multiple
  launch_k(text::attn_causal_kernel, dim3(H, (n + text::QG - 1) / text::QG), text::CT, text::causal_smem_floats(nkp) * 4, st, 
      q, kc, vc, n, H, pos0, ctx, nkp, scale, out, ldo);
  return check_launch("vt_attn_causal");
}

}  // extern "C"
