// Text-decoder kernels for the tower's consumer (FastMD2._text_layers, moondream/gpu/md2fast.py:169-199):
//   rope_qkv_kernel     rotary embedding of q and k (md2fast.py:162-167) and the KV-cache write of k and v
//                       (md2fast.py:190-191): the unfused equivalent of the reference's fused rope_cache
//   attn_causal_kernel  attention of n new tokens at positions pos0 .. pos0+n-1 over the cache with the
//                       question mask (md2fast.py:132-136: position p sees keys 0 .. p), for the question prefill
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

// One warp per (head h, new token i), two warps per CTA: scores over keys 0 .. pos0 + i with lane = key
// stride 32 (full 64-dim dots from the cache rows), softmax in fp32, then P.V with the same key split -- each
// lane a full 64-dim partial output over its keys -- and the 32 partials summed through shared memory.
// out [n][H*64].
constexpr int AW = 2;  // warps per CTA
__global__ void __launch_bounds__(AW * 32) attn_causal_kernel(const uint16_t* __restrict__ q,
                                                             const uint16_t* __restrict__ kc,
                                                             const uint16_t* __restrict__ vc, int n, int H, int pos0,
                                                             int ctx, float scale, uint16_t* __restrict__ out,
                                                             long long ldo) {
  __shared__ float p_s[AW][MAX_CTX];
  __shared__ float red[AW][32][HD + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wi = blockIdx.x * AW + warp;
  if (wi >= n * H) return;
  const int h = wi % H, i = wi / H;
  const int nk = pos0 + i + 1;  // keys 0 .. pos0 + i
  float qv[HD];
  const uint16_t* qr = q + ((size_t)h * n + i) * HD;
#pragma unroll
  for (int d = 0; d < HD; d += 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(qr + d);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      qv[d + 2 * e] = __uint_as_float(w[e] << 16) * scale;
      qv[d + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u) * scale;
    }
  }
  float* ps = p_s[warp];
  float mx = -INFINITY;
  for (int j = lane; j < nk; j += 32) {
    const uint16_t* kr = kc + ((size_t)h * ctx + j) * HD;
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < HD; d += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        s = fmaf(qv[d + 2 * e], __uint_as_float(w[e] << 16), s);
        s = fmaf(qv[d + 2 * e + 1], __uint_as_float(w[e] & 0xffff0000u), s);
      }
    }
    ps[j] = s;
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int d = 0; d < HD; d++) qv[d] = 0.f;  // reused as this lane's partial output
  for (int j = lane; j < nk; j += 32) {
    const float p = expf(ps[j] - mx);
    sum += p;
    const uint16_t* vr = vc + ((size_t)h * ctx + j) * HD;
#pragma unroll
    for (int d = 0; d < HD; d += 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(vr + d);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        qv[d + 2 * e] = fmaf(p, __uint_as_float(w[e] << 16), qv[d + 2 * e]);
        qv[d + 2 * e + 1] = fmaf(p, __uint_as_float(w[e] & 0xffff0000u), qv[d + 2 * e + 1]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int d = 0; d < HD; d++) red[warp][lane][d] = qv[d];
  __syncwarp();
  float o0 = 0.f, o1 = 0.f;
#pragma unroll 8
  for (int l = 0; l < 32; l++) {
    o0 += red[warp][l][2 * lane];
    o1 += red[warp][l][2 * lane + 1];
  }
  const float inv = 1.f / sum;
  *reinterpret_cast<uint32_t*>(out + (size_t)i * ldo + (size_t)h * HD + 2 * lane) = pack_bf2(o0 * inv, o1 * inv);
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
  text::rope_qkv_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(qkv, ld, n, H, pos0, cos_t, sin_t, q, kc,
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
  const int warps = n * H;
  text::attn_causal_kernel<<<(warps + text::AW - 1) / text::AW, text::AW * 32, 0, st>>>(q, kc, vc, n, H, pos0, ctx,
                                                                                      scale, out, ldo);
  return check_launch("vt_attn_causal");
}

}  // extern "C"
