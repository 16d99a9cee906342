// The frame squash of FastMD2.set_image on the GPU (moondream/gpu/md2fast.py:223-228: Pillow's LANCZOS resize to
// 378 x 378 on the host): Pillow's two-pass fixed-point resampling restated, so the result equals Pillow's bit
// for bit.  The per-size weight tables (22 fraction bits) are computed on the host (imgproc.py).
//   resize_pass_kernel: one thread per output sample; acc = 2^21 + sum(pixel * weight), out = clip(acc >> 22)
#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {
namespace rsz {

constexpr int PREC = 22;

// Pass along one axis: out[o, j, c] (o < n_out output positions on the resampled axis, j < n_other along the
// other axis, c < 3) = clip8(sum_k in[x0(o) + k, j, c] * w[o][k]).  Element (a, b, c) of the input -- a on the
// resampled axis, b on the other -- is at in + a * sa + b * sb + c * sc (byte strides); the output likewise.
__global__ void resize_pass_kernel(const uint8_t* __restrict__ in, long long sa, long long sb, long long sc,
                                   uint8_t* __restrict__ out, long long oa, long long ob, long long oc, int n_out,
                                   int n_other, const int* __restrict__ bounds, const int* __restrict__ w, int ksize) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= (long long)n_out * n_other * 3) return;
  const int c = (int)(t % 3);
  const int j = (int)((t / 3) % n_other);
  const int o = (int)(t / (3LL * n_other));
  const int x0 = bounds[2 * o], n = bounds[2 * o + 1];
  const int* wk = w + (size_t)o * ksize;
  const uint8_t* p = in + (long long)x0 * sa + (long long)j * sb + (long long)c * sc;
  int acc = 1 << (PREC - 1);
  for (int k = 0; k < n; k++) acc += (int)p[(long long)k * sa] * wk[k];
  int v = acc >> PREC;
  v = v < 0 ? 0 : (v > 255 ? 255 : v);
  out[(long long)o * oa + (long long)j * ob + (long long)c * oc] = (uint8_t)v;
}

}  // namespace rsz
}  // namespace vt

extern "C" {

int vt_resize_pass_u8(cudaStream_t st, const uint8_t* in, long long sa, long long sb, long long sc, uint8_t* out,
                      long long oa, long long ob, long long oc, int n_out, int n_other, const int* bounds,
                      const int* weights, int ksize) {
  using namespace vt;
  if (n_out < 0 || n_other < 0 || ksize <= 0) return set_error(E_SHAPE, "vt_resize_pass_u8: bad shape");
  if ((long long)n_out * n_other == 0) return OK;
  if (!in || !out || !bounds || !weights) return set_error(E_SHAPE, "vt_resize_pass_u8: null pointer");
  const long long n = (long long)n_out * n_other * 3;
  launch_k(rsz::resize_pass_kernel, (unsigned)((n + 255) / 256), 256, 0, st, in, sa, sb, sc, out, oa, ob, oc, n_out, n_other,
                                                                      bounds, weights, ksize);
  return check_launch("vt_resize_pass_u8");
}

}  // extern "C"
