// Attention for callers that cannot allocate device memory.
//
// vt_attn_fwd_noalloc computes what vt_attn_pack followed by vt_attn_tiles_fwd computes, but the
// attention tiles those two kernels pass between them live in a fixed array compiled into this library
// instead of a buffer the caller allocates.  Some callers have no way to allocate device memory at the
// point where they need attention:
//   * hosts that plan their whole device-memory budget at start-up and forbid allocation afterwards,
//     such as inference servers that give each model a fixed share of the GPU's memory and must not
//     grow past it while serving;
//   * plain C or FFI callers (a ctypes / cgo / JNI binding without torch) that have no device
//     allocator of their own to hand out a scratch buffer.
// They pass only Q, K, V and O, all of which they own.
//
// Limits and rules:
//   * the scratch holds at most kScratchBytes = 16 MiB of attention tiles: two crops of the vision
//     tower (16 heads x 729 tokens x head_dim 72) or one TAPNext frame (12 heads x 1280 x 64);
//     larger problems are rejected with E_SHAPE (use vt_attn_pack + vt_attn_tiles_fwd with a buffer of
//     vt_attn_tiles_bytes(...) bytes instead);
//   * every GPU that loads this library holds the 16 MiB until the process exits;
//   * every call shares the one array, which keeps what the last call wrote.  A call first writes zeros
//     into the pad rows and lanes of the part it uses (the attention kernel reads them and they must be
//     zero; vt_attn_pack then writes every other element), so what an earlier call left there does not
//     matter.  Calls that overlap on the GPU -- on streams without ordering between them, or from several
//     host threads -- race on the array;
//   * the first call on a device does its set-up with that device current: it looks up the array's
//     device address (cudaGetSymbolAddress) and sets the attention kernels' shared-memory attributes.
#include <mutex>

#include "vt_common.cuh"
#include "vt_host.h"

extern "C" long long vt_attn_tiles_bytes(int B, int T, int H, int D);
extern "C" int vt_attn_pack(cudaStream_t st, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* tiles,
                            int B, int T, int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b,
                            long long sk_t, long long sk_h, long long sv_b, long long sv_t, long long sv_h);
extern "C" int vt_attn_tiles_fwd(cudaStream_t st, const uint16_t* tiles, uint16_t* O, int B, int T, int H, int D,
                                 long long so_b, long long so_t, long long so_h, float scale);
namespace vt {
namespace attn_tc {
int prepare_device();
}
}  // namespace vt

namespace vt {
namespace noalloc {

constexpr long long kScratchBytes = 16LL << 20;
static __device__ __align__(256) uint16_t g_attn_scratch[kScratchBytes / 2];

// Device address of g_attn_scratch on the current device.  In host code the name g_attn_scratch is only
// a host-side stand-in, never a device address, so the address is looked up once per device; the same
// one-time block sets the attention kernels' attributes (attn_tc::prepare_device), so that every set-up
// step of this entry point happens on its first call per device, whatever the head_dim of later calls.
static int scratch_address(uint16_t** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(E_LAUNCH, "vt_attn_fwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(E_LAUNCH, "vt_attn_fwd_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p)
      return set_error(E_LAUNCH, "vt_attn_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    const int rc = attn_tc::prepare_device();
    if (rc) return rc;
    addr[dev] = p;
  }
  *out = static_cast<uint16_t*>(addr[dev]);
  return OK;
}

// Zeros into the pad slots of the attention tiles of B crops: every 16-byte (8-element) chunk of a row
// t >= T or of a d chunk c >= D/8, for rows t < Tt*128 and chunks c < NC of every (crop, operand, head).
// vt_attn_pack writes all the other chunks, so the two kernels together define the whole buffer.
__global__ void __launch_bounds__(256) zero_pads_kernel(uint16_t* __restrict__ tiles, int B, int T, int H, int D,
                                                        int NC, int Tt) {
  griddep_wait();  // programmatic dependent launch: the previous kernel has completed
  griddep_launch();
  const int dch = D / 8, rows = Tt * 128;
  const long long per_op = (long long)rows * NC;
  const long long total = (long long)B * 3 * H * per_op;
  const size_t op_elems = (size_t)Tt * NC * 1024;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long op = i / per_op;  // (crop * 3 + operand) * H + head
    const int r = (int)(i % per_op);
    const int t = r / NC, c = r % NC;
    if (t < T && c < dch) continue;
    const int w = (int)((op / H) % 3);
    *reinterpret_cast<uint4*>(tiles + (size_t)op * op_elems + attn_tile_off(w, t, c, NC)) = make_uint4(0, 0, 0, 0);
  }
}

}  // namespace noalloc
}  // namespace vt

extern "C" {

// Attention with no device allocation: O[b,t,h,:D] = softmax(Q K^T * scale) V, strides as vt_attn_pack /
// vt_attn_tiles_fwd; the attention tiles live in the library's fixed 16 MiB scratch (see above).
int vt_attn_fwd_noalloc(cudaStream_t st, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int B,
                        int T, int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b,
                        long long sk_t, long long sk_h, long long sv_b, long long sv_t, long long sv_h,
                        long long so_b, long long so_t, long long so_h, float scale) {
  using namespace vt;
  if (B < 0 || T < 0 || H < 0) return set_error(E_SHAPE, "vt_attn_fwd_noalloc: negative shape");
  if (B == 0 || T == 0 || H == 0) return OK;
  const long long need = vt_attn_tiles_bytes(B, T, H, D);
  if (need <= 0) return set_error(E_VARIANT, "vt_attn_fwd_noalloc: head_dim %d unsupported (multiple of 8, <= 80)", D);
  if (need > noalloc::kScratchBytes)
    return set_error(E_SHAPE,
                     "vt_attn_fwd_noalloc: B=%d T=%d H=%d D=%d needs %lld bytes of attention tiles, more than the "
                     "fixed %lld-byte scratch; call vt_attn_pack + vt_attn_tiles_fwd with a caller-owned buffer",
                     B, T, H, D, need, noalloc::kScratchBytes);
  uint16_t* tiles = nullptr;
  int rc = noalloc::scratch_address(&tiles);
  if (rc) return rc;
  const int NC = D <= 64 ? 8 : 10, Tt = (T + 127) / 128;
  const long long slots = (long long)B * 3 * H * Tt * 128 * NC;
  const long long g = (slots + 255) / 256, cap = (long long)sm_count() * 16;
  launch_k(noalloc::zero_pads_kernel, (int)(g < cap ? g : cap), 256, 0, st, tiles, B, T, H, D, NC, Tt);
  rc = check_launch("vt_attn_fwd_noalloc (pad zeros)");
  if (rc) return rc;
  rc = vt_attn_pack(st, Q, K, V, tiles, B, T, H, D, sq_b, sq_t, sq_h, sk_b, sk_t, sk_h, sv_b, sv_t, sv_h);
  if (rc) return rc;
  return vt_attn_tiles_fwd(st, tiles, O, B, T, H, D, so_b, so_t, so_h, scale);
}

}  // extern "C"
