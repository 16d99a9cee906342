// Host helpers of libvt_b200.so: error strings, the device status word, SM count and the
// cuTensorMapEncodeTiled entry point (fetched through the runtime, so no libcuda link is needed).
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <set>
#include <utility>

#include "vt_common.cuh"
#include "vt_host.h"

namespace vt {

static thread_local char g_err[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(E_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return OK;
}

int sm_count() {
  static std::atomic<int> cache[64];  // zero-initialised (static storage); 0 = not looked up yet
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int c = cache[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    c = n > 0 ? n : 148;
    cache[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

int smem_attr_once(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(E_LAUNCH, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return set_error(E_LAUNCH, "%s: setting %d bytes of dynamic shared memory: %s", what, bytes, cudaGetErrorString(e));
  done.insert({kernel, dev});
  return OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("VT_PDL");
    return e ? atoi(e) != 0 : true;
  }();
  return on;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_bf16(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                   uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(E_TMAP, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base) || (ld_elems * 2) % 16 != 0)
    return set_error(E_SHAPE, "tensor map: base %p / row pitch %llu elements not 16-byte aligned", base,
                     (unsigned long long)ld_elems);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = (box_cols * 2 == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(E_TMAP, "cuTensorMapEncodeTiled failed (%d): cols %llu rows %llu ld %llu box %ux%u", (int)r,
                     (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)ld_elems, box_cols,
                     box_rows);
  return OK;
}

// The same over an int8 matrix [rows][ld] (K-contiguous), box_cols = 128 (one 128-byte swizzle row).
int make_tmap_i8(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems, uint32_t box_cols,
                 uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(E_TMAP, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base) || ld_elems % 16 != 0 || box_cols != 128)
    return set_error(E_SHAPE, "tensor map: int8 base %p / row pitch %llu not 16-byte aligned", base,
                     (unsigned long long)ld_elems);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(E_TMAP, "cuTensorMapEncodeTiled (int8) failed (%d): cols %llu rows %llu ld %llu box %ux%u",
                     (int)r, (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)ld_elems,
                     box_cols, box_rows);
  return OK;
}

// 2-D tensor map over a row-major bf16 (elem_bytes 2) or fp32 (4) matrix [rows][ld], box = box_cols x
// box_rows, with the given swizzle (for epilogue staging boxes: the box's row is 64 or 128 bytes).
int make_tmap_epi(CUtensorMap* m, const void* base, int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                  uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(E_TMAP, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base) || (ld_elems * elem_bytes) % 16 != 0)
    return set_error(E_SHAPE, "tensor map: base %p / row pitch %llu elements not 16-byte aligned", base,
                     (unsigned long long)ld_elems);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(m, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(E_TMAP, "cuTensorMapEncodeTiled failed (%d): cols %llu rows %llu ld %llu box %ux%u", (int)r,
                     (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)ld_elems, box_cols,
                     box_rows);
  return OK;
}

}  // namespace vt

extern "C" {

const char* vt_last_error_string(void) { return vt::g_err; }

// Reads (and optionally clears) the device status word of the current device.  Synchronises the
// device.  Returns 0 when no kernel has recorded a timed-out wait.
int vt_device_status(int clear, unsigned int* status) {
  unsigned int s = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&s, vt::g_status, sizeof(s));
  if (e != cudaSuccess) return vt::set_error(vt::E_LAUNCH, "vt_device_status: %s", cudaGetErrorString(e));
  if (clear) {
    unsigned int z = 0;
    e = cudaMemcpyToSymbol(vt::g_status, &z, sizeof(z));
    if (e != cudaSuccess) return vt::set_error(vt::E_LAUNCH, "vt_device_status: %s", cudaGetErrorString(e));
  }
  if (status) *status = s;
  return 0;
}

int vt_abi_version(void) { return 1; }

}  // extern "C"

namespace vt {
// The bounded-wait protocol every kernel uses, run on two barriers that nothing completes: thread 0 waits with
// `cycles` as its limit and gives up (abort flag and status bit set), thread 32 waits with the kernels' own
// limit (kSpinCycles, ~2 s) and must leave as soon as it sees the abort flag.  result[0 / 1] = what the two
// waits returned (0: gave up).
__global__ void wait_selftest_kernel(long long cycles, int* result) {
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) result[0] = mbar_wait_for(&bar[0], 0, &abort_flag, ST_SELFTEST, cycles) ? 1 : 0;
  if (threadIdx.x == 32) result[1] = mbar_wait(&bar[1], 0, &abort_flag, ST_SELFTEST) ? 1 : 0;
}
}  // namespace vt

extern "C" {

// Failure detection without a fault: runs the bounded-wait protocol on barriers nothing completes (see
// wait_selftest_kernel).  result: 2 ints of device memory.  1000 <= cycles <= 1e9.
int vt_wait_selftest(cudaStream_t st, long long cycles, int* result) {
  using namespace vt;
  if (!result || cycles < 1000 || cycles > 1000000000LL)
    return set_error(E_SHAPE, "vt_wait_selftest: result must be non-null and 1000 <= cycles <= 1e9");
  wait_selftest_kernel<<<1, 64, 0, st>>>(cycles, result);
  return check_launch("vt_wait_selftest");
}

}  // extern "C"
