// Host-side helpers shared by the .cu files of libvt_b200.so (not part of the public C ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vt {

// Error codes, same convention as the reference's launchers (0 ok, -1 unknown variant,
// -2 shape / alignment, -4 layout mismatch), plus -3 for a CUDA launch error and -5 for a
// tensor-map encode failure.
enum : int { OK = 0, E_VARIANT = -1, E_SHAPE = -2, E_LAUNCH = -3, E_LAYOUT = -4, E_TMAP = -5 };

int set_error(int code, const char* fmt, ...);   // records the message for vt_last_error_string()

// Programmatic dependent launch: every kernel of the library is launched with the attribute that lets it
// start (prologue: barriers, TMEM, descriptor prefetch) while the previous kernel in the stream finishes;
// each kernel executes griddepcontrol.wait (griddep_wait) before its first global-memory access, so no
// kernel reads or writes memory before its predecessor has completed.  VT_PDL=0 turns the attribute off.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}
int check_launch(const char* what);              // maps cudaGetLastError() to E_LAUNCH
// Sets a kernel's maximum dynamic shared memory on the current device the first time (kernel, device) is seen;
// safe to call from several host threads at once; E_LAUNCH with the CUDA error's message if it fails.
int smem_attr_once(const void* kernel, int bytes, const char* what);
int sm_count();                                  // SMs of the current device (cached per device)
bool aligned16(const void* p);

// 2-D bf16 tensor map over a row-major matrix [rows][ld] (K-contiguous), box = box_cols x box_rows,
// 128-byte swizzle when box_cols * 2 == 128, zero fill out of bounds.  Returns E_TMAP on failure.
int make_tmap_bf16(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                   uint32_t box_cols, uint32_t box_rows);
// The same over an int8 matrix (pitch in bytes, a multiple of 16), box 128 x box_rows, 128-byte swizzle.
int make_tmap_i8(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_elems, uint32_t box_cols,
                 uint32_t box_rows);
// The same for epilogue boxes: bf16 (elem_bytes 2) or fp32 (4), swizzle 0, 64 or 128 bytes.
int make_tmap_epi(CUtensorMap* m, const void* base, int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_elems,
                  uint32_t box_cols, uint32_t box_rows, int swizzle_bytes);

}  // namespace vt
