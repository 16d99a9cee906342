// Single translation unit of libvt_b200.so.  The kernels share one device status word
// (vt::g_status), so they are compiled together rather than linked with relocatable device code.
#include "host_common.cu"
#include "gemm_tc.cu"
#include "quant.cu"
#include "attn_tc.cu"
#include "attn_noalloc.cu"
#include "elementwise.cu"
#include "ssm.cu"
#include "text.cu"
#include "resize.cu"
#include "heads.cu"
