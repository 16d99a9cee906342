/* libvt_b200.so -- C ABI of the B200 (sm_100a) vision-tower kernels.
 *
 * Conventions (the reference's, moondream/gpu/hgemm.py:21-36, hattn.py:5-16):
 *   - every function takes the CUDA stream to launch on first (torch's current stream in the Python host)
 *     and raw device pointers; the caller owns every buffer; nothing is allocated, nothing synchronises
 *     (except vt_device_status);
 *   - bf16 tensors are passed as uint16_t*; pitches / strides are in elements;
 *   - return 0 on success, negative on error (-1 unknown variant, -2 shape or alignment, -3 CUDA launch
 *     error, -4 layout mismatch, -5 tensor-map encode failure), the message in vt_last_error_string().
 */
#ifndef VT_B200_H
#define VT_B200_H
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ABI version of this header (1). */
int vt_abi_version(void);

/* Message of the last failing call on this host thread. */
const char* vt_last_error_string(void);

/* Device status word of the current device: bit i set when a kernel's bounded wait gave up at site i
 * (the kernel then unwinds instead of hanging).  Synchronises the device; clear != 0 resets the word. */
int vt_device_status(int clear, unsigned int* status);

/* Failure detection without a GPU fault: one CTA runs the kernels' bounded-wait protocol on two mbarriers that
 * nothing completes.  Its thread 0 gives up after `cycles` SM cycles (1000 <= cycles <= 1e9), sets the CTA's
 * abort flag and status bit 8; its thread 32, waiting with the kernels' own ~2 s limit, must leave on the abort
 * flag.  result (2 ints, device memory) = what the two waits returned (0: gave up).
 * Replaces: nothing in the reference (its kernels have no bounded waits); checks the mechanism behind
 * vt_device_status. */
int vt_wait_selftest(cudaStream_t stream, long long cycles, int* result);

/* C[M,N] (bf16, pitch ldc) = A[M,K] . W[N,K]^T + bias (fp32, may be NULL), optional GELU-tanh applied
 * after rounding to bf16.  A, W bf16 K-contiguous, pitches multiples of 8, bases 16-byte aligned.
 * tcgen05/TMEM tiles fed by TMA.
 * Replaces: bf16gemm_launch, moondream/gpu/hip/i8gemm.hip:534 (called from HLin._run, hgemm.py:160-162);
 * no cfg / swap / packed arguments: one persistent kernel, weights in the natural (N, K) layout. */
int vt_gemm_bf16(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw,
                 const float* bias, uint16_t* C, long long ldc, int M, int N, int K, int gelu);

/* General GEMM epilogue: out (fp32 when out_f32, else bf16) = A.W^T + bias [+ res], res fp32 (bf16 when
 * res_bf16) read at row (m % res_period) when res_period > 0 (positional embedding) else row m; res may
 * alias out (in-place residual stream).  out2 (may be NULL) receives a bf16 copy of an fp32 output.
 * GELU only with bf16 output.
 * Replaces: bf16gemm_launch (i8gemm.hip:534) plus the unfused residual add of lin_res / mlp
 * (moondream/gpu/md2fast.py:55-67) and the pos_emb add of md2fast.py:150. */
int vt_gemm_ex(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M, int N,
               int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
               long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2);

/* Superset of vt_gemm_ex with the tower's LayerNorm fusions (NULL / 0 disables each):
 *   stats_out (fp32 output, N % 32 == 0): stats_out[m][j] = (mean, sum of squared deviations) of output row
 *     m over columns 32j..32j+31, float pairs [M][N/32] -- the row statistics of the new residual stream;
 *   ln_moments / ln_c: LayerNorm of the A rows folded into this GEMM: A holds x (bf16), W holds
 *     W * diag(gamma), ln_c[n] = sum_k W[n][k] (of the bf16 W), bias holds b + W beta, and the epilogue
 *     computes rstd * (acc - mean * ln_c[n]) + bias with (mean, rstd) = ln_moments[m] (vt_row_moments);
 *   tiles_T / tiles_H / tiles_D > 0: bf16 output scattered into the attention-tile layout (N = 3*H*D).
 * Replaces: the pre-LN + linear pairs of md2fast.py:153-154 and 157 (_ln then qkv / fc1) plus the residual
 * epilogues of md2fast.py:156-157, with the LayerNorm's row statistics produced by the GEMM that writes
 * the residual stream instead of a separate F.layer_norm pass. */
int vt_gemm_fused(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M,
                  int N, int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
                  long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2, float* stats_out,
                  const float* ln_moments, const float* ln_c, int tiles_T, int tiles_H, int tiles_D);

/* Bytes of the workspace vt_gemm_fused_ws takes for an M x N output (0 for an empty one). */
long long vt_gemm_ws_bytes(int M, int N);

/* vt_gemm_fused with a caller-owned workspace (16-byte aligned, >= vt_gemm_ws_bytes(M, N) bytes, zero-filled
 * once when allocated; one workspace sized for the largest M x N serves calls of every smaller shape, one
 * at a time).  With it, a GEMM too small to occupy the GPU with 128 x 64 tiles -- few output columns at
 * small M, e.g. the text decoder's 32-token question -- splits K across CTAs: each stores its fp32 partial
 * sum in the workspace and the last to finish a row chunk adds them in slice order and runs the epilogue,
 * so results are deterministic (equal to vt_gemm_fused's up to fp32 summation order).  ws = NULL is
 * vt_gemm_fused.  gelu = 2 here (and in vt_gemm_fused_lnstats) is the gated GELU of a gated MLP: W's rows are
 * [gate | up] pairs interleaved in blocks of 16 (rows 32c .. 32c+15 gate channels 16c .., rows 32c+16 .. the
 * matching up channels), N % 32 == 0, and the bf16 output has N / 2 columns, out[m][16c + i] =
 * bf16(bf16(gelu_tanh(gate)) * up) of the bf16-rounded linear outputs (no residual, tiles or statistics).
 * Replaces: the same call sites as vt_gemm_fused (here the question prefill's linears, md2fast.py:192-199);
 * the reference's HIP GEMM has no split-K variant; with gelu = 2, ffw_up followed by the gated GELU product of
 * the TAPNext++ MLP (tapnext/npu/step8.py:482-483, mm8.cc:937-960). */
int vt_gemm_fused_ws(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw, int M,
                     int N, int K, const float* bias, void* out, long long ldo, int out_f32, int gelu, const void* res,
                     long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2, float* stats_out,
                     const float* ln_moments, const float* ln_c, int tiles_T, int tiles_H, int tiles_D, void* ws,
                     long long ws_bytes);

/* vt_gemm_fused_ws whose folded norm takes its row factors straight from the 32-column chunk statistics that
 * the last writer of the A rows left (a stats_out of an earlier call): ln_stats [M][ln_nchunk] (mean, M2) float
 * pairs, merged in this GEMM's epilogue as vt_row_moments does (ln_rms != 0: as vt_row_rms does, an RMSNorm
 * with mean 0), so the separate row-moment pass and its launch go away.  ln_mom_out [M] (may be NULL)
 * receives the (mean, rstd) pairs for a later kernel.  Every other argument as for vt_gemm_fused_ws.
 * Replaces: the same pre-norm + linear pairs as vt_gemm_fused with ln_moments (md2fast.py:153-154, 157; the
 * TAPNext++ block's norms before linear_yx / ffw_up / qkv / fc1, tapnext/npu/step8.py:474-486). */
int vt_gemm_fused_lnstats(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw,
                          int M, int N, int K, const float* bias, void* out, long long ldo, int out_f32, int gelu,
                          const void* res, long long ldr, int res_period, int res_bf16, uint16_t* out2, long long ldo2,
                          float* stats_out, const float* ln_stats, int ln_nchunk, float ln_eps, int ln_rms,
                          const float* ln_c, float* ln_mom_out, int tiles_T, int tiles_H, int tiles_D, void* ws,
                          long long ws_bytes);

/* Per-token int8 quantisation of the activation rows of a W8A8 GEMM: s[m] = max(max_k |x[m,k]|, 1e-5) / 127
 * and q[m,k] = trunc(x[m,k] / s[m] +- 0.5) (round half away from zero, IEEE fp32 division and addition),
 * from x bf16 [M, K] (pitch ldx elements, 16-byte aligned) into q int8 (pitch ldq bytes, 8-byte aligned);
 * K % 8 == 0, K <= 16384.
 * Replaces: quant_rows, moondream/gpu/hgemm.py:10-16 (its Triton kernel _quant_rows, tgemm.py:81-91), as
 * HI8Lin.quant (hgemm.py:116-117) and the shared quantisation of the LN output (md2fast.py:174) call it. */
int vt_quant_rows(cudaStream_t stream, const uint16_t* x, long long ldx, int M, int K, int8_t* q, long long ldq,
                  float* s);

/* vt_layernorm fused with vt_quant_rows of its bf16 output: the same q[M, N] (pitch ldq bytes, a multiple of
 * 4) and s[M], without the bf16 round trip through memory; y (bf16, pitch ldy) also receives the LayerNorm
 * output when not NULL.  N % 4 == 0, N <= 4096.
 * Replaces: _ln followed by HI8Lin.quant on its output, the shared activation of qkv and fc1
 * (moondream/gpu/md2fast.py:173-174). */
int vt_layernorm_quant(cudaStream_t stream, const void* x, long long ldx, int in_bf16, const float* gamma,
                       const float* beta, int M, int N, float eps, int8_t* q, long long ldq, float* s, uint16_t* y,
                       long long ldy);

/* W8A8 int8 GEMM on the tensor cores (tcgen05 kind::i8, exact int32 accumulation):
 *   out[m, n] = ((float)(A[m,:] . W[n,:]) * sa[m]) * sw[n] + bias[n],
 * GELU-tanh applied to that fp32 value when gelu != 0, then bf16 output (fp32 with out_f32, no GELU), plus
 * res (fp32, or bf16 with res_bf16; may alias out) when res != NULL.  A [M, K] and W [N, K] signed int8 with
 * pitches lda / ldw in bytes (multiples of 16, 16-byte aligned bases); sa [M] the activation scales
 * (vt_quant_rows), sw [N] the per-channel weight scales (16-byte aligned), bias [N] fp32 or NULL.  ws / ws_bytes
 * as for vt_gemm_fused_ws (the split-K partial sums are int32, so the result does not depend on the split).
 * Replaces: i8gemm_launch / i8gemm_small_launch, moondream/gpu/hip/i8gemm.hip:480-533 and 555-593 (the
 * kernel epilogue i8gemm.hip:183-197), as HI8Lin.__call__ runs them (moondream/gpu/hgemm.py:119-137). */
int vt_gemm_i8(cudaStream_t stream, const int8_t* A, long long lda, const int8_t* W, long long ldw, const float* sa,
               const float* sw, int M, int N, int K, const float* bias, void* out, long long ldo, int out_f32,
               int gelu, const void* res, long long ldr, int res_bf16, void* ws, long long ws_bytes);

/* Row statistics of x[M, N] fp32 (N % 32 == 0) in the stats_out format of vt_gemm_fused, and optionally the
 * bf16 copy xb: the LayerNorm inputs for a residual stream that no vt_gemm_fused epilogue produced.
 * Replaces: the statistics half of _ln, md2fast.py:43-44. */
int vt_rowstats(cudaStream_t stream, const float* x, long long ldx, uint16_t* xb, long long ldxb, float* stats, int M,
                int N);

/* moments[m] = (mean, rsqrt(var + eps)) of row m of a residual stream with N = 32*nchunk columns, from its
 * chunk statistics (float pairs [M][nchunk], as vt_rowstats / vt_gemm_fused stats_out write them), merged
 * with Chan's parallel formula; the ln_moments input of vt_gemm_fused.
 * Replaces: the statistics half of _ln, md2fast.py:43-44. */
int vt_row_moments(cudaStream_t stream, const float* stats, int M, int nchunk, float eps, float* moments);

/* Fused QKV projection for attention: A[M = crops*T, K] . W[3*H*D, K]^T + bias, bf16, written straight into
 * the attention-tile layout vt_attn_tiles_fwd reads (tiles: vt_attn_tiles_bytes(M/T, T, H, D) bytes,
 * zero-filled once at allocation).
 * Replaces: the qkv HLin call + chunk/view/transpose of md2fast.py:154 feeding hattn.Attn, whose V^T copy
 * (vtranspose, attn.hip:284) this layout makes unnecessary. */
int vt_gemm_qkv_tiles(cudaStream_t stream, const uint16_t* A, long long lda, const uint16_t* W, long long ldw,
                      const float* bias, uint16_t* tiles, int M, int K, int T, int H, int D);

/* Size in bytes of the attention-tile buffer for B crops x H heads x T tokens of head_dim D:
 * layout [B][q|k|v][H][ceil(T/128)][tile] bf16 with a Q tile [DP/8][128][8] and a K or V tile
 * [2][DP/8][64][8] (two 64-token halves), DP = 64 (D <= 64) or 80.  0 if unsupported. */
long long vt_attn_tiles_bytes(int B, int T, int H, int D);

/* Strided Q/K/V (element (b,t,h,d) at X + b*sx_b + t*sx_t + h*sx_h + d) -> attention tiles (zero-filled
 * once at allocation; pads are never written).
 * Replaces: vtranspose, moondream/gpu/hip/attn.hip:284 (the reference's pre-pass of hattn.Attn). */
int vt_attn_pack(cudaStream_t stream, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* tiles,
                 int B, int T, int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b,
                 long long sk_t, long long sk_h, long long sv_b, long long sv_t, long long sv_h);

/* tcgen05 flash attention from attention tiles: O[b,t,h,:D] = softmax(Q K^T * scale) V, S, P and O in TMEM;
 * O element (b,t,h,d) at O + b*so_b + t*so_t + h*so_h + d (strides multiples of 8).  Grids of fewer than two
 * 128-query tiles per SM with T > 960 split each query tile's keys over a cluster of two CTAs (results equal
 * within rounding, deterministic); for T <= 960 a row's result does not depend on B.
 * Replaces: attn_fwd2, moondream/gpu/hip/attn.hip:442 (hattn.Attn.__call__, hattn.py:26-37). */
int vt_attn_tiles_fwd(cudaStream_t stream, const uint16_t* tiles, uint16_t* O, int B, int T, int H, int D,
                      long long so_b, long long so_t, long long so_h, float scale);

/* Attention without any device allocation, for callers that cannot allocate device memory where they need
 * attention: hosts that fix their device-memory budget at start-up and allow no allocation while serving,
 * and plain C / FFI callers with no device allocator of their own.
 * Same result as vt_attn_pack + vt_attn_tiles_fwd (same strides and scale); the attention tiles live in a
 * fixed 16 MiB array inside the library (held by every GPU that loads it until exit), so problems needing
 * more than 16 MiB of tiles (vt_attn_tiles_bytes) return -2.  Every call shares the array, which keeps the
 * last call's contents; each call writes the zeros its pad rows and lanes need, and calls that overlap on
 * the GPU race on the array.  The first call on a device does the set-up (the array's device address and
 * the attention kernels' attributes) with that device current.
 * No counterpart in the reference (its attention always takes a caller-allocated V^T buffer). */
int vt_attn_fwd_noalloc(cudaStream_t stream, const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                        int B, int T, int H, int D, long long sq_b, long long sq_t, long long sq_h, long long sk_b,
                        long long sk_t, long long sk_h, long long sv_b, long long sv_t, long long sv_h,
                        long long so_b, long long so_t, long long so_h, float scale);

/* y = LayerNorm(x) * gamma + beta over rows of N (N % 4 == 0, N <= 4096); x fp32 (bf16 when in_bf16),
 * y bf16 (fp32 when out_f32); fp32 statistics.
 * Replaces: _ln / F.layer_norm, moondream/gpu/md2fast.py:43-44 (ln1, ln2, post_ln; md2fast.py:153-158). */
int vt_layernorm(cudaStream_t stream, const void* x, long long ldx, int in_bf16, const float* gamma,
                 const float* beta, void* y, long long ldy, int out_f32, int M, int N, float eps);

/* y = x * rsqrt(mean(x^2) + eps) * gamma (RMSNorm) over rows of N, layout rules of vt_layernorm.
 * Replaces: the temporal pre-norm (RMSNorm) of the TAPNext recurrent block, tapnext/npu/step8.py:474
 * (the NPU's "rms" EW op, tapnext/npu/pack8.py:115-121). */
int vt_rmsnorm(cudaStream_t stream, const void* x, long long ldx, int in_bf16, const float* gamma, void* y,
               long long ldy, int out_f32, int M, int N, float eps);

/* Patch im2col into A[B*(S/P)^2][C*P*P] (bf16, pitch ldo) with K order (c, py, px); pixel kinds:
 * 0 fp32 NCHW, 1 bf16 NCHW, 2 uint8 NHWC normalised (u/255 - 0.5)/0.5.
 * Replaces: the normalise + reshape/permute of moondream/gpu/md2fast.py:148-149. */
int vt_im2col(cudaStream_t stream, const void* pix, int kind, int B, int C, int S, int P, uint16_t* out,
              long long ldo);

/* Multi-crop combine: out[t] = [ f[0][t] , mean_{i=1..n-1} f[i][t] ] (bf16).
 * Replaces: the feature input of the projection, moondream/gpu/md2fast.py:159 (cat([x, x]) for one crop),
 * for the 13-crop frame of the benchmark configuration (global + mean of the local crops). */
int vt_crop_combine(cudaStream_t stream, const uint16_t* f, long long crop_stride, long long ldf, int n_crops, int T,
                    int W, uint16_t* out, long long ldo);

/* RMSNorm statistics for an RMSNorm folded into the GEMM after it: out[m] = (0, 1 / sqrt(mean over the row of
 * x^2 + eps)) from the per-32-column chunk statistics (mean, M2) [M][nchunk] that vt_rowstats or a residual
 * GEMM epilogue wrote; fp32.  The ln input of vt_gemm_fused then applies rstd * acc + bias (mean 0).
 * Replaces: the statistics half of the temporal pre-norm (RMSNorm), tapnext/npu/step8.py:474. */
int vt_row_rms(cudaStream_t stream, const float* stats, int M, int nchunk, float eps, float* out);

/* vt_rglru with the temporal RMSNorm folded into the gate GEMM before it: G = [gx_pre | ga_pre] fp32 from a GEMM
 * whose A was the bf16 copy of x and whose weights carry the RMSNorm gamma; the recurrence's input
 * t = bf16(x * rstd * gamma) is formed here from the fp32 stream x and rms_moments [M][2] (vt_row_rms).
 * Updates state and x (x += h) in place and writes the bf16 copy xb of the new x and its per-32-column chunk
 * statistics stats [M][W/32][2] (mean, M2) for the next block's folded LayerNorm.  W % 32 == 0.  softplus_a [W]:
 * softplus(a_param) per channel, as vt_ssm_step takes it (the caller computes it once per block).
 * Replaces: the RG-LRU step of tapnext/npu/r9/cpuemu.py:33-47 with its pre-norm (step8.py:474-479). */
int vt_rglru_fold(cudaStream_t stream, const float* G, long long ldg, const float* softplus_a, const float* rms_moments,
                  const float* rms_gamma, float* state, long long lds, float* x, long long ldx, uint16_t* xb,
                  long long ldxb, float* stats, int M, int W, float c, int first);

/* RG-LRU recurrence step over M tokens of width W on the bf16 input u (the normalised stream):
 * G = [gx_pre | ga_pre] fp32; state and the residual stream x fp32, updated in place (state <- h,
 * x <- x + h); first != 0 starts a sequence; softplus_a [W] = softplus(a_param) per channel.
 * Replaces: the RG-LRU forward restated in tapnext/npu/r9/cpuemu.py:33-47 (the NPU's EW SSM op). */
int vt_rglru(cudaStream_t stream, const float* G, long long ldg, const float* softplus_a, const uint16_t* u,
             long long ldu, float* state, long long lds, float* x, long long ldx, int M, int W, float c, int first);

/* One recurrent step of the full TAPNext++ block's temporal mixing for R tokens of width W (W % 64 == 0,
 * 64-channel heads): xc = conv_1d over the taps hist_old, hist_mid, hist_new (x_(t-3), x_(t-2), x_(t-1),
 * bf16) and xx (x_t, bf16), oldest first, + conv_b; the block-diagonal gates gx = sigmoid(xc_q wx[q] + bx),
 * ga = sigmoid(xc_q wa[q] + ba) per head q (wx / wa fp32 [W/64][64 in][64 out]); log_a = -8 ga softplus_a;
 * h = xc gx (first != 0) or a h + (xc gx) sqrt(1 - a^2) (fp32 state h, updated in place); z = bf16(h) yg,
 * where yg is the bf16 input as given, or with gelu_y != 0 its GELU-tanh (the raw y half of linear_yx; the
 * GELU rounds to bf16 as the GEMM epilogue's does).
 * Rounding follows the reference's bf16 restatement.  x_t is written over hist_old (the caller rotates
 * the three history roles); conv_w fp32 [4][W], conv_b / softplus_a / bx / ba fp32 [W].
 * Replaces: the recurrent block's conv_1d + rg_lru + (x * gelu(y)) of tapnext/npu/step8.py:477-480, whose
 * element-wise numerics the reference restates in tapnext/npu/pack8.py:252-279 (ssm_ref). */
int vt_ssm_step(cudaStream_t stream, const uint16_t* yg, const uint16_t* xx, long long ldi, uint16_t* hist_old,
                const uint16_t* hist_mid, const uint16_t* hist_new, long long ldh, float* h, long long ldhs,
                const float* conv_w, const float* conv_b, const float* softplus_a, const float* wx, const float* bx,
                const float* wa, const float* ba, uint16_t* z, long long ldz, int R, int W, int first, int gelu_y);

/* Gated MLP combine: out[r, j] = bf16(bf16(gelu_tanh(G[r, j])) * G[r, F + j]), j < F, for the bf16
 * ffw_up output G = [gate | up] [R][2F] (F % 8 == 0, 16-byte aligned rows).
 * Replaces: the gated_a / gated_b GEMM epilogues of tapnext/npu/mm8.cc:937-960 (mlp_block, step8.py:483). */
int vt_gated_gelu_mul(cudaStream_t stream, const uint16_t* G, long long ldg, uint16_t* out, long long ldo, int R, int F);

/* Exact GELU in place on a bf16 [R][N] matrix (N % 8 == 0): x = bf16(x (1 + erf(x / sqrt 2)) / 2).
 * Replaces: the ViT MLP's nn.GELU() (the gelu_pan epilogue, tapnext/npu/pack8.py:246-250 gelu_erf_ref). */
int vt_gelu_erf(cudaStream_t stream, uint16_t* x, long long ld, int R, int N);

/* Rotary embedding and KV-cache write for n new tokens at positions pos0 .. pos0+n-1 of H heads x 64:
 * qkv bf16 [n][ld] = q | k | v (head-major, ld >= 3*H*64); the first 32 dims of each q / k head rotate as
 * pairs (x_i, x_(16+i)) -> (x_i cos - x_(16+i) sin, x_i sin + x_(16+i) cos) at dims 2i, 2i+1 with the
 * angle tables cos_t / sin_t fp32 [ctx][16]; q -> q bf16 [H][n][64], k / v -> kc / vc bf16 [H][ctx][64].
 * Replaces: the rope + cache write of FastMD2._text_layers (moondream/gpu/md2fast.py:162-167, 186-191), the
 * unfused form of the reference's rope_cache. */
int vt_rope_qkv(cudaStream_t stream, const uint16_t* qkv, long long ld, int n, int H, int pos0, const float* cos_t,
                const float* sin_t, uint16_t* q, uint16_t* kc, uint16_t* vc, int ctx);

/* Causal attention of n new tokens over a KV cache: token i (position pos0 + i) attends to cache positions
 * 0 .. pos0 + i (q bf16 [H][n][64], kc / vc bf16 [H][ctx][64], ctx <= 2048), softmax(scale q k^T) v in fp32;
 * out bf16 [n][ldo], head h at columns h*64 .. h*64+63.
 * Replaces: the masked scaled_dot_product_attention of the question prefill, md2fast.py:192-193 with the
 * query mask of md2fast.py:132-136. */
int vt_attn_causal(cudaStream_t stream, const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int n, int H,
                   int pos0, int ctx, float scale, uint16_t* out, long long ldo);

/* One pass of the LANCZOS frame squash on 3-channel uint8 images: out[o, j, c] = clip(2^21 + sum_k
 * in[x0(o) + k, j, c] * w[o][k] >> 22) for o < n_out positions on the resampled axis and j < n_other along
 * the other, with bounds int32 [n_out][2] = (x0, count) and fixed-point weights int32 [n_out][ksize]
 * (22 fraction bits); element (a, b, c) of the input at in + a*sa + b*sb + c*sc bytes (a on the resampled
 * axis), of the output at out + a*oa + b*ob + c*oc.  Two passes (columns of the rows the second needs, then
 * rows) reproduce Pillow's Image.resize(..., LANCZOS) bit for bit.
 * Replaces: the host-side img.resize((378, 378), LANCZOS) of FastMD2.set_image (moondream/gpu/md2fast.py:223-228). */
int vt_resize_pass_u8(cudaStream_t stream, const uint8_t* in, long long sa, long long sb, long long sc, uint8_t* out,
                      long long oa, long long ob, long long oc, int n_out, int n_other, const int* bounds,
                      const int* weights, int ksize);

/* TAPNext++ tracking heads (fp32 on the CUDA cores), the host heads of the reference: Step8.heads_np,
 * tapnext/npu/step8.py:327-362 (numpy fp32; the torch form Step8.heads, step8.py:364-372).
 * vt_head_linear: Y[M, N] fp32 = X[M, K] . Wt + bias, X bf16 (x_bf16) or fp32 with row pitch ldx, Wt fp32
 *   [K][ldw] (the transposed nn.Linear weight, as heads_np's lin() stores it, step8.py:332-333), each output
 *   summed over k in order.  Replaces the `x @ w + b` of heads_np's mlp (step8.py:341-342, 348). */
int vt_head_linear(cudaStream_t stream, const void* X, long long ldx, int x_bf16, const float* Wt, long long ldw,
                   const float* bias, float* Y, long long ldy, int M, int N, int K);

/* In place per row of N (256 or 512) fp32 values: LayerNorm with gamma / beta group row % groups (two-pass
 * statistics), then the exact GELU 0.5 y (1 + erf(y / sqrt 2)).  Replaces heads_np's LayerNorm + erf GELU,
 * tapnext/npu/step8.py:343-347. */
int vt_head_ln_gelu(cudaStream_t stream, float* Y, long long ldy, int rows, int N, const float* gamma,
                    const float* beta, int groups, float eps);

/* Soft-argmax tracks: per query q and axis a (bins 256 or 512 logits at logits[q][a * bins]), the softmax of
 * logits * temperature restricted to +-window bins around the first maximum, renormalised; tracks[q][a] =
 * its expectation over the bin indices + 0.5.  Replaces tapnext/npu/step8.py:352-361. */
int vt_soft_argmax(cudaStream_t stream, const float* logits, long long ldl, int Q, int bins, int window,
                   float temperature, float* tracks, long long ldt);

#ifdef __cplusplus
}
#endif
#endif /* VT_B200_H */
