/* moebius-cuda C API: the moebius-cpu engine kernel layer (the Rust crate's
 * src/engine/*) re-implemented for NVIDIA B200 (sm_100a).
 *
 * Conventions (those of the reference's C ABI, src/ffi.rs:1-103):
 *  - every entry point returns an int32 status (MBX_OK = 0); on failure the
 *    message is available from mbx_last_error() on the same thread;
 *  - C++ exceptions and CUDA errors never cross the boundary;
 *  - shape errors that the reference engine asserts on (it panics, e.g.
 *    src/engine/norm.rs:59-63, src/engine/conv.rs:39-44) are returned as
 *    MBX_ERR_INVALID_ARGUMENT instead of aborting.
 *
 * Memory: tensors are dense NHWC float32 in device memory, passed as plain
 * pointers plus sizes. Every kernel call is asynchronous on the context's
 * stream (mbx_ctx_set_stream may substitute the caller's stream); outputs must
 * not alias inputs unless a function says so (the reference's rule,
 * src/unet/blocks.rs:46). Device-side bounded waits that give up record an
 * error that the next mbx_ctx_synchronize() returns as MBX_ERR_TIMEOUT.
 */
#ifndef MOEBIUS_CUDA_H
#define MOEBIUS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Every declaration below is exported from libmoebius_cuda.so. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MBX_ABI_VERSION 1u

/* Codes 0-6 keep the meaning of include/moebius_cpu.h:13-19 of the reference. */
#define MBX_OK                     0
#define MBX_ERR_INVALID_ARGUMENT   1
#define MBX_ERR_WEIGHTS            2
#define MBX_ERR_UNSUPPORTED_DEVICE 3 /* reference: MOEBIUS_ERR_UNSUPPORTED_CPU */
#define MBX_ERR_CANCELLED          4
#define MBX_ERR_IO                 5
#define MBX_ERR_INTERNAL           6
#define MBX_ERR_OUT_OF_MEMORY      7
#define MBX_ERR_CUDA               8
#define MBX_ERR_TIMEOUT            9

/* Weight storage precision (reference Param, src/engine/param.rs:14-17). */
#define MBX_DTYPE_F32 0
#define MBX_DTYPE_F16 1

/* Depthwise epilogues (reference depthwise::Epilogue, src/engine/depthwise.rs:23-28). */
#define MBX_EPILOGUE_NONE     0
#define MBX_EPILOGUE_RELU     1
#define MBX_EPILOGUE_GLU_SILU 2 /* output has c/2 channels: y[:c/2] * SiLU(y[c/2:]) */

typedef struct mbx_ctx mbx_ctx;
typedef struct mbx_param mbx_param;

uint32_t mbx_abi_version(void);

/* Message for the last failed call on the calling thread (valid until the next
 * call on this thread). Never NULL. Reference: moebius_last_error, src/ffi.rs:114-117. */
const char *mbx_last_error(void);

/* ---------------------------------------------------------------- context */

/* Creates a context on `device` (must be sm_100: B200). Replaces the engine's
 * rayon pool + require_avx2_fma check (src/pipeline.rs:119-136, src/engine/cpu.rs). */
int32_t mbx_ctx_create(int32_t device, mbx_ctx **out);
void mbx_ctx_destroy(mbx_ctx *ctx);
/* Use `stream` (a cudaStream_t) for all later calls; NULL restores the context's own stream. */
int32_t mbx_ctx_set_stream(mbx_ctx *ctx, void *stream);
void *mbx_ctx_stream(mbx_ctx *ctx);
/* Waits for the stream, then reports CUDA errors and device-side wait timeouts. */
int32_t mbx_ctx_synchronize(mbx_ctx *ctx);
/* Number of this library's kernel launches on this context so far. */
uint64_t mbx_ctx_launch_count(const mbx_ctx *ctx);

/* ---------------------------------------------------------------- memory
 * A stream-ordered best-fit caching pool: the device analogue of the
 * reference's Scratch (src/engine/mod.rs:25-117, best_fit :104-117). */
int32_t mbx_alloc(mbx_ctx *ctx, size_t bytes, void **out);
int32_t mbx_free(mbx_ctx *ctx, void *ptr);
/* Frees cached blocks smaller than min_bytes (Scratch::release_below, src/engine/mod.rs:94-97). */
int32_t mbx_pool_release_below(mbx_ctx *ctx, size_t min_bytes);
int32_t mbx_pool_stats(const mbx_ctx *ctx, size_t *cached_bytes, size_t *in_use_bytes);
/* Page-locked host buffers for asynchronous host<->device copies. */
int32_t mbx_host_alloc(size_t bytes, void **out);
int32_t mbx_host_free(void *ptr);
int32_t mbx_memcpy_h2d(mbx_ctx *ctx, void *dst, const void *src, size_t bytes);
int32_t mbx_memcpy_d2h(mbx_ctx *ctx, void *dst, const void *src, size_t bytes);
int32_t mbx_memcpy_d2d(mbx_ctx *ctx, void *dst, const void *src, size_t bytes);

/* ---------------------------------------------------------------- params
 * A dense conv weight in its stored precision (Param::load / f16_from,
 * src/engine/param.rs:21-37). `host_data` holds c_out * taps * c_in values
 * of `dtype` (uint16 IEEE half for MBX_DTYPE_F16) in the converter's layout:
 * 1x1 [c_out, c_in] (taps = 1), 3x3 [c_out, 3, 3, c_in] (taps = 9). The
 * library re-lays it once for the tensor cores (the per-GEMM f16 widening
 * of Param::view, :45-59, happens at create time instead). */
int32_t mbx_param_create(mbx_ctx *ctx, const void *host_data, int32_t dtype, int64_t c_out, int64_t taps,
                         int64_t c_in, mbx_param **out);
void mbx_param_destroy(mbx_ctx *ctx, mbx_param *param);
int32_t mbx_param_info(const mbx_param *param, int64_t *c_out, int64_t *taps, int64_t *c_in, int32_t *dtype);

/* ---------------------------------------------------------------- elementwise */

/* x = SiLU(x). Reference: ops::silu_inplace, src/engine/ops.rs:11-13. */
int32_t mbx_silu_inplace(mbx_ctx *ctx, float *x, int64_t len);
/* a += b. Reference: ops::add_inplace, src/engine/ops.rs:16-19. */
int32_t mbx_add_inplace(mbx_ctx *ctx, float *a, const float *b, int64_t len);
/* out = (x + bias[c]) + temb[item, c] over [n, hw, c]; bias or temb may be NULL.
 * out may equal x. Reference: the conv bias prefill (init_output, src/engine/conv.rs:170-190)
 * and the resnet's pre-norm temb add (src/unet/blocks.rs:98, folded at src/engine/norm.rs:5-7). */
int32_t mbx_bias_temb_add(mbx_ctx *ctx, const float *x, int64_t n, int64_t hw, int64_t c, const float *bias,
                          const float *temb, float *out);
/* out[p] = [a[p] || b[p]]. Reference: Tensor::concat_channels_into, src/engine/tensor.rs:59-73. */
int32_t mbx_concat_channels(mbx_ctx *ctx, const float *a, int64_t ca, const float *b, int64_t cb, int64_t pixels,
                            float *out);

/* ---------------------------------------------------------------- norms */

/* GroupNorm statistics pass: per-item channel scale/shift ([n, c] each) with
 * GN(x + add) = x*scale + shift. add: [n, c] or NULL.
 * Reference: GroupNorm::affine, src/engine/norm.rs:57-105 (gn_stats :110-129). */
int32_t mbx_group_norm_affine(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c,
                              int64_t groups, float eps, const float *gamma, const float *beta, const float *add,
                              float *scale_out, float *shift_out);
/* out = [SiLU](x*scale[item,c] + shift[item,c]) (+ residual).
 * Reference: apply_affine, src/engine/norm.rs:134-147 (residual: ops::add_inplace fused). */
int32_t mbx_group_norm_apply(mbx_ctx *ctx, const float *x, int64_t n, int64_t hw, int64_t c, const float *scale,
                             const float *shift, int32_t silu, const float *residual, float *out);
/* out = [SiLU](GN(x + add[item])). Reference: GroupNorm::forward, src/engine/norm.rs:41-53. */
int32_t mbx_group_norm_forward(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c,
                               int64_t groups, float eps, const float *gamma, const float *beta, const float *add,
                               int32_t silu, float *out);
/* GroupNorm forward for callers that cannot allocate device memory. No
 * counterpart in the reference: the Rust engine's scratch is plain host memory.
 * Same inputs, outputs and results as mbx_group_norm_forward, but it takes the
 * caller's cudaStream_t (NULL = the legacy default stream) on the current
 * device instead of a context, and never calls cudaMalloc/cudaFree or any
 * other allocator: its scratch (n * ceil(h*w/256) * groups * 16 + n * c * 8
 * bytes) is one fixed 8 MiB array inside the library, held by every GPU that
 * loads it until the process exits. Larger problems are rejected with
 * MBX_ERR_INVALID_ARGUMENT. The first call on a device resolves that array's
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture. All calls share the one array, so calls that overlap on the GPU
 * (other streams, other host threads) race: serialise them. */
int32_t mbx_group_norm_forward_noalloc(void *stream, const float *x, int64_t n, int64_t h, int64_t w, int64_t c,
                                       int64_t groups, float eps, const float *gamma, const float *beta,
                                       const float *add, int32_t silu, float *out);
/* LayerNorm over the channels of every token. Reference: layer_norm, src/engine/norm.rs:151-172. */
int32_t mbx_layer_norm(mbx_ctx *ctx, const float *x, int64_t tokens, int64_t c, const float *gamma,
                       const float *beta, float eps, float *out);

/* ---------------------------------------------------------------- convolutions */

/* Depthwise 3x3, stride 1, zero pad 1, bias, fused epilogue (MBX_EPILOGUE_*).
 * weight [3, 3, c], bias [c]; out has c (or c/2 for GLU) channels.
 * Reference: depthwise3x3, src/engine/depthwise.rs:31-59. */
int32_t mbx_depthwise3x3(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c,
                         const float *weight, const float *bias, int32_t epilogue, float *out);

/* out[p] = x[p] . W^T + bias (+ residual[p]); W is a taps=1 param [c_out, c_in].
 * Reference: Conv1x1::forward, src/engine/conv.rs:38-55. */
int32_t mbx_conv1x1(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param *weight, const float *bias, const float *residual, float *out);

/* Output spatial size of mbx_conv3x3. Reference: Conv3x3::output_hw, src/engine/conv.rs:77-81. */
int32_t mbx_conv3x3_output_hw(int64_t h, int64_t w, int64_t stride, const int64_t pad[4], int32_t upsample2x,
                              int64_t *ho, int64_t *wo);

/* Dense 3x3 conv (taps=9 param [c_out, 3, 3, c_in]), any stride, zero padding
 * pad = [top, left, bottom, right], optional nearest-2x upsample of the input
 * read on the fly, optional GroupNorm prologue: the input is read as
 * [SiLU](x*pro_scale[item,c] + pro_shift[item,c]) at in-image taps while padding
 * stays zero (pro_scale/pro_shift [n, c_in] or NULL), bias, optional residual
 * [n, ho, wo, c_out] added in the epilogue.
 * Reference: Conv3x3::{forward, forward_prologue, forward_im2col},
 * src/engine/conv.rs:83-130 (Winograd for stride 1 / pad 1, src/engine/winograd.rs:48-120).
 * Computed as a direct implicit GEMM on the tensor cores (3xTF32 for f32
 * weights, 2xTF32 for f16 weights, f32 accumulation). */
int32_t mbx_conv3x3(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param *weight, const float *bias, int64_t stride, const int64_t pad[4],
                    int32_t upsample2x, const float *pro_scale, const float *pro_shift, int32_t pro_silu,
                    const float *residual, float *out);

/* c[m x n] (+)= A . B with arbitrary element strides (A: rows m, cols k;
 * B: rows k, cols n); c dense row-major. f32 FMA accumulation.
 * Reference: gemm::matmul with MatRef views, src/engine/gemm.rs:25-132. */
int32_t mbx_matmul(mbx_ctx *ctx, float *c, const float *a, int64_t m, int64_t k, int64_t a_row_stride,
                   int64_t a_col_stride, const float *b, int64_t n, int64_t b_row_stride, int64_t b_col_stride,
                   int32_t accumulate);

/* ---------------------------------------------------------------- attention and scaling */

/* In place, for each of `rows` rows of n floats: softmax(scale * row), with
 * probabilities below e^flush set to zero (pass -INFINITY to keep all).
 * Reference: softmax_rows, src/vae/mod.rs:273-293 (flush = -40). */
int32_t mbx_softmax_rows(mbx_ctx *ctx, float *x, int64_t rows, int64_t n, float scale, float flush);

/* c[m x n] = a[m x k] . B^T (+ bias[n]) (+ residual[m x n]) on the tensor cores
 * (3xTF32, f32 accumulation), with B a device matrix stored [n x k] row-major
 * (b_is_kn = 0) or [k x n] row-major (b_is_kn = 1). c must not alias a or b.
 * Reference: gemm::matmul with a transposed or row-major B view
 * (src/engine/gemm.rs:25-63), as used by the attention (src/vae/mod.rs:259-262). */
int32_t mbx_gemm(mbx_ctx *ctx, float *c, const float *a, int64_t m, int64_t k, const float *b, int64_t n,
                 int32_t b_is_kn, const float *bias, const float *residual);

/* out = x * mul + add over len floats (out may equal x). Reference: the decoder's
 * latent unscale and (x + 1) / 2, src/vae/decoder.rs:81,97. */
int32_t mbx_scale_add(mbx_ctx *ctx, const float *x, int64_t len, float mul, float add, float *out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MOEBIUS_CUDA_H */
