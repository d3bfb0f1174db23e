/* moebius-cuda C API: the moebius-cpu engine kernel layer (the Rust crate's
 * src/engine/ modules) re-implemented for NVIDIA B200 (sm_100a).
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

/* Activation applied by a 1x1 conv's epilogue after bias and residual. */
#define MBX_ACT_NONE 0
#define MBX_ACT_SILU 1

typedef struct mbx_ctx mbx_ctx;
typedef struct mbx_param mbx_param;

/* A pixel rectangle (reference MoebiusRect, include/moebius_cpu.h:41-43). */
typedef struct mbx_rect {
    uint32_t x, y, width, height;
} mbx_rect;

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
/* Self-test of the device-side error path (no reference counterpart: the
 * reference runs on the CPU and has no device waits). Enqueues one kernel whose
 * single thread waits on a barrier that nothing arrives at, giving up after
 * `cycles` clock cycles (1 <= cycles <= 2^32, about 2 s at most) as every
 * bounded wait in this library does; no copy is issued. The next
 * mbx_ctx_synchronize() then returns MBX_ERR_TIMEOUT and clears the record, and
 * the context stays usable. */
int32_t mbx_selftest_wait_timeout(mbx_ctx *ctx, int64_t cycles);

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
/* mbx_depthwise3x3 with a GroupNorm prologue: the input is read as
 * [SiLU](x*pro_scale[item,c] + pro_shift[item,c]) at in-image taps while padding
 * stays zero (pro_scale/pro_shift [n, c], e.g. from mbx_group_norm_affine); the
 * results equal mbx_group_norm_apply followed by mbx_depthwise3x3, bit for bit.
 * No single reference counterpart: GroupNorm::forward (with SiLU) feeding
 * DWConv2d::forward inside DwResnet::forward, src/unet/blocks.rs:84-112. */
int32_t mbx_depthwise3x3_fused(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c,
                               const float *pro_scale, const float *pro_shift, int32_t pro_silu,
                               const float *weight, const float *bias, int32_t epilogue, float *out);

/* out[p] = x[p] . W^T + bias (+ residual[p]); W is a taps=1 param [c_out, c_in].
 * Reference: Conv1x1::forward, src/engine/conv.rs:38-55. */
int32_t mbx_conv1x1(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param *weight, const float *bias, const float *residual, float *out);

/* mbx_conv1x1 with two fusions (no single reference counterpart): an optional
 * GroupNorm prologue, the input read as [SiLU](x*pro_scale[item,c] +
 * pro_shift[item,c]) (pro_scale/pro_shift [n, c_in] or NULL; reference:
 * GroupNorm::forward feeding the conv, src/unet/transformer.rs:324-325), and an
 * epilogue activation `act` (MBX_ACT_*) after bias and residual (reference:
 * Conv1x1::forward then silu_inplace, src/unet/transformer.rs:351-352). With a
 * prologue the library first writes the normalised input into pool scratch of
 * x's size (one memory-bound pass), then runs the conv on it. */
int32_t mbx_conv1x1_fused(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                          const mbx_param *weight, const float *bias, const float *pro_scale,
                          const float *pro_shift, int32_t pro_silu, const float *residual, int32_t act,
                          float *out);

/* Output spatial size of mbx_conv3x3. Reference: Conv3x3::output_hw, src/engine/conv.rs:77-81. */
int32_t mbx_conv3x3_output_hw(int64_t h, int64_t w, int64_t stride, const int64_t pad[4], int32_t upsample2x,
                              int64_t *ho, int64_t *wo);

/* Dense 3x3 conv (taps=9 param [c_out, 3, 3, c_in]), any stride, zero padding
 * pad = [top, left, bottom, right], optional nearest-2x upsample of the input
 * read on the fly, optional GroupNorm prologue: the input is read as
 * [SiLU](x*pro_scale[item,c] + pro_shift[item,c]) at in-image taps while padding
 * stays zero (pro_scale/pro_shift [n, c_in] or NULL; applied as one pass into pool
 * scratch of x's size before the conv), bias, optional residual
 * [n, ho, wo, c_out] added in the epilogue.
 * Reference: Conv3x3::{forward, forward_prologue, forward_im2col},
 * src/engine/conv.rs:83-130 (Winograd for stride 1 / pad 1, src/engine/winograd.rs:48-120).
 * Computed as a direct implicit GEMM on the tensor cores (3xTF32 for f32
 * weights, 2xTF32 for f16 weights, f32 accumulation). */
int32_t mbx_conv3x3(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param *weight, const float *bias, int64_t stride, const int64_t pad[4],
                    int32_t upsample2x, const float *pro_scale, const float *pro_shift, int32_t pro_silu,
                    const float *residual, float *out);
/* A 1x1 or 3x3 convolution (taps from the weight) whose epilogue also gathers the GroupNorm
 * statistics of its output, ending with that output's GroupNorm affine: out as mbx_conv1x1_fused /
 * mbx_conv3x3 give it, then scale_out / shift_out [n, c_out] as mbx_group_norm_affine(out, groups,
 * eps, gamma, beta, add) gives them, without reading out again. The statistics are per-channel f32
 * sums over 256-pixel chunks folded per group in f64, as in the separate pass. For a 1x1 weight,
 * stride must be 1 and upsample2x 0 (pad is ignored and may be NULL). Output maps that are not a
 * multiple of 256 pixels, or c_out not a multiple of 4, take the separate statistics pass.
 * Reference: Conv1x1::forward / Conv3x3::forward (src/engine/conv.rs:38-102) followed by
 * GroupNorm::affine (src/engine/norm.rs:57-129), as src/unet/blocks.rs:84-112 and
 * src/vae/mod.rs:190-211 call them. */
int32_t mbx_conv_group_norm_affine(mbx_ctx *ctx, const float *x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                                   const mbx_param *weight, const float *bias, int64_t stride, const int64_t pad[4],
                                   int32_t upsample2x, const float *pro_scale, const float *pro_shift,
                                   int32_t pro_silu, const float *residual, int32_t act, float *out, int64_t groups,
                                   float eps, const float *gamma, const float *beta, const float *add,
                                   float *scale_out, float *shift_out);

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

/* ---------------------------------------------------------------- lambda layers (UNet) */

/* Content lambda of `items` independent row sets: for each item,
 * lambda[kk][j] = sum_r e[r][kk] * values[r][j] / sum_r e[r][kk] with
 * e = exp(keys - column max over r), a softmax over rows per key channel.
 * keys: rows x k with row stride key_stride floats; values: rows x vd with row
 * stride value_stride; item i starts at i * rows * stride. out: [items][k][vd].
 * Reference: softmax_lambda, src/unet/lambda.rs:318-359 (chunk sums folded in f64). */
int32_t mbx_lambda_content(mbx_ctx *ctx, const float *keys, int64_t key_stride, const float *values,
                           int64_t value_stride, int64_t items, int64_t rows, int64_t k, int64_t vd,
                           float *lambda_out);

/* Self-lambda output added into `out` [n, h, w, 8k] (8 heads of k channels):
 * out[p, hd*k + v] += sum_kk q[p, hd*k + kk] * lambda[item][kk][v]
 *                     + a[p*8 + hd][225] + sum_{d < 225} a[p*8 + hd][d] * V[p + d, v]
 * where d = ky*15 + kx walks the 15x15 window centred on p (zero outside the
 * map) and V[p, v] = v_ptr[p * v_stride + v]. q [n, h, w, 8k]; lambda
 * [n][k][k] (from mbx_lambda_content); a [n*h*w*8][a_stride], a_stride >= 228
 * and a multiple of 4, holding Q . [W | b] (225 taps, then the bias column).
 * k must be a multiple of 8; q, a, v, out 16-byte aligned, v_stride a
 * multiple of 4. Reference: SelfLambda::forward + tap_filter,
 * src/unet/lambda.rs:107-184. */
int32_t mbx_self_lambda_position(mbx_ctx *ctx, const float *q, const float *lambda_c, const float *a,
                                 int64_t a_stride, const float *v, int64_t v_stride, int64_t n, int64_t h,
                                 int64_t w, int64_t k, float *out);

/* Cross-lambda output added into `out` [n, hw, 8k]: for item i with branch
 * b = i % branch_period,
 * out[p, hd*k + v] += sum_kk q[p, hd*k + kk] * lambda_c[b][kk][v]
 *                     + sum_m (sum_kk q[p, hd*k + kk] * e_table[p][m][kk]) * v_table[b][m][v]
 * over the m = 10 conditioning tokens; e_table [hw][10][k] (shared by all
 * items), lambda_c [branches][k][k], v_table [branches][10][k]. k a multiple of
 * 8, pointers 16-byte aligned. Reference: CrossLambda::forward + position_term,
 * src/unet/lambda.rs:252-294. */
int32_t mbx_cross_lambda_position(mbx_ctx *ctx, const float *q, const float *e_table, const float *lambda_c,
                                  const float *v_table, int64_t branch_period, int64_t n, int64_t hw, int64_t k,
                                  float *out);

/* ---------------------------------------------------------------- inpaint pipeline */

/* n square model-size inputs used whole (8-bit RGB or RGBA, `channels` 3|4,
 * tightly packed [n, h, w, channels]; masks [n, h, w], >= 128 = inpaint) ->
 * encoder batch images_out [2n, h, w, 3] = (rgb_0, masked_0, rgb_1, ...) in
 * [-1, 1], binary masks bin_out [n, h, w] (0 / 255), latent masks
 * mask_lat [n, h/8, w/8] (0 / 1, pixel (8y, 8x)) and, unless NULL,
 * nonempty_out [n] (1 where the mask has a pixel >= 128). h and w multiples
 * of 8. Reference: to_model (src/imaging/resize.rs:32-57, a same-size window
 * is a copy), src/pipeline.rs:202-204,236-252. */
int32_t mbx_inpaint_prepare(mbx_ctx *ctx, const uint8_t *image, const uint8_t *mask, int64_t n, int64_t h,
                            int64_t w, int64_t channels, float *images_out, uint8_t *bin_out, float *mask_lat,
                            int32_t *nonempty_out);

/* Posterior sample: z[p, c] = (mean + exp(0.5 * clamp(logvar, -30, 20)) * noise[p, c]) * scale
 * with moments [pixels][8] = mean(4) | logvar(4); z, noise [pixels][4].
 * Reference: encoder sample, src/vae/encoder.rs:219-230. */
int32_t mbx_vae_sample(mbx_ctx *ctx, const float *moments, const float *noise, int64_t pixels, float scale,
                       float *z);

/* Starting latents of n inpaints: init = noise_init + noise_offset_scale * noise_offset[i][c];
 * x = init when pure_noise, else sqrt_alpha * z_pairs[2i] + sqrt_one_minus_alpha * init.
 * z_pairs [2n, hw, 4] (encoder output: image latent, masked latent per inpaint);
 * noise_init, x [n, hw, 4]; noise_offset [n][4].
 * Reference: src/pipeline.rs:295-311, Ddim::add_noise src/scheduler.rs:78-85. */
int32_t mbx_latents_init(mbx_ctx *ctx, const float *z_pairs, const float *noise_init, const float *noise_offset,
                         int64_t n, int64_t hw, float noise_offset_scale, float sqrt_alpha,
                         float sqrt_one_minus_alpha, int32_t pure_noise, float *x);

/* UNet input [n * copies, hw, 9]: per pixel x(4) | mask_lat(1) | masked latent(4)
 * (z_pairs[2i + 1]), written `copies` times per inpaint (2 = CFG uncond/cond).
 * Reference: src/pipeline.rs:318-322 and the CFG tiling in UNet::forward,
 * src/unet/mod.rs:226-231. */
int32_t mbx_unet_input(mbx_ctx *ctx, const float *x, const float *mask_lat, const float *z_pairs, int64_t n,
                       int64_t hw, int64_t copies, float *out);

/* Guidance combine and one eta = 0 DDIM update of x [n, hw, 4] in place:
 * e = copies == 2 ? eps_u + guidance * (eps_c - eps_u) : eps; x0 = (x - coef[0]*e) / coef[1];
 * x = coef[2]*x0 + coef[3]*e with coef = {sqrt(1-a_t), sqrt(a_t), sqrt(a_prev), sqrt(1-a_prev)}.
 * eps [n * copies, hw, 4]. Reference: src/pipeline.rs:323-336, Ddim::step src/scheduler.rs:87-97. */
int32_t mbx_cfg_ddim_step(mbx_ctx *ctx, const float *eps, int64_t n, int64_t hw, int64_t copies, float guidance,
                          const float coef[4], float *x);

/* Pillow GaussianBlur(radius) of n single-channel 8-bit images [n, h, w]
 * (three fractional box passes per axis, rows first), byte-exact. `scratch`
 * holds n*h*w bytes; out may equal in. Reference: pil_gaussian_blur,
 * src/imaging/blend.rs:26-100. */
int32_t mbx_gaussian_blur_u8(mbx_ctx *ctx, const uint8_t *in, int64_t n, int64_t h, int64_t w, float radius,
                             uint8_t *scratch, uint8_t *out);

/* Feathered paste of decoded images result [n, h, w, 3] (in [0, 1], truncated
 * to 8 bits) into image [n, h, w, channels] in place through the blurred
 * binary mask `blurred` [n, h, w]: out = res*m + (1 - m)*src in f64, m = blurred/255.
 * Items whose nonempty[i] is 0 are left untouched (nonempty may be NULL).
 * Reference: to_u8 and paste (Paste::Feather), src/imaging/blend.rs:20-23,174-215;
 * an empty mask returns before any change, src/pipeline.rs:202-204. */
int32_t mbx_feather_paste(mbx_ctx *ctx, const float *result, const uint8_t *blurred, uint8_t *image, int64_t n,
                          int64_t h, int64_t w, int64_t channels, const int32_t *nonempty);

/* DPM-Solver++(2M) step of the Fast preset: e as in mbx_cfg_ddim_step, x0 = (x - coef[0]*e) * coef[1];
 * order 0 (the last step): x = x0; order 1: x = coef[2]*x + coef[3]*x0; order 2:
 * x = coef[2]*x + coef[3]*x0 - coef[4]*x0_prev. x0 is stored into x0_prev (orders 1, 2).
 * coef = {sigma_t, 1/alpha_t, sigma_next/sigma_t, phi or c0, c1}, computed in f64 and
 * rounded to f32 as the reference does (mbx_dpm_coefficients).
 * Reference: Dpm2M::step, src/scheduler.rs:107-152; src/pipeline.rs:323-344. */
int32_t mbx_cfg_dpm_step(mbx_ctx *ctx, const float *eps, int64_t n, int64_t hw, int64_t copies, float guidance,
                         const float coef[5], int32_t order, float *x, float *x0_prev);

/* Host-only: the coefficients of DPM-Solver++(2M) step i of the schedule (steps, strength,
 * spacing 0 leading / 1 trailing) with history restarted at step `restart_at` (-1 = never):
 * coef[5] and order as mbx_cfg_dpm_step takes them. Reference: src/scheduler.rs:100-152. */
int32_t mbx_dpm_coefficients(uint32_t steps, double strength, int32_t trailing, int64_t i, int64_t restart_at,
                             float coef[5], int32_t *order);

/* ---- Images of any size around the model window (reference src/imaging/ modules). ----
 * Images are 8-bit RGB or RGBA with a row stride in bytes; masks are 8-bit with
 * a row stride. A buffer may hold only a region of the whole image: origin_x,
 * origin_y give the image coordinates of its first pixel, width and height the
 * whole image's extent. All pixel work is byte-exact with the reference. */

/* Host-only: the square crop window (x, y, side) for a mask bbox (bx, by, bw, bh) in a
 * width x height image, never smaller than min(model_side, long side) and never larger
 * than the long side; *source receives the part of the window inside the image.
 * Reference: CropPlan::new / source_rect, src/imaging/crop.rs:30-62 (model_side = IMAGE_SIZE). */
int32_t mbx_crop_window(uint32_t bx, uint32_t by, uint32_t bw, uint32_t bh, uint32_t width, uint32_t height,
                        int64_t model_side, int64_t window[3], mbx_rect *source);

/* Host-only: Pillow's Lanczos3 coefficients for in_size -> out_size samples (the formulation
 * of fast_image_resize's convolution): bounds [out][2] = (first input, count), coeffs
 * [out][ksize] in 22-bit fixed point. With bounds == NULL only *ksize is written.
 * Reference: resize_u8, src/imaging/resize.rs:16-25. */
int32_t mbx_lanczos_table(int64_t in_size, int64_t out_size, int32_t *bounds, int32_t *coeffs, int64_t *ksize);

/* Binarise (>= 128 -> 255, else 0) and dilate n masks [n][h][mask_stride] with a k x k
 * square, anchor k/2 (k <= 1: binarise only) into out [n][h][w] (packed).
 * scratch: n*h*w bytes. Reference: dilate, src/imaging/mod.rs:61-89. */
int32_t mbx_mask_dilate(mbx_ctx *ctx, const uint8_t *mask, int64_t n, int64_t h, int64_t w, int64_t mask_stride,
                        int64_t k, uint8_t *scratch, uint8_t *out);

/* Bounding box of the pixels >= 128 of each of n masks: box [n][4] = {x0, y0, x1, y1}
 * (inclusive; x1 = -1 for an empty mask), device int32. Reference: MaskRef::bbox,
 * src/imaging/mod.rs:38-53. */
int32_t mbx_mask_bbox(mbx_ctx *ctx, const uint8_t *mask, int64_t n, int64_t h, int64_t w, int64_t mask_stride,
                      int32_t *box);

/* The window (win_x, win_y, side) -> model-size 8-bit RGB rgb_out [model_side]^2 x 3 and
 * binary mask bin_out [model_side]^2: edge replication past the image for the colour, zeros
 * for the mask, Lanczos3 (a copy when side == model_side), the mask re-thresholded at 128.
 * image / mask hold the region [origin, origin + region size) which must contain the
 * window's part inside the image. Reference: to_model, src/imaging/resize.rs:27-57. */
int32_t mbx_window_to_model(mbx_ctx *ctx, const uint8_t *image, int64_t stride, int64_t channels,
                            const uint8_t *mask, int64_t mask_stride, int64_t origin_x, int64_t origin_y,
                            int64_t region_w, int64_t region_h, int64_t width, int64_t height, int64_t win_x,
                            int64_t win_y, int64_t side, int64_t model_side, uint8_t *rgb_out, uint8_t *bin_out);

/* n decoded images [n][model_side]^2 x 3 in [0, 1] -> 8-bit windows out [n][side]^2 x 3
 * (truncation, then Lanczos3). Reference: from_model, src/imaging/resize.rs:61-67. */
int32_t mbx_model_to_window(mbx_ctx *ctx, const float *rgb, int64_t n, int64_t model_side, int64_t side,
                            uint8_t *out);

/* Pastes n window results result [n][side]^2 x 3 into n image regions in place
 * (image [n][region_h][stride], mask [n][region_h][mask_stride]; the region must
 * cover the window's source rectangle plus a 16 px margin clipped to the image).
 * mode: MBX_PASTE_NONE (1) copy, MBX_PASTE_FEATHER (2) or MBX_PASTE_FEATHER_COMPENSATE (3).
 * Items whose active[i] is 0 are left untouched (active may be NULL).
 * Reference: paste, src/imaging/blend.rs:104-215. */
int32_t mbx_paste(mbx_ctx *ctx, uint8_t *image, int64_t n, int64_t stride, int64_t channels, const uint8_t *mask,
                  int64_t mask_stride, int64_t origin_x, int64_t origin_y, int64_t region_w, int64_t region_h,
                  int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, const uint8_t *result,
                  uint32_t mode, const int32_t *active);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MOEBIUS_CUDA_H */
