/* moebius-cuda engine API: the moebius-cpu inpainting engine (UNet + VAE +
 * DDIM / DPM-Solver++ pipeline) running on the kernels of moebius_cuda.h, for
 * one B200.
 *
 * Mirrors the reference's outer C ABI, include/moebius_cpu.h:48-67 (status
 * codes, thread-local last error, engine create / destroy / inpaint, a
 * progress callback that can cancel), plus batch and component entry points.
 * Status codes and mbx_last_error() are those of moebius_cuda.h.
 *
 * mbx_inpaint takes images of any size (square crop window around the mask,
 * Lanczos3 to and from the model size, src/imaging/ modules); the batch call takes
 * model-size images, each used whole. Both presets (Exact, Fast), every paste
 * mode and mask dilation are built. */
#ifndef MOEBIUS_CUDA_ENGINE_H
#define MOEBIUS_CUDA_ENGINE_H

#include <stdint.h>

#include "moebius_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MBX_PRESET_EXACT 0u /* reference MOEBIUS_PRESET_EXACT */
#define MBX_PRESET_FAST  1u /* reference MOEBIUS_PRESET_FAST: 10 trailing DPM-Solver++(2M) steps, CFG for 3, ROI encode */

#define MBX_PASTE_DEFAULT            0u
#define MBX_PASTE_NONE               1u
#define MBX_PASTE_FEATHER            2u
#define MBX_PASTE_FEATHER_COMPENSATE 3u

typedef struct mbx_engine mbx_engine;

/* Zero-initialised = Exact preset defaults. Same fields as the reference's
 * MoebiusParams (include/moebius_cpu.h:31-39). */
typedef struct mbx_inpaint_params {
    uint32_t preset;      /* MBX_PRESET_* */
    uint32_t steps;       /* 0 = preset default (20 Exact, 10 Fast) */
    float guidance;       /* <= 0 = preset default (2.5) */
    uint64_t seed;
    uint32_t paste;       /* MBX_PASTE_* */
    uint32_t mask_dilate; /* px, 0 = off */
} mbx_inpaint_params;

/* stage: 0 encode, 1 denoise, 2 decode. Return non-zero to cancel. When a
 * callback is given the engine waits for each step to finish before
 * reporting it; without one, steps are queued back to back. */
typedef int32_t (*mbx_progress_fn)(void *user, uint32_t stage, uint32_t done, uint32_t total);

/* weights_dir holds unet.safetensors and vae.safetensors in the reference
 * converter's format (tools/convert_weights.py: f16 or f32 GEMM weights, f32
 * everything else; the VAE file's metadata carries scaling_factor 0.13025).
 * The network widths and latent size are read from the weight shapes.
 * Reference: moebius_engine_create (threads -> the CUDA device). */
int32_t mbx_engine_create(const char *weights_dir, int32_t device, mbx_engine **out);
void mbx_engine_destroy(mbx_engine *engine);

/* Runs the engine's work on `stream` (a cudaStream_t; NULL = its own stream). */
int32_t mbx_engine_set_stream(mbx_engine *engine, void *stream);

/* Kernels this engine has launched so far (graph replays count every kernel in the graph). */
uint64_t mbx_engine_launch_count(const mbx_engine *engine);

/* latent side, model image side and the three UNet level widths. */
int32_t mbx_engine_info(const mbx_engine *engine, int64_t *latent_side, int64_t *image_side, int64_t widths[3]);

/* In-place inpaint of one 8-bit RGB/RGBA host image of any size where mask >= 128;
 * alpha is preserved; *changed receives the rectangle written (empty for an empty
 * mask). Noise comes from `seed` (a deterministic generator of this library: the
 * reference's Rust generator cannot be reproduced). params, progress and changed
 * may be NULL. On MBX_ERR_CANCELLED the image is untouched. Reference:
 * moebius_inpaint, include/moebius_cpu.h:60-67, src/pipeline.rs:138-213. */
int32_t mbx_inpaint(mbx_engine *engine, uint8_t *pixels, uint32_t width, uint32_t height, uint32_t stride,
                    uint32_t channels, const uint8_t *mask, uint32_t mask_stride, const mbx_inpaint_params *params,
                    mbx_progress_fn progress, void *user, mbx_rect *changed);

/* mbx_inpaint with caller-supplied host noise (the reference's NoiseSet,
 * src/pipeline.rs:67-92): noise_vae [2][L][L][4] (image, masked image),
 * noise_init [L][L][4], noise_offset [4], L = the latent side; all three or none.
 * Reference: Engine::inpaint_with_noise, src/pipeline.rs:150-161. */
int32_t mbx_inpaint_with_noise(mbx_engine *engine, uint8_t *pixels, uint32_t width, uint32_t height,
                               uint32_t stride, uint32_t channels, const uint8_t *mask, uint32_t mask_stride,
                               const mbx_inpaint_params *params, const float *noise_vae, const float *noise_init,
                               const float *noise_offset, mbx_progress_fn progress, void *user, mbx_rect *changed);

/* n independent inpaints of side x side images (side = the model side, each image
 * used whole), processed together (the UNet runs at batch 2n for classifier-free
 * guidance, n for the Fast preset's conditional-only steps). pixels [n][side][side][channels]
 * (modified in place), masks [n][side][side]. Explicit noise (the reference's
 * NoiseSet, src/pipeline.rs:67-92), or all three NULL for seeded noise
 * (inpaint i uses seed + i):
 *   noise_vae    [2n][side/8][side/8][4]  (image, masked image posterior noise per inpaint)
 *   noise_init   [n][side/8][side/8][4]
 *   noise_offset [n][4]
 * device_buffers != 0: every pointer is device memory of the engine's device;
 * else host memory (copied in and out on the engine's stream; the call returns
 * when the results are back). Reference: Engine::inpaint_with_noise,
 * src/pipeline.rs:152-373, run for each inpaint. */
int32_t mbx_inpaint_batch(mbx_engine *engine, uint8_t *pixels, const uint8_t *masks, int64_t n, uint32_t side,
                          uint32_t channels, const mbx_inpaint_params *params, const float *noise_vae,
                          const float *noise_init, const float *noise_offset, int32_t device_buffers,
                          mbx_progress_fn progress, void *user);

/* One UNet evaluation on device buffers: x [items][L][L][9] -> eps [items][L][L][4]
 * at `timestep`. cfg != 0: items are (uncond, cond) pairs; else all cond.
 * Reference: UNet::forward, src/unet/mod.rs:200-301 (CFG tiling done by the caller). */
int32_t mbx_engine_unet_forward(mbx_engine *engine, const float *x, int64_t items, int64_t timestep, int32_t cfg,
                                float *eps);

/* VAE on device buffers. encode: images [b][h][w][3] in [-1, 1], noise
 * [b][h/8][w/8][4] -> scaled latents z [b][h/8][w/8][4] (src/vae/encoder.rs:173-216).
 * decode: scaled latents [b][h][w][4] -> (x + 1) / 2 [b][8h][8w][3] (src/vae/decoder.rs:74-99). */
int32_t mbx_engine_vae_encode(mbx_engine *engine, const float *images, const float *noise, int64_t b, int64_t h,
                              int64_t w, float *z);
int32_t mbx_engine_vae_decode(mbx_engine *engine, const float *latents, int64_t b, int64_t h, int64_t w,
                              float *out);

/* DDIM schedule of the Exact preset family (reference Ddim, src/scheduler.rs:19-98):
 * the denoised timesteps for `steps` at `strength` (spacing 0 leading, 1 trailing),
 * written to `out` (room for `steps` entries); *count receives their number. */
int32_t mbx_ddim_timesteps(uint32_t steps, double strength, int32_t trailing, int64_t *out, int64_t *count);
/* The 1000 f32 cumulative alpha products (scaled-linear betas 0.00085..0.012). */
int32_t mbx_ddim_alphas_cumprod(float *out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MOEBIUS_CUDA_ENGINE_H */
