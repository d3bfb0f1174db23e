/* Drop-in C API: the reference moebius-cpu library's outer C interface
 * (include/moebius_cpu.h:1-73 of moebius-cpu, implemented there by src/ffi.rs:105-233),
 * declared with the same names, types, constants and struct layouts, and
 * exported by libmoebius_cuda.so. A C host written against moebius-cpu
 * relinks against this library without changing a call.
 *
 * Behaviour on the GPU build:
 *   - moebius_engine_create loads the weights onto one B200. `threads` (the
 *     reference's rayon pool size) has no meaning on the GPU and is ignored; the
 *     device is 0, or the index in the environment variable
 *     MOEBIUS_CUDA_DEVICE. Without a B200 it returns
 *     MOEBIUS_ERR_UNSUPPORTED_CPU (the reference's "this processor cannot run
 *     the engine" code).
 *   - moebius_inpaint runs the engine's mbx_inpaint (include/moebius_cuda_engine.h).
 *     Several host threads may call it on one engine, as with the reference
 *     (src/pipeline.rs:119-136); they take turns on the engine's GPU.
 *   - Status codes are the reference's 0-6. GPU-side failures (device memory
 *     exhausted, a CUDA error, a device wait that gave up) are reported as
 *     MOEBIUS_ERR_INTERNAL with the cause in moebius_last_error().
 */
#ifndef MOEBIUS_CUDA_DROPIN_MOEBIUS_CPU_H
#define MOEBIUS_CUDA_DROPIN_MOEBIUS_CPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MOEBIUS_ABI_VERSION 1u

/* Status codes returned by every int32_t entry point. */
#define MOEBIUS_OK                   0
#define MOEBIUS_ERR_INVALID_ARGUMENT 1
#define MOEBIUS_ERR_WEIGHTS          2
#define MOEBIUS_ERR_UNSUPPORTED_CPU  3 /* here: no B200 (sm_100) device */
#define MOEBIUS_ERR_CANCELLED        4
#define MOEBIUS_ERR_IO               5
#define MOEBIUS_ERR_INTERNAL         6

#define MOEBIUS_PRESET_EXACT 0u
#define MOEBIUS_PRESET_FAST  1u

#define MOEBIUS_PASTE_DEFAULT            0u
#define MOEBIUS_PASTE_NONE               1u
#define MOEBIUS_PASTE_FEATHER            2u
#define MOEBIUS_PASTE_FEATHER_COMPENSATE 3u

/* Opaque engine handle. */
typedef struct MoebiusEngine MoebiusEngine;

/* All-zero fields select the Exact preset's defaults. */
typedef struct MoebiusParams {
    uint32_t preset;      /* one of MOEBIUS_PRESET_* */
    uint32_t steps;       /* 0: the preset's step count */
    float    guidance;    /* <= 0: the preset's guidance scale */
    uint64_t seed;        /* noise seed */
    uint32_t paste;       /* one of MOEBIUS_PASTE_* */
    uint32_t mask_dilate; /* dilation radius in pixels, 0 = none */
} MoebiusParams;

/* A rectangle of image pixels. */
typedef struct MoebiusRect {
    uint32_t x, y, width, height;
} MoebiusRect;

/* Called with stage 0 (encode), 1 (denoise) or 2 (decode) and its progress;
 * a non-zero return cancels the inpaint. */
typedef int32_t (*MoebiusProgressFn)(void *user, uint32_t stage, uint32_t done, uint32_t total);

/* MOEBIUS_ABI_VERSION of the library. */
uint32_t moebius_abi_version(void);

/* Text of the calling thread's last failure; never NULL. */
const char *moebius_last_error(void);

/* Loads unet.safetensors and vae.safetensors from the UTF-8 directory
 * `weights_dir`. `threads` is accepted for compatibility and ignored. */
int32_t moebius_engine_create(const char *weights_dir, uint32_t threads, MoebiusEngine **out);

/* Frees an engine (NULL is ignored). */
void moebius_engine_destroy(MoebiusEngine *engine);

/* Inpaints the 8-bit RGB or RGBA image `pixels` (rows `stride` bytes apart) in
 * place wherever `mask` (rows `mask_stride` bytes apart) is >= 128; alpha is
 * kept. `params`, `progress` and `changed` may be NULL; `changed` receives the
 * rectangle that was rewritten. A cancelled call leaves the image as it was. */
int32_t moebius_inpaint(const MoebiusEngine *engine, uint8_t *pixels, uint32_t width, uint32_t height,
                        uint32_t stride, uint32_t channels, const uint8_t *mask, uint32_t mask_stride,
                        const MoebiusParams *params, MoebiusProgressFn progress, void *user, MoebiusRect *changed);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MOEBIUS_CUDA_DROPIN_MOEBIUS_CPU_H */
