// Per-inpaint element work of the Exact pipeline (reference src/pipeline.rs,
// src/scheduler.rs, src/vae/encoder.rs, src/imaging/{resize,blend}.rs), for a
// batch of n inpaints whose model-size images are used whole:
//
//  * prepare: 8-bit RGB(A) + mask → model RGB in [-1, 1] (f64 arithmetic, as
//    to_model), binary mask, masked image, nearest 8×-down latent mask
//    (pipeline.rs:236-252, resize.rs:32-57). Images go out as the encoder batch
//    [image_0, masked_0, image_1, masked_1, ...] (pipeline.rs:277).
//  * vae_sample: z = (mean + exp(½·clamp(logvar, −30, 20))·noise)·scale
//    (encoder.rs:219-230).
//  * latents_init: init = noise + offset·noise_offset[c]; x = init (strength ≥ 1)
//    or √ᾱ·z_img + √(1−ᾱ)·init (pipeline.rs:295-311, scheduler.rs:78-85).
//  * unet_input: [x ‖ mask_lat ‖ z_masked] per pixel, tiled over the CFG copies
//    (pipeline.rs:318-322, unet/mod.rs:226-231).
//  * cfg_ddim_step: ε = ε_u + g·(ε_c − ε_u) and the η = 0 DDIM update
//    (pipeline.rs:323-336, scheduler.rs:87-97).
//  * cfg_dpm_step: the same ε and one DPM-Solver++(2M) update (scheduler.rs:107-152).
//  * blur_lines: Pillow's 3-pass fractional box blur along rows or columns in
//    24-bit fixed point (blend.rs:41-100), byte-exact.
//  * feather_paste: 8-bit truncation of the decoded image and the feathered
//    blend with the blurred mask in f64 (blend.rs:20-23,174-215).
// Every f32 / f64 expression is written with explicitly rounded operations so
// that no multiply-add is contracted: the results follow the reference's
// operation order exactly.
#include <cmath>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kLatentChannels = 4;
constexpr int kUnetIn = 9;

__global__ void prepare_kernel(const uint8_t* __restrict__ img, const uint8_t* __restrict__ mask, int64_t n,
                               int64_t h, int64_t w, int ch, float* __restrict__ images, uint8_t* __restrict__ bin,
                               float* __restrict__ mask_lat, int32_t* __restrict__ nonempty) {
    const int64_t hw = h * w, total = n * hw;
    const int64_t lw = w / 8, lhw = (h / 8) * lw;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / hw, p = e - i * hw;
        const bool masked = mask[e] >= 128;
        bin[e] = masked ? 255 : 0;
        if (masked && nonempty) nonempty[i] = 1;  // every writer stores the same value
        const float keep = masked ? 0.0f : 1.0f;
        float* rgb = images + ((2 * i) * hw + p) * 3;
        float* msk = images + ((2 * i + 1) * hw + p) * 3;
        const uint8_t* src = img + e * ch;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float v = (float)__dadd_rn(__dmul_rn(__ddiv_rn((double)src[c], 255.0), 2.0), -1.0);
            rgb[c] = v;
            msk[c] = __fmul_rn(v, keep);
        }
        const int64_t y = p / w, x = p - y * w;
        if ((y & 7) == 0 && (x & 7) == 0) mask_lat[i * lhw + (y / 8) * lw + x / 8] = masked ? 1.0f : 0.0f;
    }
}

__global__ void vae_sample_kernel(const float* __restrict__ moments, const float* __restrict__ noise, int64_t pixels,
                                  float scale, float* __restrict__ z) {
    const int64_t total = pixels * kLatentChannels;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = e / kLatentChannels, c = e - p * kLatentChannels;
        const float mean = moments[p * 2 * kLatentChannels + c];
        const float lv = fminf(fmaxf(moments[p * 2 * kLatentChannels + kLatentChannels + c], -30.0f), 20.0f);
        z[e] = __fmul_rn(fmaf(expf(__fmul_rn(0.5f, lv)), noise[e], mean), scale);
    }
}

__global__ void latents_init_kernel(const float* __restrict__ z_pairs, const float* __restrict__ noise_init,
                                    const float* __restrict__ noise_offset, int64_t n, int64_t hw, float offset_scale,
                                    float sa, float sb, int pure, float* __restrict__ x) {
    const int64_t per = hw * kLatentChannels, total = n * per;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / per, r = e - i * per;
        const int c = (int)(r % kLatentChannels);
        const float init = __fadd_rn(noise_init[e], __fmul_rn(offset_scale, noise_offset[i * kLatentChannels + c]));
        x[e] = pure ? init : __fadd_rn(__fmul_rn(sa, z_pairs[(2 * i) * per + r]), __fmul_rn(sb, init));
    }
}

__global__ void unet_input_kernel(const float* __restrict__ x, const float* __restrict__ mask_lat,
                                  const float* __restrict__ z_pairs, int64_t n, int64_t hw, int copies,
                                  float* __restrict__ out) {
    const int64_t total = n * hw;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / hw, p = e - i * hw;
        float v[kUnetIn];
#pragma unroll
        for (int c = 0; c < kLatentChannels; ++c) v[c] = x[e * kLatentChannels + c];
        v[4] = mask_lat[e];
#pragma unroll
        for (int c = 0; c < kLatentChannels; ++c) v[5 + c] = z_pairs[((2 * i + 1) * hw + p) * kLatentChannels + c];
        for (int cp = 0; cp < copies; ++cp) {
            float* o = out + ((i * copies + cp) * hw + p) * kUnetIn;
#pragma unroll
            for (int c = 0; c < kUnetIn; ++c) o[c] = v[c];
        }
    }
}

__global__ void cfg_ddim_kernel(const float* __restrict__ eps, int64_t n, int64_t per, int copies, float guidance,
                                float sqrt_b_t, float sqrt_a_t, float sqrt_a_prev, float sqrt_b_prev,
                                float* __restrict__ x) {
    const int64_t total = n * per;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / per, r = e - i * per;
        float ep;
        if (copies == 2) {
            const float u = eps[(2 * i) * per + r], c = eps[(2 * i + 1) * per + r];
            ep = __fadd_rn(u, __fmul_rn(guidance, __fsub_rn(c, u)));
        } else {
            ep = eps[i * per + r];
        }
        const float x0 = __fdiv_rn(__fsub_rn(x[e], __fmul_rn(sqrt_b_t, ep)), sqrt_a_t);
        x[e] = __fadd_rn(__fmul_rn(sqrt_a_prev, x0), __fmul_rn(sqrt_b_prev, ep));
    }
}

// ε (guidance combine, or the cond-only copy), the data prediction x0 = (x − σ·ε)·(1/α) and the
// DPM-Solver++(2M) update (scheduler.rs:121-151): order 0 = the last step (x = x0); 1 = first
// order x = keep·x + φ·x0; 2 = second order x = keep·x + c0·x0 − c1·x0_prev. x0 is kept in x0_prev
// for the next step.
__global__ void cfg_dpm_kernel(const float* __restrict__ eps, int64_t n, int64_t per, int copies, float guidance,
                               float sigma, float inv_alpha, float keep, float c0, float c1, int order,
                               float* __restrict__ x, float* __restrict__ x0_prev) {
    const int64_t total = n * per;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / per, r = e - i * per;
        float ep;
        if (copies == 2) {
            const float u = eps[(2 * i) * per + r], c = eps[(2 * i + 1) * per + r];
            ep = __fadd_rn(u, __fmul_rn(guidance, __fsub_rn(c, u)));
        } else {
            ep = eps[i * per + r];
        }
        const float xv = x[e];
        const float x0 = __fmul_rn(__fsub_rn(xv, __fmul_rn(sigma, ep)), inv_alpha);
        float out;
        if (order == 0) {
            out = x0;
        } else if (order == 1) {
            out = __fadd_rn(__fmul_rn(keep, xv), __fmul_rn(c0, x0));
        } else {
            out = __fsub_rn(__fadd_rn(__fmul_rn(keep, xv), __fmul_rn(c0, x0)), __fmul_rn(c1, x0_prev[e]));
        }
        x[e] = out;
        if (order != 0) x0_prev[e] = x0;
    }
}

// out[i][:] = row[:] for i < copies (the timestep embedding of every item of a UNet batch).
__global__ void broadcast_rows_kernel(const float* __restrict__ row, int64_t len, int64_t copies,
                                      float* __restrict__ out) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < len * copies;
         e += (int64_t)gridDim.x * blockDim.x)
        out[e] = row[e % len];
}

// One CTA per line; `passes` fractional box passes with 8-bit rounding after each.
__global__ void blur_lines_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t lines_per_item,
                                  int64_t item_stride, int64_t line_stride, int64_t elem_stride, int len, int radius,
                                  uint32_t ww, uint32_t fw, int passes) {
    extern __shared__ uint8_t line[];
    uint8_t* a = line;
    uint8_t* b = line + len;
    const int64_t item = blockIdx.x / lines_per_item, l = blockIdx.x - item * lines_per_item;
    const int64_t base = item * item_stride + l * line_stride;
    for (int x = threadIdx.x; x < len; x += blockDim.x) a[x] = in[base + x * elem_stride];
    __syncthreads();
    for (int pass = 0; pass < passes; ++pass) {
        for (int x = threadIdx.x; x < len; x += blockDim.x) {
            auto at = [&](int i) -> uint32_t { return a[i < 0 ? 0 : (i >= len ? len - 1 : i)]; };
            uint32_t acc = 0;
            for (int i = x - radius; i <= x + radius; ++i) acc += at(i);
            const uint32_t far = at(x - radius - 1) + at(x + radius + 1);
            b[x] = (uint8_t)((acc * ww + far * fw + (1u << 23)) >> 24);
        }
        __syncthreads();
        uint8_t* t = a;
        a = b;
        b = t;
    }
    for (int x = threadIdx.x; x < len; x += blockDim.x) out[base + x * elem_stride] = a[x];
}

__global__ void feather_paste_kernel(const float* __restrict__ result, const uint8_t* __restrict__ blurred,
                                     uint8_t* __restrict__ image, int64_t pixels, int64_t item_pixels, int ch,
                                     const int32_t* __restrict__ nonempty) {
    for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < pixels;
         p += (int64_t)gridDim.x * blockDim.x) {
        if (nonempty && !nonempty[p / item_pixels]) continue;  // empty mask: the image is untouched
        const double m = __ddiv_rn((double)blurred[p], 255.0);
        const double keep = __dadd_rn(1.0, -m);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            // to_u8: clamp to [0, 1], ×255, truncate (NaN → 0).
            const float v = fminf(fmaxf(result[p * 3 + c], 0.0f), 1.0f);
            const uint8_t r8 = (uint8_t)__fmul_rn(v, 255.0f);
            uint8_t* dst = image + p * ch + c;
            const double res = __ddiv_rn((double)r8, 255.0), orig = __ddiv_rn((double)*dst, 255.0);
            const double o = __dmul_rn(__dadd_rn(__dmul_rn(res, m), __dmul_rn(keep, orig)), 255.0);
            *dst = (uint8_t)(o <= 0.0 ? 0.0 : (o >= 255.0 ? 255.0 : o));
        }
    }
}

}  // namespace

void launch_inpaint_prepare(mbx_ctx* ctx, const uint8_t* img, const uint8_t* mask, int64_t n, int64_t h, int64_t w,
                            int ch, float* images, uint8_t* bin, float* mask_lat, int32_t* nonempty) {
    if (nonempty) check_cuda(cudaMemsetAsync(nonempty, 0, size_t(n) * 4, ctx->stream), "inpaint flags");
    prepare_kernel<<<grid_for(ctx, n * h * w, 256), 256, 0, ctx->stream>>>(img, mask, n, h, w, ch, images, bin,
                                                                         mask_lat, nonempty);
    after_launch(ctx, "inpaint_prepare");
}

void launch_vae_sample(mbx_ctx* ctx, const float* moments, const float* noise, int64_t pixels, float scale,
                       float* z) {
    vae_sample_kernel<<<grid_for(ctx, pixels * kLatentChannels, 256), 256, 0, ctx->stream>>>(moments, noise, pixels,
                                                                                           scale, z);
    after_launch(ctx, "vae_sample");
}

void launch_latents_init(mbx_ctx* ctx, const float* z_pairs, const float* noise_init, const float* noise_offset,
                         int64_t n, int64_t hw, float offset_scale, float sa, float sb, bool pure, float* x) {
    latents_init_kernel<<<grid_for(ctx, n * hw * kLatentChannels, 256), 256, 0, ctx->stream>>>(
        z_pairs, noise_init, noise_offset, n, hw, offset_scale, sa, sb, pure ? 1 : 0, x);
    after_launch(ctx, "latents_init");
}

void launch_unet_input(mbx_ctx* ctx, const float* x, const float* mask_lat, const float* z_pairs, int64_t n,
                       int64_t hw, int copies, float* out) {
    unet_input_kernel<<<grid_for(ctx, n * hw, 256), 256, 0, ctx->stream>>>(x, mask_lat, z_pairs, n, hw, copies, out);
    after_launch(ctx, "unet_input");
}

void launch_cfg_ddim(mbx_ctx* ctx, const float* eps, int64_t n, int64_t per, int copies, float guidance,
                     const float coef[4], float* x) {
    cfg_ddim_kernel<<<grid_for(ctx, n * per, 256), 256, 0, ctx->stream>>>(eps, n, per, copies, guidance, coef[0],
                                                                         coef[1], coef[2], coef[3], x);
    after_launch(ctx, "cfg_ddim_step");
}

void launch_cfg_dpm(mbx_ctx* ctx, const float* eps, int64_t n, int64_t per, int copies, float guidance,
                    const float coef[5], int order, float* x, float* x0_prev) {
    cfg_dpm_kernel<<<grid_for(ctx, n * per, 256), 256, 0, ctx->stream>>>(eps, n, per, copies, guidance, coef[0],
                                                                        coef[1], coef[2], coef[3], coef[4], order, x,
                                                                        x0_prev);
    after_launch(ctx, "cfg_dpm_step");
}

void launch_broadcast_rows(mbx_ctx* ctx, const float* row, int64_t len, int64_t copies, float* out) {
    broadcast_rows_kernel<<<grid_for(ctx, len * copies, 256), 256, 0, ctx->stream>>>(row, len, copies, out);
    after_launch(ctx, "broadcast_rows");
}

void launch_blur_lines(mbx_ctx* ctx, const uint8_t* in, uint8_t* out, int64_t lines, int64_t lines_per_item,
                       int64_t item_stride, int64_t line_stride, int64_t elem_stride, int len, int radius,
                       uint32_t ww, uint32_t fw, int passes) {
    const int threads = len < 512 ? ((len + 31) / 32) * 32 : 512;
    blur_lines_kernel<<<(unsigned)lines, threads, 2 * len, ctx->stream>>>(in, out, lines_per_item, item_stride,
                                                                          line_stride, elem_stride, len, radius, ww,
                                                                          fw, passes);
    after_launch(ctx, "blur_lines");
}

void launch_feather_paste(mbx_ctx* ctx, const float* result, const uint8_t* blurred, uint8_t* image, int64_t pixels,
                          int64_t item_pixels, int ch, const int32_t* nonempty) {
    feather_paste_kernel<<<grid_for(ctx, pixels, 256), 256, 0, ctx->stream>>>(result, blurred, image, pixels,
                                                                            item_pixels, ch, nonempty);
    after_launch(ctx, "feather_paste");
}

namespace {
// Pillow's _gaussian_blur_radius in f32 with f64 sqrt / floor (src/imaging/blend.rs:26-39).
float gaussian_box_radius(float sigma, uint32_t passes) {
    const float sigma2 = sigma * sigma / (float)passes;
    const float big_l = (float)std::sqrt(12.0 * (double)sigma2 + 1.0);
    const float l = (float)std::floor(((double)big_l - 1.0) / 2.0);
    float a = (2.0f * l + 1.0f) * (l * (l + 1.0f) - 3.0f * sigma2);
    a /= 6.0f * (sigma2 - (l + 1.0f) * (l + 1.0f));
    return l + a;
}
}  // namespace

void gaussian_blur(mbx_ctx* ctx, const uint8_t* in, int64_t n, int64_t h, int64_t w, float radius, uint8_t* scratch,
                   uint8_t* out) {
    MBX_REQUIRE(h <= 16384 && w <= 16384, "blur: sides above 16384");
    if (n * h * w == 0) return;
    if (!(radius > 0.0f)) {
        if (out != in)
            check_cuda(cudaMemcpyAsync(out, in, size_t(n * h * w), cudaMemcpyDeviceToDevice, ctx->stream),
                       "blur copy");
        return;
    }
    const uint32_t passes = 3;
    const float fr = gaussian_box_radius(radius, passes);
    const int rad = (int)fr;
    const uint32_t ww = (uint32_t)((float)(1u << 24) / (fr * 2.0f + 1.0f));
    const uint32_t fw = ((1u << 24) - (uint32_t)(rad * 2 + 1) * ww) / 2;
    launch_blur_lines(ctx, in, scratch, n * h, h, h * w, w, 1, (int)w, rad, ww, fw, (int)passes);
    launch_blur_lines(ctx, scratch, out, n * w, w, h * w, 1, w, (int)h, rad, ww, fw, (int)passes);
}

}  // namespace mbx
