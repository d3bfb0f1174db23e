// Pixel-space work around the model window for images of any size (reference
// src/imaging/{mod,crop,resize,blend}.rs), all byte-exact:
//
//  * mask_dilate: binarise (>= 128 → 255) and dilate with a k × k square,
//    anchor k / 2, as a row pass and a column pass of running maxima
//    (imaging/mod.rs:61-89).
//  * mask_bbox: bounding box of the pixels >= 128 per item (imaging/mod.rs:38-53).
//  * window_to_model: the square crop window read with edge replication (the
//    mask with zeros) past the image, Lanczos3-resampled to the model side in
//    Pillow's two-pass 22-bit fixed-point formulation, horizontal pass first, the
//    mask re-thresholded at 128 (resize.rs:27-57). The horizontal pass carries
//    R, G, B and the mask as one 4-byte pixel. Same-size windows are a copy.
//  * model_to_window: 8-bit truncation of the decoded image and the Lanczos3
//    resample back to the window side (resize.rs:61-67).
//  * paste: Paste::None copies the result into the source rectangle; Feather
//    blends it through the Pillow-blurred binary mask of the rectangle plus a
//    16 px margin, in f64; FeatherCompensate first shifts the result by 1.1 ×
//    the per-channel mean difference (source − result) over the ring around the
//    mask bbox (blend.rs:104-215). Sums are exact 64-bit integer counts, so the
//    means do not depend on the reduction order.
// The resampling coefficients are computed on the host (double, the C library's
// sin) exactly as Pillow's precompute_coeffs / normalize_coeffs_8bpc do, then
// uploaded; the kernels only do the integer convolution.
#include <algorithm>
#include <cmath>
#include <vector>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kLanczosBits = 22;
constexpr int kBlurMargin = 16;  // blend.rs:102
constexpr int kRingOff = 10;     // blend.rs:109

__device__ __forceinline__ uint8_t clip8(int32_t acc) {
    const int32_t v = acc >> kLanczosBits;  // arithmetic shift: floor
    return (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
}

// ------------------------------------------------------------------ dilation

// Row pass: out[y][x] = max over x' ∈ [x − before, x + after] ∩ [0, w) of bin(mask[y][x']).
__global__ void dilate_rows_kernel(const uint8_t* __restrict__ mask, int64_t n, int64_t h, int64_t w, int64_t stride,
                                   int before, int after, uint8_t* __restrict__ out) {
    const int64_t total = n * h * w;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = e / w, x = e - row * w;
        const uint8_t* line = mask + row * stride;  // rows of all items are h·stride apart per item
        const int64_t lo = x - before < 0 ? 0 : x - before, hi = x + after >= w ? w - 1 : x + after;
        uint8_t m = 0;
        for (int64_t i = lo; i <= hi && !m; ++i) m = line[i] >= 128 ? 255 : 0;
        out[e] = m;
    }
}

// Column pass over the packed row-pass output.
__global__ void dilate_cols_kernel(const uint8_t* __restrict__ in, int64_t n, int64_t h, int64_t w, int before,
                                   int after, uint8_t* __restrict__ out) {
    const int64_t total = n * h * w;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = e / (h * w), r = e - item * h * w, y = r / w, x = r - y * w;
        const uint8_t* plane = in + item * h * w;
        const int64_t lo = y - before < 0 ? 0 : y - before, hi = y + after >= h ? h - 1 : y + after;
        uint8_t m = 0;
        for (int64_t i = lo; i <= hi && !m; ++i) m = plane[i * w + x];
        out[e] = m;
    }
}

// ------------------------------------------------------------------ bbox

__global__ void bbox_init_kernel(int32_t* box, int64_t n) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) {
        box[4 * i + 0] = INT32_MAX;
        box[4 * i + 1] = INT32_MAX;
        box[4 * i + 2] = -1;
        box[4 * i + 3] = -1;
    }
}

// grid.y = item; each thread folds its pixels, then one atomic per warp and coordinate.
__global__ void bbox_kernel(const uint8_t* __restrict__ mask, int64_t h, int64_t w, int64_t stride, int32_t* box) {
    const int64_t item = blockIdx.y;
    const uint8_t* m = mask + item * h * stride;
    int32_t x0 = INT32_MAX, y0 = INT32_MAX, x1 = -1, y1 = -1;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < h * w; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t y = e / w, x = e - y * w;
        if (m[y * stride + x] >= 128) {
            x0 = min(x0, (int32_t)x);
            x1 = max(x1, (int32_t)x);
            y0 = min(y0, (int32_t)y);
            y1 = max(y1, (int32_t)y);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        x0 = min(x0, __shfl_xor_sync(0xffffffffu, x0, o));
        y0 = min(y0, __shfl_xor_sync(0xffffffffu, y0, o));
        x1 = max(x1, __shfl_xor_sync(0xffffffffu, x1, o));
        y1 = max(y1, __shfl_xor_sync(0xffffffffu, y1, o));
    }
    if ((threadIdx.x & 31) == 0 && x1 >= 0) {
        atomicMin(box + 4 * item + 0, x0);
        atomicMin(box + 4 * item + 1, y0);
        atomicMax(box + 4 * item + 2, x1);
        atomicMax(box + 4 * item + 3, y1);
    }
}

// ------------------------------------------------------------------ resampling

struct Window {
    const uint8_t* image;  // pixel (origin_x, origin_y) of the image
    const uint8_t* mask;
    int64_t stride, mask_stride, channels;
    int64_t origin_x, origin_y;  // image coordinates of image[0]
    int64_t width, height;       // the whole image
    int64_t win_x, win_y;        // window origin in image coordinates
};

// R, G, B and the binary mask at window pixel (wx, wy): edge replication for the
// colour, zero for the mask outside the image.
__device__ __forceinline__ uchar4 window_pixel(const Window& g, int64_t wx, int64_t wy) {
    const int64_t x = g.win_x + wx, y = g.win_y + wy;
    const int64_t xc = x < 0 ? 0 : (x >= g.width ? g.width - 1 : x);
    const int64_t yc = y < 0 ? 0 : (y >= g.height ? g.height - 1 : y);
    const int64_t rx = xc - g.origin_x, ry = yc - g.origin_y;
    const uint8_t* p = g.image + ry * g.stride + rx * g.channels;
    const bool inside = x >= 0 && x < g.width && y >= 0 && y < g.height;
    const uint8_t m = inside && g.mask[ry * g.mask_stride + rx] >= 128 ? 255 : 0;
    return make_uchar4(p[0], p[1], p[2], m);
}

// Same-size window: the copy (no resampling) into model RGB and the binary mask.
__global__ void window_copy_kernel(Window g, int64_t side, uint8_t* __restrict__ rgb, uint8_t* __restrict__ bin) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < side * side;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t wy = e / side, wx = e - wy * side;
        const uchar4 v = window_pixel(g, wx, wy);
        rgb[3 * e + 0] = v.x;
        rgb[3 * e + 1] = v.y;
        rgb[3 * e + 2] = v.z;
        bin[e] = v.w;
    }
}

// Horizontal pass over the window: tmp[wy][xx] (RGBM) for side rows × out_w columns.
__global__ void window_h_kernel(Window g, int64_t side, int64_t out_w, const int32_t* __restrict__ bounds,
                                const int32_t* __restrict__ coeffs, int ksize, uchar4* __restrict__ tmp) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < side * out_w;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t wy = e / out_w, xx = e - wy * out_w;
        const int first = bounds[2 * xx], count = bounds[2 * xx + 1];
        const int32_t* k = coeffs + xx * (int64_t)ksize;
        int32_t a0 = 1 << (kLanczosBits - 1), a1 = a0, a2 = a0, a3 = a0;
        for (int i = 0; i < count; ++i) {
            const uchar4 v = window_pixel(g, first + i, wy);
            const int32_t c = k[i];
            a0 += (int32_t)v.x * c;
            a1 += (int32_t)v.y * c;
            a2 += (int32_t)v.z * c;
            a3 += (int32_t)v.w * c;
        }
        tmp[e] = make_uchar4(clip8(a0), clip8(a1), clip8(a2), clip8(a3));
    }
}

// Vertical pass RGBM → model RGB + re-thresholded mask.
__global__ void window_v_kernel(const uchar4* __restrict__ tmp, int64_t out_h, int64_t cols,
                                const int32_t* __restrict__ bounds, const int32_t* __restrict__ coeffs, int ksize,
                                uint8_t* __restrict__ rgb, uint8_t* __restrict__ bin) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < out_h * cols;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t yy = e / cols, x = e - yy * cols;
        const int first = bounds[2 * yy], count = bounds[2 * yy + 1];
        const int32_t* k = coeffs + yy * (int64_t)ksize;
        int32_t a0 = 1 << (kLanczosBits - 1), a1 = a0, a2 = a0, a3 = a0;
        for (int i = 0; i < count; ++i) {
            const uchar4 v = tmp[(int64_t)(first + i) * cols + x];
            const int32_t c = k[i];
            a0 += (int32_t)v.x * c;
            a1 += (int32_t)v.y * c;
            a2 += (int32_t)v.z * c;
            a3 += (int32_t)v.w * c;
        }
        rgb[3 * e + 0] = clip8(a0);
        rgb[3 * e + 1] = clip8(a1);
        rgb[3 * e + 2] = clip8(a2);
        bin[e] = clip8(a3) >= 128 ? 255 : 0;
    }
}

// to_u8 (blend.rs:20-24): clamp to [0, 1], × 255 in f32, truncate; NaN → 0.
__device__ __forceinline__ uint8_t to_u8(float v) {
    const float c = fminf(fmaxf(v, 0.0f), 1.0f);  // fmaxf(NaN, 0) = 0
    return (uint8_t)__fmul_rn(c, 255.0f);
}

__global__ void to_u8_kernel(const float* __restrict__ in, int64_t len, uint8_t* __restrict__ out) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < len; e += (int64_t)gridDim.x * blockDim.x)
        out[e] = to_u8(in[e]);
}

// Horizontal pass of the decoded image (f32 RGB, to_u8 on load): [n·rows][in_w] → [n·rows][out_w], 3 channels.
__global__ void model_h_kernel(const float* __restrict__ in, int64_t rows, int64_t in_w, int64_t out_w,
                               const int32_t* __restrict__ bounds, const int32_t* __restrict__ coeffs, int ksize,
                               uint8_t* __restrict__ out) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < rows * out_w;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = e / out_w, xx = e - row * out_w;
        const int first = bounds[2 * xx], count = bounds[2 * xx + 1];
        const int32_t* k = coeffs + xx * (int64_t)ksize;
        const float* src = in + (row * in_w + first) * 3;
        int32_t a0 = 1 << (kLanczosBits - 1), a1 = a0, a2 = a0;
        for (int i = 0; i < count; ++i) {
            const int32_t c = k[i];
            a0 += (int32_t)to_u8(src[3 * i + 0]) * c;
            a1 += (int32_t)to_u8(src[3 * i + 1]) * c;
            a2 += (int32_t)to_u8(src[3 * i + 2]) * c;
        }
        out[3 * e + 0] = clip8(a0);
        out[3 * e + 1] = clip8(a1);
        out[3 * e + 2] = clip8(a2);
    }
}

// Vertical pass, 3 channels: [n][in_h][cols] → [n][out_h][cols].
__global__ void resize_v3_kernel(const uint8_t* __restrict__ in, int64_t n, int64_t in_h, int64_t out_h, int64_t cols,
                                 const int32_t* __restrict__ bounds, const int32_t* __restrict__ coeffs, int ksize,
                                 uint8_t* __restrict__ out) {
    const int64_t total = n * out_h * cols;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = e / (out_h * cols), r = e - item * out_h * cols, yy = r / cols, x = r - yy * cols;
        const int first = bounds[2 * yy], count = bounds[2 * yy + 1];
        const int32_t* k = coeffs + yy * (int64_t)ksize;
        const uint8_t* src = in + ((item * in_h + first) * cols + x) * 3;
        int32_t a0 = 1 << (kLanczosBits - 1), a1 = a0, a2 = a0;
        for (int i = 0; i < count; ++i) {
            const int32_t c = k[i];
            const uint8_t* p = src + (int64_t)i * cols * 3;
            a0 += (int32_t)p[0] * c;
            a1 += (int32_t)p[1] * c;
            a2 += (int32_t)p[2] * c;
        }
        out[3 * e + 0] = clip8(a0);
        out[3 * e + 1] = clip8(a1);
        out[3 * e + 2] = clip8(a2);
    }
}

// ------------------------------------------------------------------ paste

struct PasteGeom {
    uint8_t* image;  // [n][region_h][stride], pixel (origin_x, origin_y) first
    const uint8_t* mask;
    int64_t stride, mask_stride, channels, region_h;
    int64_t sx, sy, sw, sh;  // source rectangle, buffer coordinates
    int64_t bx, by, bw, bh;  // blur region, buffer coordinates
    const uint8_t* result;   // [n][side][side][3]
    int64_t side, ox, oy;    // window side; source rectangle origin inside the window
    const int32_t* active;   // per item, or null
};

__global__ void paste_copy_kernel(PasteGeom g, int64_t n) {
    const int64_t per = g.sw * g.sh;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * per; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = e / per, r = e - item * per, y = r / g.sw, x = r - y * g.sw;
        if (g.active && !g.active[item]) continue;
        const uint8_t* res = g.result + ((item * g.side + g.oy + y) * g.side + g.ox + x) * 3;
        uint8_t* dst = g.image + (item * g.region_h + g.sy + y) * g.stride + (g.sx + x) * g.channels;
        dst[0] = res[0];
        dst[1] = res[1];
        dst[2] = res[2];
    }
}

// Binary mask of the blur region: [n][bh][bw], 255 where mask >= lo.
__global__ void region_binarize_kernel(PasteGeom g, int64_t n, int lo, uint8_t* __restrict__ out) {
    const int64_t per = g.bw * g.bh;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * per; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = e / per, r = e - item * per, y = r / g.bw, x = r - y * g.bw;
        out[e] = g.mask[(item * g.region_h + g.by + y) * g.mask_stride + g.bx + x] >= lo ? 255 : 0;
    }
}

// bbox {r0, c0, r1, c1} of the set pixels inside the source rectangle, rectangle coordinates.
__global__ void ring_bbox_kernel(PasteGeom g, const uint8_t* __restrict__ region, int32_t* box) {
    const int64_t item = blockIdx.y;
    const uint8_t* reg = region + item * g.bw * g.bh;
    int32_t r0 = INT32_MAX, c0 = INT32_MAX, r1 = -1, c1 = -1;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < g.sw * g.sh;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t y = e / g.sw, x = e - y * g.sw;
        if (reg[(g.sy - g.by + y) * g.bw + g.sx - g.bx + x]) {
            r0 = min(r0, (int32_t)y);
            r1 = max(r1, (int32_t)y);
            c0 = min(c0, (int32_t)x);
            c1 = max(c1, (int32_t)x);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        r0 = min(r0, __shfl_xor_sync(0xffffffffu, r0, o));
        c0 = min(c0, __shfl_xor_sync(0xffffffffu, c0, o));
        r1 = max(r1, __shfl_xor_sync(0xffffffffu, r1, o));
        c1 = max(c1, __shfl_xor_sync(0xffffffffu, c1, o));
    }
    if ((threadIdx.x & 31) == 0 && r1 >= 0) {  // box = {r0, c0, r1, c1}: minima first, as bbox_init sets
        atomicMin(box + 4 * item + 0, r0);
        atomicMin(box + 4 * item + 1, c0);
        atomicMax(box + 4 * item + 2, r1);
        atomicMax(box + 4 * item + 3, c1);
    }
}

// The ring box of blend.rs:131-137 from the set-pixel bbox (numpy integer arithmetic).
struct Ring {
    int64_t y0, y1, x0, x1;
};

__device__ __forceinline__ Ring ring_of(const int32_t* b, int64_t w, int64_t h) {
    const int64_t r0 = b[0], c0 = b[1], r1 = b[2], c1 = b[3];
    const int64_t hh = (r1 - r0 + 1 + kRingOff) / 2, hw = (c1 - c0 + 1 + kRingOff) / 2;
    const int64_t cr = (r0 + r1) / 2, cc = (c0 + c1) / 2;
    Ring r;
    r.y0 = cr - hh < 0 ? 0 : cr - hh;
    r.y1 = cr + hh > h - 1 ? h - 1 : cr + hh;
    r.x0 = cc - hw < 0 ? 0 : cc - hw;
    r.x1 = cc + hw > w - 1 ? w - 1 : cc + hw;
    return r;
}

// sums[item] = {Σ src R, G, B, Σ result R, G, B, count} over the ring's unset pixels.
__global__ void ring_sum_kernel(PasteGeom g, const uint8_t* __restrict__ region, const int32_t* __restrict__ box,
                                unsigned long long* sums) {
    const int64_t item = blockIdx.y;
    const int32_t* b = box + 4 * item;
    if (b[2] < 0) return;  // no set pixel: plain Feather
    const Ring r = ring_of(b, g.sw, g.sh);
    const int64_t rw = r.x1 - r.x0 + 1, total = rw * (r.y1 - r.y0 + 1);
    const uint8_t* reg = region + item * g.bw * g.bh;
    unsigned long long s[7] = {0, 0, 0, 0, 0, 0, 0};
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t y = r.y0 + e / rw, x = r.x0 + e % rw;
        if (reg[(g.sy - g.by + y) * g.bw + g.sx - g.bx + x]) continue;
        const uint8_t* src = g.image + (item * g.region_h + g.sy + y) * g.stride + (g.sx + x) * g.channels;
        const uint8_t* res = g.result + ((item * g.side + g.oy + y) * g.side + g.ox + x) * 3;
        for (int c = 0; c < 3; ++c) {
            s[c] += src[c];
            s[3 + c] += res[c];
        }
        s[6] += 1;
    }
    for (int c = 0; c < 7; ++c) {
        unsigned long long v = s[c];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0 && v) atomicAdd(sums + 7 * item + c, v);
    }
}

// out = (res/255 [+ shift])·m + (1 − m)·src/255 in f64, [clamped,] ×255, truncated (blend.rs:196-212).
__global__ void paste_blend_kernel(PasteGeom g, int64_t n, const uint8_t* __restrict__ blurred,
                                   const unsigned long long* __restrict__ sums, double fac) {
    const int64_t per = g.sw * g.sh;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * per; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = e / per, r = e - item * per, y = r / g.sw, x = r - y * g.sw;
        if (g.active && !g.active[item]) continue;
        bool comp = false;
        double shift[3] = {0.0, 0.0, 0.0};
        if (sums && sums[7 * item + 6] > 0) {
            comp = true;
            const double cnt = (double)sums[7 * item + 6];
            for (int c = 0; c < 3; ++c) {
                const double d = __dadd_rn(__ddiv_rn((double)sums[7 * item + c], cnt),
                                           -__ddiv_rn((double)sums[7 * item + 3 + c], cnt));
                shift[c] = __ddiv_rn(__dmul_rn(fac, d), 255.0);
            }
        }
        const double m =
            __ddiv_rn((double)blurred[item * g.bw * g.bh + (g.sy - g.by + y) * g.bw + g.sx - g.bx + x], 255.0);
        const double keep = __dadd_rn(1.0, -m);
        const uint8_t* res = g.result + ((item * g.side + g.oy + y) * g.side + g.ox + x) * 3;
        uint8_t* dst = g.image + (item * g.region_h + g.sy + y) * g.stride + (g.sx + x) * g.channels;
        for (int c = 0; c < 3; ++c) {
            double rv = __ddiv_rn((double)res[c], 255.0);
            if (comp) rv = __dadd_rn(rv, shift[c]);
            const double orig = __ddiv_rn((double)dst[c], 255.0);
            double o = __dadd_rn(__dmul_rn(rv, m), __dmul_rn(keep, orig));
            if (comp) o = o < 0.0 ? 0.0 : (o > 1.0 ? 1.0 : o);
            o = __dmul_rn(o, 255.0);
            dst[c] = (uint8_t)(o <= 0.0 ? 0.0 : (o >= 255.0 ? 255.0 : o));  // saturating truncation
        }
    }
}

// Pillow's Lanczos3 filter: sinc(x)·sinc(x/3) on [−3, 3).
double lanczos3(double x) {
    auto sinc = [](double v) {
        if (v == 0.0) return 1.0;
        v = v * M_PI;
        return std::sin(v) / v;
    };
    return (-3.0 <= x && x < 3.0) ? sinc(x) * sinc(x / 3.0) : 0.0;
}

// A resampling table on the device (bounds [out][2], coefficients [out][ksize]).
struct DeviceTable {
    PoolBuf bounds, coeffs;
    int ksize = 0;
    DeviceTable(mbx_ctx* ctx, int64_t in, int64_t out) {
        int64_t k = 0;
        lanczos_table(in, out, nullptr, nullptr, &k);
        ksize = (int)k;
        std::vector<int32_t> b(size_t(2 * out)), c(size_t(out * k));
        lanczos_table(in, out, b.data(), c.data(), &k);
        bounds = PoolBuf(ctx, b.size() * 4);
        coeffs = PoolBuf(ctx, c.size() * 4);
        check_cuda(cudaMemcpyAsync(bounds.p, b.data(), b.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "lanczos");
        // Copies from pageable memory have read the host buffer when they return.
        check_cuda(cudaMemcpyAsync(coeffs.p, c.data(), c.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "lanczos");
    }
};

}  // namespace

void lanczos_table(int64_t in, int64_t out, int32_t* bounds, int32_t* coeffs, int64_t* ksize) {
    const double scale = (double)in / (double)out;
    const double fscale = scale < 1.0 ? 1.0 : scale;
    const double support = 3.0 * fscale;
    const int64_t k = (int64_t)std::ceil(support) * 2 + 1;
    *ksize = k;
    if (!bounds) return;
    const double ss = 1.0 / fscale;
    std::vector<double> w((size_t)k);
    for (int64_t xx = 0; xx < out; ++xx) {
        const double center = ((double)xx + 0.5) * scale;
        int64_t xmin = (int64_t)(center - support + 0.5);
        if (xmin < 0) xmin = 0;
        int64_t xmax = (int64_t)(center + support + 0.5);
        if (xmax > in) xmax = in;
        xmax -= xmin;
        double ww = 0.0;
        for (int64_t x = 0; x < xmax; ++x) {
            w[size_t(x)] = lanczos3(((double)(x + xmin) - center + 0.5) * ss);
            ww += w[size_t(x)];
        }
        for (int64_t x = 0; x < k; ++x) {
            double v = x < xmax ? w[size_t(x)] : 0.0;
            if (x < xmax && ww != 0.0) v /= ww;
            const double f = v * (double)(1 << kLanczosBits);
            coeffs[xx * k + x] = x < xmax ? (int32_t)(v < 0 ? -0.5 + f : 0.5 + f) : 0;
        }
        bounds[2 * xx] = (int32_t)xmin;
        bounds[2 * xx + 1] = (int32_t)xmax;
    }
}

void launch_mask_dilate(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t stride, int64_t k,
                        uint8_t* scratch, uint8_t* out) {
    const int before = k <= 1 ? 0 : (int)(k / 2), after = k <= 1 ? 0 : (int)(k - 1 - k / 2);
    dilate_rows_kernel<<<grid_for(ctx, n * h * w, 256), 256, 0, ctx->stream>>>(mask, n, h, w, stride, before, after,
                                                                             k <= 1 ? out : scratch);
    after_launch(ctx, "mask_dilate");
    if (k <= 1) return;
    dilate_cols_kernel<<<grid_for(ctx, n * h * w, 256), 256, 0, ctx->stream>>>(scratch, n, h, w, before, after, out);
    after_launch(ctx, "mask_dilate");
}

void launch_mask_bbox(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t stride,
                      int32_t* box) {
    bbox_init_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(box, n);
    after_launch(ctx, "mask_bbox");
    const int64_t blocks = std::min<int64_t>((h * w + 255) / 256, 4 * (int64_t)ctx->sm_count);
    bbox_kernel<<<dim3((unsigned)blocks, (unsigned)n), 256, 0, ctx->stream>>>(mask, h, w, stride, box);
    after_launch(ctx, "mask_bbox");
}

void launch_window_to_model(mbx_ctx* ctx, const uint8_t* image, int64_t stride, int64_t channels,
                            const uint8_t* mask, int64_t mask_stride, int64_t origin_x, int64_t origin_y,
                            int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, int64_t model,
                            uint8_t* rgb, uint8_t* bin) {
    Window g{image, mask, stride, mask_stride, channels, origin_x, origin_y, width, height, win_x, win_y};
    if (side == model) {
        window_copy_kernel<<<grid_for(ctx, side * side, 256), 256, 0, ctx->stream>>>(g, side, rgb, bin);
        after_launch(ctx, "window_to_model");
        return;
    }
    DeviceTable t(ctx, side, model);
    PoolBuf tmp(ctx, size_t(side * model) * 4);
    window_h_kernel<<<grid_for(ctx, side * model, 256), 256, 0, ctx->stream>>>(
        g, side, model, t.bounds.as<int32_t>(), t.coeffs.as<int32_t>(), t.ksize, tmp.as<uchar4>());
    after_launch(ctx, "window_to_model");
    window_v_kernel<<<grid_for(ctx, model * model, 256), 256, 0, ctx->stream>>>(
        tmp.as<uchar4>(), model, model, t.bounds.as<int32_t>(), t.coeffs.as<int32_t>(), t.ksize, rgb, bin);
    after_launch(ctx, "window_to_model");
}

void launch_model_to_window(mbx_ctx* ctx, const float* rgb, int64_t n, int64_t model, int64_t side, uint8_t* out) {
    if (side == model) {
        to_u8_kernel<<<grid_for(ctx, n * model * model * 3, 256), 256, 0, ctx->stream>>>(rgb, n * model * model * 3,
                                                                                       out);
        after_launch(ctx, "model_to_window");
        return;
    }
    DeviceTable t(ctx, model, side);
    PoolBuf tmp(ctx, size_t(n * model * side * 3));
    model_h_kernel<<<grid_for(ctx, n * model * side, 256), 256, 0, ctx->stream>>>(
        rgb, n * model, model, side, t.bounds.as<int32_t>(), t.coeffs.as<int32_t>(), t.ksize, tmp.as<uint8_t>());
    after_launch(ctx, "model_to_window");
    resize_v3_kernel<<<grid_for(ctx, n * side * side, 256), 256, 0, ctx->stream>>>(
        tmp.as<uint8_t>(), n, model, side, side, t.bounds.as<int32_t>(), t.coeffs.as<int32_t>(), t.ksize, out);
    after_launch(ctx, "model_to_window");
}

void launch_paste(mbx_ctx* ctx, uint8_t* image, int64_t n, int64_t stride, int64_t channels, const uint8_t* mask,
                  int64_t mask_stride, int64_t origin_x, int64_t origin_y, int64_t region_w, int64_t region_h,
                  int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, const uint8_t* result,
                  uint32_t mode, const int32_t* active) {
    // Source rectangle (crop.rs:44-51) and blur region (blend.rs:176-183), image coordinates.
    const int64_t sx0 = std::max<int64_t>(win_x, 0), sy0 = std::max<int64_t>(win_y, 0);
    const int64_t sx1 = std::min<int64_t>(win_x + side, width), sy1 = std::min<int64_t>(win_y + side, height);
    if (sx1 <= sx0 || sy1 <= sy0 || n == 0) return;
    const int64_t bx0 = std::max<int64_t>(sx0 - kBlurMargin, 0), by0 = std::max<int64_t>(sy0 - kBlurMargin, 0);
    const int64_t bx1 = std::min<int64_t>(sx1 + kBlurMargin, width), by1 = std::min<int64_t>(sy1 + kBlurMargin, height);
    MBX_REQUIRE(bx0 >= origin_x && by0 >= origin_y && bx1 <= origin_x + region_w && by1 <= origin_y + region_h,
                "paste: the buffers must cover the source rectangle plus a 16 px margin (clipped to the image)");
    PasteGeom g;
    g.image = image;
    g.mask = mask;
    g.stride = stride;
    g.mask_stride = mask_stride;
    g.channels = channels;
    g.region_h = region_h;
    g.sx = sx0 - origin_x;
    g.sy = sy0 - origin_y;
    g.sw = sx1 - sx0;
    g.sh = sy1 - sy0;
    g.bx = bx0 - origin_x;
    g.by = by0 - origin_y;
    g.bw = bx1 - bx0;
    g.bh = by1 - by0;
    g.result = result;
    g.side = side;
    g.ox = sx0 - win_x;
    g.oy = sy0 - win_y;
    g.active = active;
    const int64_t per = g.sw * g.sh;
    if (mode == 1) {  // Paste::None
        paste_copy_kernel<<<grid_for(ctx, n * per, 256), 256, 0, ctx->stream>>>(g, n);
        after_launch(ctx, "paste");
        return;
    }
    const bool comp = mode == 3;
    const int64_t rplane = g.bw * g.bh;
    PoolBuf region(ctx, size_t(n * rplane)), blurred(ctx, size_t(n * rplane)), scratch(ctx, size_t(n * rplane));
    region_binarize_kernel<<<grid_for(ctx, n * rplane, 256), 256, 0, ctx->stream>>>(g, n, comp ? 129 : 128,
                                                                                  region.as<uint8_t>());
    after_launch(ctx, "paste");
    gaussian_blur(ctx, region.as<uint8_t>(), n, g.bh, g.bw, 3.0f, scratch.as<uint8_t>(), blurred.as<uint8_t>());
    PoolBuf box, sums;
    if (comp) {
        box = PoolBuf(ctx, size_t(n) * 16);
        sums = PoolBuf(ctx, size_t(n) * 7 * 8);
        bbox_init_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(box.as<int32_t>(), n);
        after_launch(ctx, "paste");
        check_cuda(cudaMemsetAsync(sums.p, 0, size_t(n) * 7 * 8, ctx->stream), "paste sums");
        const int64_t blocks = std::min<int64_t>((per + 255) / 256, 4 * (int64_t)ctx->sm_count);
        ring_bbox_kernel<<<dim3((unsigned)blocks, (unsigned)n), 256, 0, ctx->stream>>>(g, region.as<uint8_t>(),
                                                                                       box.as<int32_t>());
        after_launch(ctx, "paste");
        ring_sum_kernel<<<dim3((unsigned)blocks, (unsigned)n), 256, 0, ctx->stream>>>(
            g, region.as<uint8_t>(), box.as<int32_t>(), sums.as<unsigned long long>());
        after_launch(ctx, "paste");
    }
    paste_blend_kernel<<<grid_for(ctx, n * per, 256), 256, 0, ctx->stream>>>(
        g, n, blurred.as<uint8_t>(), comp ? sums.as<unsigned long long>() : nullptr, 1.1);
    after_launch(ctx, "paste");
}

}  // namespace mbx
