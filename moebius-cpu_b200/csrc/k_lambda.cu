// Multi-query λ layers of the UNet transformer blocks (reference
// src/unet/lambda.rs). Notation: C = 8·k channels, 8 heads of k query / value
// channels, N = H·W pixels per item.
//
//  * lambda_content (softmax_lambda, lambda.rs:322-359): per item
//    λc[kk][j] = Σ_r e[r][kk]·v[r][j] / Σ_r e[r][kk], e = exp(key − colmax).
//    Three passes: per 256-row chunk column maxima; per chunk the exponentials,
//    their f32 sums and the partial products (a [k × 40-column] slab per CTA);
//    then the fold over chunks (sums in f64, as the reference folds its chunk
//    sums) and the 1/Σ scaling.
//  * self_position (SelfLambda::forward + tap_filter, lambda.rs:107-184):
//    out[p, h·k + v] += Σ_kk Q[p,h,kk]·λc[kk][v] + A[p,h,225]
//                       + Σ_δ A[p,h,δ]·V[p+δ, v]      (15×15 window, zero pad 7)
//    with A = Q·W_aug computed beforehand by the tensor-core GEMM. One CTA per
//    8×8 pixel tile and v-slice; a thread owns one (pixel, head) and VS value
//    channels in registers, so A is read once per slice and the window of V
//    (22×22 pixels × VS channels) comes from shared memory.
//  * cross_position (CrossLambda::forward + position_term, lambda.rs:252-294):
//    out[p, h·k + v] += Σ_kk Q[p,h,kk]·λc[b][kk][v] + Σ_m (Σ_kk Q[p,h,kk]·E[p,m,kk])·V[b][m][v]
//    for the item's conditioning branch b; λc and V are load-time constants.
#include <cfloat>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kHeads = 8;
constexpr int kWin = 15;
constexpr int kTaps = kWin * kWin;
constexpr int kPad = kWin / 2;
constexpr int kTile = 8;                    // 8×8 output pixels per CTA
constexpr int kHalo = kTile + kWin - 1;     // 22
constexpr int kLamChunk = 256;              // rows per partial (the reference's SOFTMAX_CHUNK)
constexpr int kLamRows = 32;                // rows staged in shared memory at a time
constexpr int kLamCols = 40;                // λ columns per CTA of the partial pass
constexpr int kTokens = 10;

// ---------------------------------------------------------------- content λ

__global__ void lambda_colmax_kernel(const float* __restrict__ keys, int64_t ks, int64_t rows, int k, int chunks,
                                     float* __restrict__ pmax) {
    const int chunk = blockIdx.x, item = blockIdx.y;
    const float* kb = keys + (int64_t)item * rows * ks;
    const int64_t r0 = (int64_t)chunk * kLamChunk;
    const int64_t r1 = r0 + kLamChunk < rows ? r0 + kLamChunk : rows;
    for (int kk = threadIdx.x; kk < k; kk += blockDim.x) {
        float m = -FLT_MAX;
        for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, __ldg(kb + r * ks + kk));
        pmax[((int64_t)item * chunks + chunk) * k + kk] = m;
    }
}

// Block: k·G threads (G = column groups of 8 in this CTA's slab); thread (kk, g)
// accumulates λ[kk][j0 + 8g .. +8] over the chunk's rows.
__global__ void lambda_partial_kernel(const float* __restrict__ keys, int64_t ks, const float* __restrict__ vals,
                                      int64_t vs, int64_t rows, int k, int vd, int chunks,
                                      const float* __restrict__ pmax, float* __restrict__ plam,
                                      float* __restrict__ psum) {
    extern __shared__ float smem[];
    const int chunk = blockIdx.x, item = blockIdx.y, j0 = blockIdx.z * kLamCols;
    const int ncols = vd - j0 < kLamCols ? vd - j0 : kLamCols;
    const int groups = (ncols + 7) / 8;
    float* colmax = smem;                          // [k]
    float* e_t = colmax + k;                       // [kLamRows][k]
    float* v_t = e_t + kLamRows * k;               // [kLamRows][kLamCols]
    const int tid = threadIdx.x, nthr = blockDim.x;
    for (int kk = tid; kk < k; kk += nthr) {
        float m = -FLT_MAX;
        for (int c = 0; c < chunks; ++c) m = fmaxf(m, pmax[((int64_t)item * chunks + c) * k + kk]);
        colmax[kk] = m;
    }
    const float* kb = keys + (int64_t)item * rows * ks;
    const float* vb = vals + (int64_t)item * rows * vs;
    const int64_t r0 = (int64_t)chunk * kLamChunk;
    const int64_t r1 = r0 + kLamChunk < rows ? r0 + kLamChunk : rows;
    const int kk = tid / groups, g = tid - kk * groups;
    const bool active = kk < k;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    float s = 0.0f;
    __syncthreads();
    for (int64_t rt = r0; rt < r1; rt += kLamRows) {
        const int nr = (int)(r1 - rt < kLamRows ? r1 - rt : kLamRows);
        for (int i = tid; i < nr * k; i += nthr) {
            const int rr = i / k, c = i - rr * k;
            e_t[rr * k + c] = expf(__ldg(kb + (rt + rr) * ks + c) - colmax[c]);
        }
        for (int i = tid; i < nr * kLamCols; i += nthr) {
            const int rr = i / kLamCols, c = i - rr * kLamCols;
            v_t[rr * kLamCols + c] = c < ncols ? __ldg(vb + (rt + rr) * vs + j0 + c) : 0.0f;
        }
        __syncthreads();
        if (active) {
            for (int rr = 0; rr < nr; ++rr) {
                const float ev = e_t[rr * k + kk];
                s += ev;
                const float* vr = v_t + rr * kLamCols + 8 * g;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(ev, vr[j], acc[j]);
            }
        }
        __syncthreads();
    }
    if (!active) return;
    const int64_t base = ((int64_t)item * chunks + chunk) * k + kk;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (8 * g + j < ncols) plam[base * vd + j0 + 8 * g + j] = acc[j];
    if (blockIdx.z == 0 && g == 0) psum[base] = s;
}

__global__ void lambda_finalize_kernel(const float* __restrict__ plam, const float* __restrict__ psum, int64_t items,
                                       int k, int vd, int chunks, float* __restrict__ lam) {
    const int64_t total = items * k * vd;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(e % vd);
        const int64_t ik = e / vd;  // item·k + kk
        const int64_t item = ik / k, kk = ik - item * k;
        float a = 0.0f;
        double s = 0.0;
        for (int c = 0; c < chunks; ++c) {
            const int64_t b = (item * chunks + c) * k + kk;
            a += plam[b * vd + j];
            s += (double)psum[b];
        }
        lam[e] = a * (float)(1.0 / s);
    }
}

// ---------------------------------------------------------------- self-λ position term

// Shared layout: V window [kHalo²][VS + 4] (4 floats of padding keep the four pixels a
// warp reads in distinct banks), then λc slice [k][VS].
template <int VS>
__global__ void __launch_bounds__(512, 1)
    self_position_kernel(const float* __restrict__ q, const float* __restrict__ lam, const float* __restrict__ a,
                         int a_stride, const float* __restrict__ v, int64_t v_stride, int H, int W, int k,
                         int tiles_x, float* __restrict__ out) {
    extern __shared__ float4 smem4[];
    float* halo = reinterpret_cast<float*>(smem4);
    constexpr int HS = VS + 4;
    float* lam_s = halo + kHalo * kHalo * HS;
    const int item = blockIdx.z, j0 = blockIdx.y * VS;
    const int ty0 = (blockIdx.x / tiles_x) * kTile, tx0 = (blockIdx.x % tiles_x) * kTile;
    const int c = kHeads * k;
    const int64_t item_px = (int64_t)item * H * W;
    const int tid = threadIdx.x;

    // V window for this slice (zero outside the map = the reference's skipped taps).
    for (int i = tid; i < kHalo * kHalo * (VS / 4); i += 512) {
        const int row = i / (VS / 4), c4 = i - row * (VS / 4);
        const int hy = row / kHalo, hx = row - hy * kHalo;
        const int iy = ty0 + hy - kPad, ix = tx0 + hx - kPad;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (iy >= 0 && iy < H && ix >= 0 && ix < W)
            val = __ldg(reinterpret_cast<const float4*>(v + (item_px + (int64_t)iy * W + ix) * v_stride + j0) + c4);
        *reinterpret_cast<float4*>(halo + row * HS + 4 * c4) = val;
    }
    const float* lam_i = lam + (int64_t)item * k * k;
    for (int i = tid; i < k * VS; i += 512) {
        const int kk = i / VS, j = i - kk * VS;
        lam_s[i] = __ldg(lam_i + (int64_t)kk * k + j0 + j);
    }
    __syncthreads();

    const int h = tid & 7, p = tid >> 3;
    const int ty = p >> 3, tx = p & 7;
    const int y = ty0 + ty, x = tx0 + tx;
    if (y >= H || x >= W) return;
    const int64_t pix = item_px + (int64_t)y * W + x;

    float acc[VS];
#pragma unroll
    for (int j = 0; j < VS; ++j) acc[j] = 0.0f;
    // Content term Yc = Q·λc.
    const float* qrow = q + pix * c + h * k;
    for (int kk = 0; kk < k; kk += 4) {
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qrow + kk));
        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float* lr = lam_s + (kk + u) * VS;
#pragma unroll
            for (int j = 0; j < VS; j += 4) {
                const float4 l4 = *reinterpret_cast<const float4*>(lr + j);
                acc[j] = fmaf(qv[u], l4.x, acc[j]);
                acc[j + 1] = fmaf(qv[u], l4.y, acc[j + 1]);
                acc[j + 2] = fmaf(qv[u], l4.z, acc[j + 2]);
                acc[j + 3] = fmaf(qv[u], l4.w, acc[j + 3]);
            }
        }
    }
    // Position term: the Q·b column first, then the 225 taps in (ky, kx) order.
    const float* arow = a + (pix * kHeads + h) * (int64_t)a_stride;
    const float4 last = __ldg(reinterpret_cast<const float4*>(arow + kTaps - 1));  // tap 224, Q·b, 0, 0
#pragma unroll
    for (int j = 0; j < VS; ++j) acc[j] += last.y;
    const float* hbase = halo + (ty * kHalo + tx) * HS;
    auto tap = [&](int d, float coef) {
        const int ky = d / kWin, kx = d - ky * kWin;
        const float* hr = hbase + (ky * kHalo + kx) * HS;
#pragma unroll
        for (int j = 0; j < VS; j += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(hr + j);
            acc[j] = fmaf(coef, v4.x, acc[j]);
            acc[j + 1] = fmaf(coef, v4.y, acc[j + 1]);
            acc[j + 2] = fmaf(coef, v4.z, acc[j + 2]);
            acc[j + 3] = fmaf(coef, v4.w, acc[j + 3]);
        }
    };
    // The coefficients stream from global memory four taps at a time; the next group's load is
    // issued before this group's FMAs so its latency hides behind them.
    float4 c4 = __ldg(reinterpret_cast<const float4*>(arow));
#pragma unroll 1
    for (int d = 0; d < kTaps - 1; d += 4) {
        const float4 cur = c4;
        if (d + 4 < kTaps - 1) c4 = __ldg(reinterpret_cast<const float4*>(arow + d + 4));
        tap(d, cur.x);
        tap(d + 1, cur.y);
        tap(d + 2, cur.z);
        tap(d + 3, cur.w);
    }
    tap(kTaps - 1, last.x);
    float* o = out + pix * c + h * k + j0;
#pragma unroll
    for (int j = 0; j < VS; j += 4) {
        float4 r = *reinterpret_cast<float4*>(o + j);
        r.x += acc[j];
        r.y += acc[j + 1];
        r.z += acc[j + 2];
        r.w += acc[j + 3];
        *reinterpret_cast<float4*>(o + j) = r;
    }
}

// ---------------------------------------------------------------- cross-λ

template <int VS>
__global__ void __launch_bounds__(512, 1)
    cross_position_kernel(const float* __restrict__ q, const float* __restrict__ e_table,
                          const float* __restrict__ lam, const float* __restrict__ vtab, int period, int64_t hw,
                          int k, float* __restrict__ out) {
    extern __shared__ float4 smem4[];
    float* lam_s = reinterpret_cast<float*>(smem4);  // [k][VS]
    float* v_s = lam_s + k * VS;                     // [kTokens][VS]
    const int item = blockIdx.z, j0 = blockIdx.y * VS;
    const int branch = item % period;
    const float* lam_b = lam + (int64_t)branch * k * k;
    const float* v_b = vtab + (int64_t)branch * kTokens * k;
    const int tid = threadIdx.x;
    for (int i = tid; i < k * VS; i += 512) {
        const int kk = i / VS, j = i - kk * VS;
        lam_s[i] = __ldg(lam_b + (int64_t)kk * k + j0 + j);
    }
    for (int i = tid; i < kTokens * VS; i += 512) {
        const int m = i / VS, j = i - m * VS;
        v_s[i] = __ldg(v_b + (int64_t)m * k + j0 + j);
    }
    __syncthreads();
    const int h = tid & 7;
    const int64_t p = (int64_t)blockIdx.x * 64 + (tid >> 3);
    if (p >= hw) return;
    const int c = kHeads * k;
    const int64_t pix = (int64_t)item * hw + p;
    const float* qrow = q + pix * c + h * k;
    const float* erow = e_table + p * kTokens * k;

    // B[m] = Q_h · E[p, m]
    float bm[kTokens];
#pragma unroll
    for (int m = 0; m < kTokens; ++m) bm[m] = 0.0f;
    for (int kk = 0; kk < k; kk += 4) {
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qrow + kk));
#pragma unroll
        for (int m = 0; m < kTokens; ++m) {
            const float4 e4 = __ldg(reinterpret_cast<const float4*>(erow + m * k + kk));
            bm[m] = fmaf(q4.x, e4.x, bm[m]);
            bm[m] = fmaf(q4.y, e4.y, bm[m]);
            bm[m] = fmaf(q4.z, e4.z, bm[m]);
            bm[m] = fmaf(q4.w, e4.w, bm[m]);
        }
    }
    float acc[VS];
#pragma unroll
    for (int j = 0; j < VS; ++j) acc[j] = 0.0f;
    for (int kk = 0; kk < k; kk += 4) {
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(qrow + kk));
        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float* lr = lam_s + (kk + u) * VS;
#pragma unroll
            for (int j = 0; j < VS; j += 4) {
                const float4 l4 = *reinterpret_cast<const float4*>(lr + j);
                acc[j] = fmaf(qv[u], l4.x, acc[j]);
                acc[j + 1] = fmaf(qv[u], l4.y, acc[j + 1]);
                acc[j + 2] = fmaf(qv[u], l4.z, acc[j + 2]);
                acc[j + 3] = fmaf(qv[u], l4.w, acc[j + 3]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kTokens; ++m) {
        const float* vr = v_s + m * VS;
#pragma unroll
        for (int j = 0; j < VS; ++j) acc[j] = fmaf(bm[m], vr[j], acc[j]);
    }
    float* o = out + pix * c + h * k + j0;
#pragma unroll
    for (int j = 0; j < VS; j += 4) {
        float4 r = *reinterpret_cast<float4*>(o + j);
        r.x += acc[j];
        r.y += acc[j + 1];
        r.z += acc[j + 2];
        r.w += acc[j + 3];
        *reinterpret_cast<float4*>(o + j) = r;
    }
}

// Value channels per CTA slice: the largest supported width dividing k.
int slice_width(int64_t k) {
    for (int vs : {80, 40, 32, 16, 8})
        if (k % vs == 0) return vs;
    return 0;
}

template <typename F>
void dispatch_vs(int vs, F&& f) {
    switch (vs) {
        case 80: f(std::integral_constant<int, 80>{}); break;
        case 40: f(std::integral_constant<int, 40>{}); break;
        case 32: f(std::integral_constant<int, 32>{}); break;
        case 16: f(std::integral_constant<int, 16>{}); break;
        case 8: f(std::integral_constant<int, 8>{}); break;
        default: fail(MBX_ERR_INVALID_ARGUMENT, "lambda: head width must be a multiple of 8");
    }
}

template <typename K>
void set_smem(K kernel, int bytes) {
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
               "lambda smem attribute");
}

}  // namespace

int64_t lambda_chunks(int64_t rows) { return (rows + kLamChunk - 1) / kLamChunk; }

void launch_lambda_content(mbx_ctx* ctx, const float* keys, int64_t ks, const float* vals, int64_t vs,
                           int64_t items, int64_t rows, int64_t k, int64_t vd, float* pmax, float* plam,
                           float* psum, float* lam) {
    MBX_REQUIRE(k >= 1 && k <= 1024 && vd >= 1, "lambda: bad widths");
    MBX_REQUIRE(items < 65536, "lambda: too many items");
    const int64_t chunks = lambda_chunks(rows);
    MBX_REQUIRE(chunks < (int64_t(1) << 31), "lambda: too many rows");
    lambda_colmax_kernel<<<dim3((unsigned)chunks, (unsigned)items), (unsigned)std::min<int64_t>(k, 256), 0,
                           ctx->stream>>>(keys, ks, rows, (int)k, (int)chunks, pmax);
    after_launch(ctx, "lambda_colmax");
    const int slabs = (int)((vd + kLamCols - 1) / kLamCols);
    const int groups = (int)(std::min<int64_t>(vd, kLamCols) + 7) / 8;
    const int threads = (int)k * groups;
    MBX_REQUIRE(threads <= 1024, "lambda: k too large for one CTA");
    const int smem = (int)(k + kLamRows * k + kLamRows * kLamCols) * 4;
    static bool configured = false;
    if (!configured) {
        set_smem(lambda_partial_kernel, 64 * 1024);
        configured = true;
    }
    MBX_REQUIRE(smem <= 64 * 1024, "lambda: k too large for the staging tile");
    lambda_partial_kernel<<<dim3((unsigned)chunks, (unsigned)items, (unsigned)slabs), threads, smem, ctx->stream>>>(
        keys, ks, vals, vs, rows, (int)k, (int)vd, (int)chunks, pmax, plam, psum);
    after_launch(ctx, "lambda_partial");
    lambda_finalize_kernel<<<grid_for(ctx, items * k * vd, 256), 256, 0, ctx->stream>>>(plam, psum, items, (int)k,
                                                                                        (int)vd, (int)chunks, lam);
    after_launch(ctx, "lambda_finalize");
}

void launch_self_position(mbx_ctx* ctx, const float* q, const float* lam, const float* a, int64_t a_stride,
                          const float* v, int64_t v_stride, int64_t n, int64_t h, int64_t w, int64_t k, float* out) {
    const int vs = slice_width(k);
    MBX_REQUIRE(vs > 0, "self lambda: head width must be a multiple of 8");
    const int tiles_x = (int)((w + kTile - 1) / kTile), tiles_y = (int)((h + kTile - 1) / kTile);
    MBX_REQUIRE(n < 65536 && (int64_t)tiles_x * tiles_y < (int64_t(1) << 31), "self lambda: grid too large");
    dispatch_vs(vs, [&](auto c) {
        constexpr int VS = decltype(c)::value;
        const int smem = (kHalo * kHalo * (VS + 4) + (int)k * VS) * 4;
        MBX_REQUIRE(smem <= 227 * 1024, "self lambda: head width too large");
        auto kern = self_position_kernel<VS>;
        static bool configured = false;
        if (!configured) {
            set_smem(kern, 227 * 1024);
            configured = true;
        }
        kern<<<dim3((unsigned)(tiles_x * tiles_y), (unsigned)(k / VS), (unsigned)n), 512, smem, ctx->stream>>>(
            q, lam, a, (int)a_stride, v, v_stride, (int)h, (int)w, (int)k, tiles_x, out);
    });
    after_launch(ctx, "self_lambda_position");
}

void launch_cross_position(mbx_ctx* ctx, const float* q, const float* e_table, const float* lam, const float* vtab,
                           int64_t period, int64_t n, int64_t hw, int64_t k, float* out) {
    const int vs = slice_width(k);
    MBX_REQUIRE(vs > 0, "cross lambda: head width must be a multiple of 8");
    MBX_REQUIRE(n < 65536 && (hw + 63) / 64 < (int64_t(1) << 31), "cross lambda: grid too large");
    dispatch_vs(vs, [&](auto c) {
        constexpr int VS = decltype(c)::value;
        const int smem = ((int)k * VS + kTokens * VS) * 4;
        MBX_REQUIRE(smem <= 227 * 1024, "cross lambda: head width too large");
        auto kern = cross_position_kernel<VS>;
        static bool configured = false;
        if (!configured) {
            set_smem(kern, 227 * 1024);
            configured = true;
        }
        kern<<<dim3((unsigned)((hw + 63) / 64), (unsigned)(k / VS), (unsigned)n), 512, smem, ctx->stream>>>(
            q, e_table, lam, vtab, (int)period, hw, (int)k, out);
    });
    after_launch(ctx, "cross_lambda_position");
}

}  // namespace mbx
