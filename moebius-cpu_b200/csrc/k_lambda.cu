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
//    8×8 pixel tile and v-slice; a thread owns one pixel, two heads and half of
//    the VS value channels in registers, so A is read once per slice, the
//    window of V (22×22 pixels × VS channels) comes from shared memory and each
//    V vector read there serves both heads.
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
constexpr int kColmaxThreads = 1024;        // column-max CTA: row slices × columns
constexpr int kLamCols = 40;                // λ columns per CTA of the partial pass
constexpr int kTokens = 10;

// ---------------------------------------------------------------- content λ

// Per 256-row chunk column maxima. The CTA's threads split into P = max(1, 1024 / k) row slices
// of k columns each (max is exact, so the split does not change the result), then fold the
// slices in shared memory.
__global__ void __launch_bounds__(kColmaxThreads) lambda_colmax_kernel(const float* __restrict__ keys, int64_t ks,
                                                                        int64_t rows, int k, int chunks,
                                                                        float* __restrict__ pmax) {
    __shared__ float part[kColmaxThreads];
    const int chunk = blockIdx.x, item = blockIdx.y;
    const float* kb = keys + (int64_t)item * rows * ks;
    const int64_t r0 = (int64_t)chunk * kLamChunk;
    const int64_t r1 = r0 + kLamChunk < rows ? r0 + kLamChunk : rows;
    const int slices = k < kColmaxThreads ? kColmaxThreads / k : 1;
    for (int c0 = 0; c0 < k; c0 += kColmaxThreads) {
        const int cols = min(k - c0, kColmaxThreads);
        const int p = threadIdx.x / cols, kk = c0 + threadIdx.x - p * cols;
        float m = -FLT_MAX;
        if (p < slices) {
#pragma unroll 8
            for (int64_t r = r0 + p; r < r1; r += slices) m = fmaxf(m, __ldg(kb + r * ks + kk));
        }
        part[threadIdx.x] = m;
        __syncthreads();
        if (threadIdx.x < cols) {
            float v = part[threadIdx.x];
            for (int q = 1; q < slices; ++q) v = fmaxf(v, part[q * cols + threadIdx.x]);
            pmax[((int64_t)item * chunks + chunk) * k + c0 + threadIdx.x] = v;
        }
        __syncthreads();
    }
}

// Block: k·G threads (G = column groups of 8 in this CTA's slab); thread (kk, g)
// accumulates λ[kk][j0 + 8g .. +8] over the chunk's rows. The rows are staged in shared memory
// `stage` at a time (the whole chunk where it fits), so the loads of a stage are all in flight
// together. VEC: 128-bit staging loads (k, vd and both row strides multiples of 4, 16-byte aligned).
template <bool VEC>
__global__ void lambda_partial_kernel(const float* __restrict__ keys, int64_t ks, const float* __restrict__ vals,
                                      int64_t vs, int64_t rows, int k, int vd, int chunks, int stage,
                                      const float* __restrict__ pmax, float* __restrict__ plam,
                                      float* __restrict__ psum) {
    extern __shared__ float4 smem_v[];  // float4: the staging tiles take 128-bit stores
    float* smem = reinterpret_cast<float*>(smem_v);
    const int chunk = blockIdx.x, item = blockIdx.y, j0 = blockIdx.z * kLamCols;
    const int ncols = vd - j0 < kLamCols ? vd - j0 : kLamCols;
    const int groups = (ncols + 7) / 8;
    float* colmax = smem;                          // [k]
    float* e_t = colmax + k;                       // [stage][k]
    float* v_t = e_t + stage * k;                  // [stage][kLamCols]
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
    for (int64_t rt = r0; rt < r1; rt += stage) {
        const int nr = (int)(r1 - rt < stage ? r1 - rt : stage);
        if constexpr (VEC) {
            const int k4 = k >> 2;
#pragma unroll 4
            for (int i = tid; i < nr * k4; i += nthr) {
                const int rr = i / k4, c = 4 * (i - rr * k4);
                const float4 kv = __ldg(reinterpret_cast<const float4*>(kb + (rt + rr) * ks + c));
                *reinterpret_cast<float4*>(e_t + rr * k + c) =
                    make_float4(expf(kv.x - colmax[c]), expf(kv.y - colmax[c + 1]), expf(kv.z - colmax[c + 2]),
                                expf(kv.w - colmax[c + 3]));
            }
            constexpr int kCols4 = kLamCols / 4;
#pragma unroll 4
            for (int i = tid; i < nr * kCols4; i += nthr) {
                const int rr = i / kCols4, c = 4 * (i - rr * kCols4);
                *reinterpret_cast<float4*>(v_t + rr * kLamCols + c) =
                    c < ncols ? __ldg(reinterpret_cast<const float4*>(vb + (rt + rr) * vs + j0 + c))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        } else {
#pragma unroll 4
            for (int i = tid; i < nr * k; i += nthr) {
                const int rr = i / k, c = i - rr * k;
                e_t[rr * k + c] = expf(__ldg(kb + (rt + rr) * ks + c) - colmax[c]);
            }
#pragma unroll 4
            for (int i = tid; i < nr * kLamCols; i += nthr) {
                const int rr = i / kLamCols, c = i - rr * kLamCols;
                v_t[rr * kLamCols + c] = c < ncols ? __ldg(vb + (rt + rr) * vs + j0 + c) : 0.0f;
            }
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

// Halo row stride in floats: at least VS and ≡ 8 or 24 (mod 32), so the eight 16-byte reads of a
// warp (four neighbouring pixels × two interleaved float4 groups) fall in distinct banks.
__host__ __device__ constexpr int halo_stride(int vs) { return vs + (vs % 16 == 0 ? 8 : 0); }

// Shared layout: V window [kHalo²][HS], then λc slice [k][VS]. A thread owns one pixel, two heads
// (2·hp and 2·hp + 1) and every other float4 group of the VS value channels (groups of parity jh),
// so each V vector read from shared memory feeds both heads: 8 FMAs per 16-byte read.
template <int VS>
__global__ void __launch_bounds__(512, 1)
    self_position_kernel(const float* __restrict__ q, const float* __restrict__ lam, const float* __restrict__ a,
                         int a_stride, const float* __restrict__ v, int64_t v_stride, int H, int W, int k,
                         int tiles_x, float* __restrict__ out) {
    static_assert(VS % 8 == 0, "a thread takes every other float4 group of the slice");
    constexpr int HS = halo_stride(VS);
    constexpr int NG = VS / 8;  // float4 groups per thread
    extern __shared__ float4 smem4[];
    float* halo = reinterpret_cast<float*>(smem4);
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

    // Lane = (pixel of four, group parity, head pair); warp = half a tile row.
    const int lane = tid & 31, wid = tid >> 5;
    const int hp = lane & 3, jh = (lane >> 2) & 1;
    const int ty = wid >> 1, tx = (wid & 1) * 4 + (lane >> 3);
    const int y = ty0 + ty, x = tx0 + tx;
    if (y >= H || x >= W) return;
    const int64_t pix = item_px + (int64_t)y * W + x;
    const int h0 = 2 * hp;

    // acc0 / acc1: heads h0 / h0 + 1; element 4·i + e is value channel j0 + 8·i + 4·jh + e.
    float acc0[4 * NG], acc1[4 * NG];
#pragma unroll
    for (int j = 0; j < 4 * NG; ++j) acc0[j] = acc1[j] = 0.0f;
    // Content term Yc = Q·λc.
    const float* q0 = q + pix * c + h0 * k;
    const float* q1 = q0 + k;
    // k is a multiple of 8: two steps per trip keep two groups of loads in flight.
#pragma unroll 2
    for (int kk = 0; kk < k; kk += 4) {
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(q0 + kk));
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(q1 + kk));
        const float qa[4] = {a4.x, a4.y, a4.z, a4.w}, qb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float* lr = lam_s + (kk + u) * VS + 4 * jh;
#pragma unroll
            for (int i = 0; i < NG; ++i) {
                const float4 l4 = *reinterpret_cast<const float4*>(lr + 8 * i);
                acc0[4 * i] = fmaf(qa[u], l4.x, acc0[4 * i]);
                acc0[4 * i + 1] = fmaf(qa[u], l4.y, acc0[4 * i + 1]);
                acc0[4 * i + 2] = fmaf(qa[u], l4.z, acc0[4 * i + 2]);
                acc0[4 * i + 3] = fmaf(qa[u], l4.w, acc0[4 * i + 3]);
                acc1[4 * i] = fmaf(qb[u], l4.x, acc1[4 * i]);
                acc1[4 * i + 1] = fmaf(qb[u], l4.y, acc1[4 * i + 1]);
                acc1[4 * i + 2] = fmaf(qb[u], l4.z, acc1[4 * i + 2]);
                acc1[4 * i + 3] = fmaf(qb[u], l4.w, acc1[4 * i + 3]);
            }
        }
    }
    // Position term: the Q·b column first, then the 225 taps in (ky, kx) order.
    const float* arow0 = a + (pix * kHeads + h0) * (int64_t)a_stride;
    const float* arow1 = arow0 + a_stride;
    const float4 last0 = __ldg(reinterpret_cast<const float4*>(arow0 + kTaps - 1));  // tap 224, Q·b, 0, 0
    const float4 last1 = __ldg(reinterpret_cast<const float4*>(arow1 + kTaps - 1));
#pragma unroll
    for (int j = 0; j < 4 * NG; ++j) {
        acc0[j] += last0.y;
        acc1[j] += last1.y;
    }
    const float* hbase = halo + (ty * kHalo + tx) * HS + 4 * jh;
    // Tap d (0 ≤ d < 225) of a block of window rows starting at row `row0`: `dd` = d − 15·row0 is a
    // compile-time constant inside the unrolled blocks below, so the window offset is an immediate.
    auto tap = [&](const float* hrow0, int dd, float ca, float cb) {
        const int ky = dd / kWin, kx = dd - ky * kWin;
        const float* hr = hrow0 + (ky * kHalo + kx) * HS;
#pragma unroll
        for (int i = 0; i < NG; ++i) {
            const float4 v4 = *reinterpret_cast<const float4*>(hr + 8 * i);
            acc0[4 * i] = fmaf(ca, v4.x, acc0[4 * i]);
            acc0[4 * i + 1] = fmaf(ca, v4.y, acc0[4 * i + 1]);
            acc0[4 * i + 2] = fmaf(ca, v4.z, acc0[4 * i + 2]);
            acc0[4 * i + 3] = fmaf(ca, v4.w, acc0[4 * i + 3]);
            acc1[4 * i] = fmaf(cb, v4.x, acc1[4 * i]);
            acc1[4 * i + 1] = fmaf(cb, v4.y, acc1[4 * i + 1]);
            acc1[4 * i + 2] = fmaf(cb, v4.z, acc1[4 * i + 2]);
            acc1[4 * i + 3] = fmaf(cb, v4.w, acc1[4 * i + 3]);
        }
    };
    // Taps in (ky, kx) order, in blocks of 60 (4 window rows, 15 coefficient float4s): three full
    // blocks, then 44 taps and tap 224 (from last0 / last1). Inside a block everything is unrolled;
    // the coefficients stream from global memory a float4 (four taps) at a time, the next one
    // loaded before the current four taps' FMAs.
    constexpr int kBlock = 4 * kWin;
    if constexpr (NG > 5) {
        // 80-channel slices: 80 accumulators leave no registers for the unrolled blocks' window
        // loads in flight (it spilled), so one float4 of coefficients (four taps) per iteration.
        float4 ca4 = __ldg(reinterpret_cast<const float4*>(arow0));
        float4 cb4 = __ldg(reinterpret_cast<const float4*>(arow1));
#pragma unroll 1
        for (int d = 0; d < kTaps - 1; d += 4) {
            const float4 ca = ca4, cb = cb4;
            if (d + 4 < kTaps - 1) {
                ca4 = __ldg(reinterpret_cast<const float4*>(arow0 + d + 4));
                cb4 = __ldg(reinterpret_cast<const float4*>(arow1 + d + 4));
            }
            tap(hbase, d, ca.x, cb.x);
            tap(hbase, d + 1, ca.y, cb.y);
            tap(hbase, d + 2, ca.z, cb.z);
            tap(hbase, d + 3, ca.w, cb.w);
        }
        tap(hbase, kTaps - 1, last0.x, last1.x);
    } else {
#pragma unroll 1
    for (int blk = 0; blk < 3; ++blk) {
        const float* hrow0 = hbase + blk * 4 * kHalo * HS;
        const float* c0p = arow0 + blk * kBlock;
        const float* c1p = arow1 + blk * kBlock;
        float4 ca4 = __ldg(reinterpret_cast<const float4*>(c0p));
        float4 cb4 = __ldg(reinterpret_cast<const float4*>(c1p));
#pragma unroll
        for (int g = 0; g < kBlock / 4; ++g) {
            const float4 ca = ca4, cb = cb4;
            if (g + 1 < kBlock / 4) {
                ca4 = __ldg(reinterpret_cast<const float4*>(c0p + 4 * (g + 1)));
                cb4 = __ldg(reinterpret_cast<const float4*>(c1p + 4 * (g + 1)));
            }
            tap(hrow0, 4 * g, ca.x, cb.x);
            tap(hrow0, 4 * g + 1, ca.y, cb.y);
            tap(hrow0, 4 * g + 2, ca.z, cb.z);
            tap(hrow0, 4 * g + 3, ca.w, cb.w);
        }
    }
    {
        const float* hrow0 = hbase + 12 * kHalo * HS;
        const float* c0p = arow0 + 3 * kBlock;
        const float* c1p = arow1 + 3 * kBlock;
        float4 ca4 = __ldg(reinterpret_cast<const float4*>(c0p));
        float4 cb4 = __ldg(reinterpret_cast<const float4*>(c1p));
#pragma unroll
        for (int g = 0; g < 11; ++g) {
            const float4 ca = ca4, cb = cb4;
            if (g + 1 < 11) {
                ca4 = __ldg(reinterpret_cast<const float4*>(c0p + 4 * (g + 1)));
                cb4 = __ldg(reinterpret_cast<const float4*>(c1p + 4 * (g + 1)));
            }
            tap(hrow0, 4 * g, ca.x, cb.x);
            tap(hrow0, 4 * g + 1, ca.y, cb.y);
            tap(hrow0, 4 * g + 2, ca.z, cb.z);
            tap(hrow0, 4 * g + 3, ca.w, cb.w);
        }
        tap(hrow0, 44, last0.x, last1.x);  // tap 224
    }
    }
    float* o0 = out + pix * c + h0 * k + j0 + 4 * jh;
    float* o1 = o0 + k;
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        float4 r = *reinterpret_cast<float4*>(o0 + 8 * i);
        r.x += acc0[4 * i];
        r.y += acc0[4 * i + 1];
        r.z += acc0[4 * i + 2];
        r.w += acc0[4 * i + 3];
        *reinterpret_cast<float4*>(o0 + 8 * i) = r;
        float4 t = *reinterpret_cast<float4*>(o1 + 8 * i);
        t.x += acc1[4 * i];
        t.y += acc1[4 * i + 1];
        t.z += acc1[4 * i + 2];
        t.w += acc1[4 * i + 3];
        *reinterpret_cast<float4*>(o1 + 8 * i) = t;
    }
}

// ---------------------------------------------------------------- cross-λ

// Shared layout: λc slice [k][VS], then the branch's values [kTokens][VS]. Threads map as in
// self_position_kernel: one pixel, two heads, every other float4 group of the slice.
template <int VS>
__global__ void __launch_bounds__(512, 1)
    cross_position_kernel(const float* __restrict__ q, const float* __restrict__ e_table,
                          const float* __restrict__ lam, const float* __restrict__ vtab, int period, int64_t hw,
                          int k, float* __restrict__ out) {
    static_assert(VS % 8 == 0, "a thread takes every other float4 group of the slice");
    constexpr int NG = VS / 8;
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
    const int lane = tid & 31, wid = tid >> 5;
    const int hp = lane & 3, jh = (lane >> 2) & 1;
    const int64_t p = (int64_t)blockIdx.x * 64 + wid * 4 + (lane >> 3);
    if (p >= hw) return;
    const int c = kHeads * k;
    const int h0 = 2 * hp;
    const int64_t pix = (int64_t)item * hw + p;
    const float* q0 = q + pix * c + h0 * k;
    const float* q1 = q0 + k;
    const float* erow = e_table + p * kTokens * k;

    // B[m] = Q_h · E[p, m] for both heads.
    float bm0[kTokens], bm1[kTokens];
#pragma unroll
    for (int m = 0; m < kTokens; ++m) bm0[m] = bm1[m] = 0.0f;
    auto b_step = [&](int kk) {
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(q0 + kk));
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(q1 + kk));
#pragma unroll
        for (int m = 0; m < kTokens; ++m) {
            const float4 e4 = __ldg(reinterpret_cast<const float4*>(erow + m * k + kk));
            bm0[m] = fmaf(a4.x, e4.x, bm0[m]);
            bm0[m] = fmaf(a4.y, e4.y, bm0[m]);
            bm0[m] = fmaf(a4.z, e4.z, bm0[m]);
            bm0[m] = fmaf(a4.w, e4.w, bm0[m]);
            bm1[m] = fmaf(b4.x, e4.x, bm1[m]);
            bm1[m] = fmaf(b4.y, e4.y, bm1[m]);
            bm1[m] = fmaf(b4.z, e4.z, bm1[m]);
            bm1[m] = fmaf(b4.w, e4.w, bm1[m]);
        }
    };
    if constexpr (NG <= 5) {
        // k is a multiple of 8: two steps per trip keep two groups of table loads in flight (the
        // 80-channel slices have no registers to spare for it).
#pragma unroll 2
        for (int kk = 0; kk < k; kk += 4) b_step(kk);
    } else {
        for (int kk = 0; kk < k; kk += 4) b_step(kk);
    }
    // acc0 / acc1: heads h0 / h0 + 1; element 4·i + e is value channel j0 + 8·i + 4·jh + e.
    float acc0[4 * NG], acc1[4 * NG];
#pragma unroll
    for (int j = 0; j < 4 * NG; ++j) acc0[j] = acc1[j] = 0.0f;
    for (int kk = 0; kk < k; kk += 4) {
        const float4 a4 = __ldg(reinterpret_cast<const float4*>(q0 + kk));
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(q1 + kk));
        const float qa[4] = {a4.x, a4.y, a4.z, a4.w}, qb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float* lr = lam_s + (kk + u) * VS + 4 * jh;
#pragma unroll
            for (int i = 0; i < NG; ++i) {
                const float4 l4 = *reinterpret_cast<const float4*>(lr + 8 * i);
                acc0[4 * i] = fmaf(qa[u], l4.x, acc0[4 * i]);
                acc0[4 * i + 1] = fmaf(qa[u], l4.y, acc0[4 * i + 1]);
                acc0[4 * i + 2] = fmaf(qa[u], l4.z, acc0[4 * i + 2]);
                acc0[4 * i + 3] = fmaf(qa[u], l4.w, acc0[4 * i + 3]);
                acc1[4 * i] = fmaf(qb[u], l4.x, acc1[4 * i]);
                acc1[4 * i + 1] = fmaf(qb[u], l4.y, acc1[4 * i + 1]);
                acc1[4 * i + 2] = fmaf(qb[u], l4.z, acc1[4 * i + 2]);
                acc1[4 * i + 3] = fmaf(qb[u], l4.w, acc1[4 * i + 3]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kTokens; ++m) {
        const float* vr = v_s + m * VS + 4 * jh;
#pragma unroll
        for (int i = 0; i < NG; ++i) {
            const float4 v4 = *reinterpret_cast<const float4*>(vr + 8 * i);
            acc0[4 * i] = fmaf(bm0[m], v4.x, acc0[4 * i]);
            acc0[4 * i + 1] = fmaf(bm0[m], v4.y, acc0[4 * i + 1]);
            acc0[4 * i + 2] = fmaf(bm0[m], v4.z, acc0[4 * i + 2]);
            acc0[4 * i + 3] = fmaf(bm0[m], v4.w, acc0[4 * i + 3]);
            acc1[4 * i] = fmaf(bm1[m], v4.x, acc1[4 * i]);
            acc1[4 * i + 1] = fmaf(bm1[m], v4.y, acc1[4 * i + 1]);
            acc1[4 * i + 2] = fmaf(bm1[m], v4.z, acc1[4 * i + 2]);
            acc1[4 * i + 3] = fmaf(bm1[m], v4.w, acc1[4 * i + 3]);
        }
    }
    float* o0 = out + pix * c + h0 * k + j0 + 4 * jh;
    float* o1 = o0 + k;
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        float4 r = *reinterpret_cast<float4*>(o0 + 8 * i);
        r.x += acc0[4 * i];
        r.y += acc0[4 * i + 1];
        r.z += acc0[4 * i + 2];
        r.w += acc0[4 * i + 3];
        *reinterpret_cast<float4*>(o0 + 8 * i) = r;
        float4 t = *reinterpret_cast<float4*>(o1 + 8 * i);
        t.x += acc1[4 * i];
        t.y += acc1[4 * i + 1];
        t.z += acc1[4 * i + 2];
        t.w += acc1[4 * i + 3];
        *reinterpret_cast<float4*>(o1 + 8 * i) = t;
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
    ensure_smem_limit(reinterpret_cast<const void*>(kernel), bytes, "lambda smem attribute");
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
    lambda_colmax_kernel<<<dim3((unsigned)chunks, (unsigned)items), kColmaxThreads, 0, ctx->stream>>>(
        keys, ks, rows, (int)k, (int)chunks, pmax);
    after_launch(ctx, "lambda_colmax");
    const int slabs = (int)((vd + kLamCols - 1) / kLamCols);
    const int groups = (int)(std::min<int64_t>(vd, kLamCols) + 7) / 8;
    const int threads = (int)k * groups;
    MBX_REQUIRE(threads <= 1024, "lambda: k too large for one CTA");
    // Rows per staging pass: the whole chunk where its exponentials and values fit (in 100 KB, for
    // two CTAs per SM, when the grid is larger than one CTA per SM), else the largest power of two
    // down to 32.
    const int64_t ctas = chunks * items * slabs;
    const int limit = ctas <= ctx->sm_count ? 227 * 1024 : 100 * 1024;
    int stage = kLamChunk;
    auto stage_bytes = [&](int r) { return (int)(k + (int64_t)r * k + (int64_t)r * kLamCols) * 4; };
    while (stage > 32 && stage_bytes(stage) > limit) stage /= 2;
    const int smem = stage_bytes(stage);
    MBX_REQUIRE(smem <= 227 * 1024, "lambda: k too large for the staging tile");
    const bool vec = k % 4 == 0 && vd % 4 == 0 && ks % 4 == 0 && vs % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(keys) & 15) == 0 && (reinterpret_cast<uintptr_t>(vals) & 15) == 0;
    auto launch = [&](auto kern) {
        set_smem(kern, 227 * 1024);
        kern<<<dim3((unsigned)chunks, (unsigned)items, (unsigned)slabs), threads, smem, ctx->stream>>>(
            keys, ks, vals, vs, rows, (int)k, (int)vd, (int)chunks, stage, pmax, plam, psum);
    };
    if (vec) launch(lambda_partial_kernel<true>);
    else launch(lambda_partial_kernel<false>);
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
        const int smem = (kHalo * kHalo * halo_stride(VS) + (int)k * VS) * 4;
        MBX_REQUIRE(smem <= 227 * 1024, "self lambda: head width too large");
        auto kern = self_position_kernel<VS>;
        set_smem(kern, 227 * 1024);
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
        set_smem(kern, 227 * 1024);
        kern<<<dim3((unsigned)((hw + 63) / 64), (unsigned)(k / VS), (unsigned)n), 512, smem, ctx->stream>>>(
            q, e_table, lam, vtab, (int)period, hw, (int)k, out);
    });
    after_launch(ctx, "cross_lambda_position");
}

}  // namespace mbx
