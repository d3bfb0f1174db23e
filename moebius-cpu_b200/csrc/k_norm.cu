// GroupNorm (stats pass + fused apply) and LayerNorm for NHWC float32.
//
// GroupNorm follows the reference's numerics (src/engine/norm.rs:57-129):
// per-channel f32 partial Σy, Σy² over 256-pixel chunks (y = x + add[item]),
// folded into f64 per group, chunk partials summed in f64 in chunk order
// (deterministic: no atomics), var = E[y²] − mean² clamped at 0. The apply
// pass is out = [SiLU](x·scale + shift) (+ residual) with 128-bit accesses.
#include <algorithm>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kGnChunk = 256;   // pixels per stats task (the reference's STATS_CHUNK)
constexpr int kGnThreads = 256;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// One CTA per (pixel chunk, item, channel slice of whole groups): small maps (few chunks) still
// fill the GPU. V = 4 (float4 lanes over channels) or 1.
template <int V, bool ADD>
__global__ void __launch_bounds__(kGnThreads) gn_partials_kernel(const float* __restrict__ x, int64_t hw, int c,
                                                                 int groups, int cs, const float* __restrict__ add,
                                                                 double* __restrict__ part) {
    extern __shared__ float red[];  // [2][rows][cs]
    const int cv = cs / V;
    const int64_t chunk = blockIdx.x, b = blockIdx.y, chunks = gridDim.x;
    const int c0 = blockIdx.z * cs;
    const int64_t p0 = chunk * kGnChunk;
    const int npx = (int)(hw - p0 < kGnChunk ? hw - p0 : kGnChunk);
    const int t = threadIdx.x;
    const bool narrow = cv <= kGnThreads;
    const int rows = narrow ? kGnThreads / cv : 1;
    const int r = narrow ? t / cv : 0;
    float* rs = red;
    float* rq = red + rows * cs;
    const float* xb = x + (b * hw + p0) * (int64_t)c + c0;
    if (r < rows) {
        for (int j = narrow ? t % cv : t; j < cv; j += narrow ? cv : kGnThreads) {
            float s[V], q[V], a[V];
#pragma unroll
            for (int k = 0; k < V; ++k) {
                s[k] = 0.0f;
                q[k] = 0.0f;
                a[k] = ADD ? add[b * c + c0 + j * V + k] : 0.0f;
            }
#pragma unroll 8
            for (int p = r; p < npx; p += rows) {
                float v[V];
                if constexpr (V == 4) {
                    const float4 f = __ldg(reinterpret_cast<const float4*>(xb + (int64_t)p * c) + j);
                    v[0] = f.x;
                    v[1] = f.y;
                    v[2] = f.z;
                    v[3] = f.w;
                } else {
                    v[0] = __ldg(xb + (int64_t)p * c + j);
                }
#pragma unroll
                for (int k = 0; k < V; ++k) {
                    const float y = ADD ? v[k] + a[k] : v[k];
                    s[k] += y;
                    q[k] = fmaf(y, y, q[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < V; ++k) {
                rs[r * cs + j * V + k] = s[k];
                rq[r * cs + j * V + k] = q[k];
            }
        }
    }
    __syncthreads();
    // Per-channel chunk partial (f32, in row order), kept in row 0.
    for (int ch = t; ch < cs; ch += kGnThreads) {
        float s = rs[ch], q = rq[ch];
        for (int rr = 1; rr < rows; ++rr) {
            s += rs[rr * cs + ch];
            q += rq[rr * cs + ch];
        }
        rs[ch] = s;
        rq[ch] = q;
    }
    __syncthreads();
    // f64 fold per group (src/engine/norm.rs:78-80).
    const int cg = c / groups;
    const int g0 = c0 / cg;
    for (int gl = t; gl < cs / cg; gl += kGnThreads) {
        double ss = 0.0, qq = 0.0;
        for (int ch = gl * cg; ch < (gl + 1) * cg; ++ch) {
            ss += (double)rs[ch];
            qq += (double)rq[ch];
        }
        double* dst = part + ((b * chunks + chunk) * groups + g0 + gl) * 2;
        dst[0] = ss;
        dst[1] = qq;
    }
}

// One CTA per item: chunk partials → mean / rstd → per-channel scale, shift
// (src/engine/norm.rs:91-102). One warp per group: lanes sum strided chunks in
// f64, then a fixed shuffle tree (deterministic).
__global__ void __launch_bounds__(1024) gn_finalize_kernel(const double* __restrict__ part, int64_t chunks,
                                                           int64_t hw, int c, int groups, float eps,
                                                           const float* __restrict__ gamma,
                                                           const float* __restrict__ beta,
                                                           const float* __restrict__ add, float* __restrict__ scale,
                                                           float* __restrict__ shift) {
    extern __shared__ double gstat[];  // [groups][2] = mean, rstd
    const int64_t b = blockIdx.x;
    const int cg = c / groups;
    const double count = (double)hw * (double)cg;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int g = warp; g < groups; g += nwarps) {
        double sum = 0.0, sumsq = 0.0;
        for (int64_t ch = lane; ch < chunks; ch += 32) {
            const double* src = part + ((b * chunks + ch) * groups + g) * 2;
            sum += src[0];
            sumsq += src[1];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            sumsq += __shfl_xor_sync(0xffffffffu, sumsq, o);
        }
        if (lane == 0) {
            const double mean = sum / count;
            const double var = fmax(sumsq / count - mean * mean, 0.0);
            gstat[2 * g] = mean;
            gstat[2 * g + 1] = 1.0 / sqrt(var + (double)eps);
        }
    }
    __syncthreads();
    for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
        const int g = ch / cg;
        const double mean = gstat[2 * g], rstd = gstat[2 * g + 1];
        const double sc = rstd * (double)gamma[ch];
        const double pre = add ? (double)add[b * c + ch] : 0.0;
        scale[b * c + ch] = (float)sc;
        shift[b * c + ch] = (float)((double)beta[ch] + (pre - mean) * sc);
    }
}

// Epilogue statistics → GroupNorm partials. Chunk k of item b (pixels 256k … 256k + 255) is the
// two 128-row M tiles 2·(b·chunks + k) and the next of the producing conv, whose eight per-warp sum
// rows [2][c] lie next to each other. One CTA per chunk: per channel the eight f32 sums in a fixed
// order (coalesced across threads), then each group's channels folded in f64
// (src/engine/norm.rs:78-80), as gn_partials_kernel does.
__global__ void __launch_bounds__(256) gn_fold_tiles_kernel(const float* __restrict__ tp, int c, int groups,
                                                             double* __restrict__ part) {
    extern __shared__ float chunk_sums[];  // [2][c]
    const int64_t gc = blockIdx.x;
    const float* base = tp + gc * 16 * (int64_t)c;
    for (int ch = threadIdx.x; ch < c; ch += blockDim.x) {
        float sum = 0.0f, sq = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            sum += __ldg(base + (int64_t)k * 2 * c + ch);
            sq += __ldg(base + (int64_t)k * 2 * c + c + ch);
        }
        chunk_sums[ch] = sum;
        chunk_sums[c + ch] = sq;
    }
    __syncthreads();
    const int cg = c / groups;
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
        double ss = 0.0, qq = 0.0;
        for (int ch = g * cg; ch < (g + 1) * cg; ++ch) {
            ss += (double)chunk_sums[ch];
            qq += (double)chunk_sums[c + ch];
        }
        part[(gc * groups + g) * 2] = ss;
        part[(gc * groups + g) * 2 + 1] = qq;
    }
}

// grid.y = item; each thread keeps one channel vector's scale/shift in registers.
template <int V, bool SILU, bool RES>
__global__ void __launch_bounds__(256) gn_apply_kernel(const float* __restrict__ x, int64_t hw, int c,
                                                       const float* __restrict__ scale,
                                                       const float* __restrict__ shift,
                                                       const float* __restrict__ residual, float* __restrict__ out) {
    const int cv = c / V;
    const int64_t item = blockIdx.y;
    ChanStationary m;
    if (!m.init(cv)) return;
    for (int j = m.j; j < cv; j += blockDim.x) {
        float a[V], b[V];
#pragma unroll
        for (int k = 0; k < V; ++k) {
            a[k] = __ldg(scale + item * c + j * V + k);
            b[k] = __ldg(shift + item * c + j * V + k);
        }
        const int64_t base = item * hw * c + (int64_t)j * V;
#pragma unroll 4
        for (int64_t p = m.p0; p < hw; p += m.step) {
            const int64_t i = base + p * c;
            if constexpr (V == 4) {
                const float4 v = ldg_stream(reinterpret_cast<const float4*>(x + i));
                float4 y = make_float4(fmaf(v.x, a[0], b[0]), fmaf(v.y, a[1], b[1]), fmaf(v.z, a[2], b[2]),
                                       fmaf(v.w, a[3], b[3]));
                if (SILU) {
                    y.x = dev_silu(y.x);
                    y.y = dev_silu(y.y);
                    y.z = dev_silu(y.z);
                    y.w = dev_silu(y.w);
                }
                if (RES) {
                    const float4 r = ldg_stream(reinterpret_cast<const float4*>(residual + i));
                    y.x += r.x;
                    y.y += r.y;
                    y.z += r.z;
                    y.w += r.w;
                }
                stg_stream(reinterpret_cast<float4*>(out + i), y);
            } else {
                float y = fmaf(x[i], a[0], b[0]);
                if (SILU) y = dev_silu(y);
                if (RES) y += residual[i];
                out[i] = y;
            }
        }
        if (cv <= (int)blockDim.x) break;
    }
}

// LayerNorm, one warp per token, NV float4 per lane held in registers.
template <int NV>
__global__ void ln_warp_kernel(const float* __restrict__ x, int64_t tokens, int c, const float* __restrict__ gamma,
                               const float* __restrict__ beta, float eps, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int cv = c / 4;
    for (int64_t tok = warp; tok < tokens; tok += nwarps) {
        const float4* src = reinterpret_cast<const float4*>(x + tok * c);
        float4 v[NV];
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int j = lane + 32 * i;
            v[i] = j < cv ? ldg_stream(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum / (float)c;
        float vs = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int j = lane + 32 * i;
            if (j < cv) {
                const float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
                vs += (a * a + b * b) + (cc * cc + d * d);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
        const float rstd = 1.0f / sqrtf(vs / (float)c + eps);
        float4* dst = reinterpret_cast<float4*>(out + tok * c);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int j = lane + 32 * i;
            if (j < cv) {
                const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + j);
                const float4 bb = __ldg(reinterpret_cast<const float4*>(beta) + j);
                float4 y;
                y.x = fmaf((v[i].x - mean) * rstd, g.x, bb.x);
                y.y = fmaf((v[i].y - mean) * rstd, g.y, bb.y);
                y.z = fmaf((v[i].z - mean) * rstd, g.z, bb.z);
                y.w = fmaf((v[i].w - mean) * rstd, g.w, bb.w);
                stg_stream(dst + j, y);
            }
        }
    }
}

// Any channel count: one warp per token, three passes over the row.
__global__ void ln_generic_kernel(const float* __restrict__ x, int64_t tokens, int c, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, float eps, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t tok = warp; tok < tokens; tok += nwarps) {
        const float* s = x + tok * c;
        float sum = 0.0f;
        for (int j = lane; j < c; j += 32) sum += s[j];
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum / (float)c;
        float vs = 0.0f;
        for (int j = lane; j < c; j += 32) vs += (s[j] - mean) * (s[j] - mean);
        for (int o = 16; o > 0; o >>= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
        const float rstd = 1.0f / sqrtf(vs / (float)c + eps);
        for (int j = lane; j < c; j += 32) out[tok * c + j] = fmaf((s[j] - mean) * rstd, gamma[j], beta[j]);
    }
}

}  // namespace

int64_t gn_chunks(int64_t hw) { return (hw + kGnChunk - 1) / kGnChunk; }

void launch_gn_partials(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, int64_t groups,
                        const float* add, double* part) {
    const int64_t chunks = gn_chunks(hw);
    MBX_REQUIRE(chunks < (int64_t(1) << 31) && n < 65536, "GroupNorm tensor too large");
    const bool vec = c % 4 == 0 && aligned16(x) && (!add || aligned16(add));
    const int V = vec ? 4 : 1;
    // Channel slices of whole groups, at most 128 channels each (a multiple of V), so small maps
    // with few pixel chunks still fill the GPU. The slicing depends on c alone, so an item's
    // partial sums do not depend on the batch it is in.
    const int64_t cg = c / groups;
    int64_t gps = groups;
    for (int64_t d = groups; d >= 1; --d) {
        if (groups % d || (d * cg) % V) continue;
        gps = d;
        if (d * cg <= 128) break;
    }
    const int64_t cs = gps * cg;
    const int64_t cv = cs / V;
    const int rows = cv <= kGnThreads ? int(kGnThreads / cv) : 1;
    const size_t smem = size_t(2) * rows * cs * sizeof(float);
    dim3 grid((unsigned)chunks, (unsigned)n, (unsigned)(groups / gps));
    auto run = [&](auto kernel) {
        if (smem > 48 * 1024) ensure_smem_limit(reinterpret_cast<const void*>(kernel), (int)smem, "gn smem attribute");
        kernel<<<grid, kGnThreads, smem, ctx->stream>>>(x, hw, (int)c, (int)groups, (int)cs, add, part);
    };
    if (vec)
        add ? run(gn_partials_kernel<4, true>) : run(gn_partials_kernel<4, false>);
    else
        add ? run(gn_partials_kernel<1, true>) : run(gn_partials_kernel<1, false>);
    after_launch(ctx, "group_norm partials");
}

void launch_gn_fold_tiles(mbx_ctx* ctx, const float* tile_part, int64_t n, int64_t hw, int64_t c, int64_t groups,
                          double* part) {
    MBX_REQUIRE(hw % kGnChunk == 0, "GroupNorm fold: maps of a multiple of 256 pixels");
    const int64_t chunks = n * gn_chunks(hw);
    MBX_REQUIRE(chunks < (int64_t(1) << 31), "GroupNorm fold: too many chunks");
    const int smem = (int)(2 * c * sizeof(float));
    if (smem > 48 * 1024)
        ensure_smem_limit(reinterpret_cast<const void*>(gn_fold_tiles_kernel), smem, "gn fold smem attribute");
    const int threads = (int)std::min<int64_t>(256, (c + 31) / 32 * 32);
    gn_fold_tiles_kernel<<<(unsigned)chunks, threads, smem, ctx->stream>>>(tile_part, (int)c, (int)groups, part);
    after_launch(ctx, "group_norm fold");
}

void launch_gn_finalize(mbx_ctx* ctx, const double* part, int64_t n, int64_t hw, int64_t c, int64_t groups,
                        float eps, const float* gamma, const float* beta, const float* add, float* scale,
                        float* shift) {
    gn_finalize_kernel<<<(unsigned)n, 1024, groups * 2 * sizeof(double), ctx->stream>>>(
        part, gn_chunks(hw), hw, (int)c, (int)groups, eps, gamma, beta, add, scale, shift);
    after_launch(ctx, "group_norm finalize");
}

void launch_gn_apply(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* scale,
                     const float* shift, bool silu, const float* residual, float* out) {
    MBX_REQUIRE(n < 65536, "group_norm apply: too many items");
    const bool vec = c % 4 == 0 && aligned16(x) && aligned16(out) && aligned16(scale) && aligned16(shift) &&
                     (!residual || aligned16(residual));
    const int threads = 256;
    const int cv = (int)(vec ? c / 4 : c);
    const int rows = cv <= threads ? threads / cv : 1;
    const int64_t per_item = (hw + rows - 1) / rows;
    const int64_t want = std::max<int64_t>(1, (int64_t)ctx->sm_count * 8 / n);
    dim3 grid((unsigned)std::min<int64_t>(per_item, want), (unsigned)n);
    const int ci = (int)c;
#define MBX_GN_APPLY(VV, S, R) \
    gn_apply_kernel<VV, S, R><<<grid, threads, 0, ctx->stream>>>(x, hw, ci, scale, shift, residual, out)
    if (vec) {
        if (silu) {
            if (residual) MBX_GN_APPLY(4, true, true); else MBX_GN_APPLY(4, true, false);
        } else {
            if (residual) MBX_GN_APPLY(4, false, true); else MBX_GN_APPLY(4, false, false);
        }
    } else {
        if (silu) {
            if (residual) MBX_GN_APPLY(1, true, true); else MBX_GN_APPLY(1, true, false);
        } else {
            if (residual) MBX_GN_APPLY(1, false, true); else MBX_GN_APPLY(1, false, false);
        }
    }
#undef MBX_GN_APPLY
    after_launch(ctx, "group_norm apply");
}

void launch_layer_norm(mbx_ctx* ctx, const float* x, int64_t tokens, int64_t c, const float* gamma,
                       const float* beta, float eps, float* out) {
    const int threads = 256;
    const int grid = grid_for(ctx, tokens, threads / 32);
    const bool vec = c % 4 == 0 && aligned16(x) && aligned16(out) && aligned16(gamma) && aligned16(beta);
    const int nv = (int)((c / 4 + 31) / 32);
    if (vec && nv <= 16) {
        switch (nv) {
#define MBX_LN_CASE(NV)                                                                                  \
    case NV:                                                                                             \
        ln_warp_kernel<NV><<<grid, threads, 0, ctx->stream>>>(x, tokens, (int)c, gamma, beta, eps, out); \
        break;
            MBX_LN_CASE(1)
            MBX_LN_CASE(2)
            MBX_LN_CASE(3)
            MBX_LN_CASE(4)
            MBX_LN_CASE(5)
            MBX_LN_CASE(6)
            MBX_LN_CASE(7)
            MBX_LN_CASE(8)
            MBX_LN_CASE(9)
            MBX_LN_CASE(10)
            MBX_LN_CASE(11)
            MBX_LN_CASE(12)
            MBX_LN_CASE(13)
            MBX_LN_CASE(14)
            MBX_LN_CASE(15)
            MBX_LN_CASE(16)
#undef MBX_LN_CASE
        }
    } else {
        ln_generic_kernel<<<grid, threads, 0, ctx->stream>>>(x, tokens, (int)c, gamma, beta, eps, out);
    }
    after_launch(ctx, "layer_norm");
}

}  // namespace mbx
