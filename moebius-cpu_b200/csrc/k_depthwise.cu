// Depthwise 3×3, stride 1, zero padding 1, NHWC, bias and a fused epilogue
// (reference src/engine/depthwise.rs:31-185).
//
// Each thread owns one channel vector (4 channels, or 1 for channel counts
// that are not multiples of 4) at one x position and walks a strip of 16 or 64
// output rows in blocks of 4 (1 for GLU): each block loads its 6 (3) input rows
// at once, so many loads are in flight per thread (the left and right pixels
// are the neighbouring threads' centre pixels and the block-overlap rows were
// loaded by the previous block, so both come from L1). A CTA covers 8 channel vectors × 16 x-positions; the x-halo columns
// belong to neighbouring CTAs that run at the same time, so they come from L2,
// and DRAM traffic is about one read of the input (+3% y-halo) plus one write. Taps are accumulated bias-first in
// (ky, kx) order with fma(tap, x, acc) as in acc_block (:112-143); padding
// taps contribute nothing.
#include <algorithm>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kDwThreads = 128;
// Output rows per thread strip: 64 on large maps (y-halo re-read 2/64), 16 on the UNet's
// small ones (64² and below), where more, shorter strips keep more loads in flight.
inline int strip_rows(int64_t h) { return h >= 256 ? 64 : 16; }
constexpr int kDwQuads = 8;  // channel vectors per CTA row (16 x-positions per CTA)

template <int V>
struct Vec {
    float v[V];
};

template <int V>
__device__ __forceinline__ Vec<V> vload(const float* p) {
    Vec<V> r;
    if constexpr (V == 4) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(p));
        r.v[0] = f.x;
        r.v[1] = f.y;
        r.v[2] = f.z;
        r.v[3] = f.w;
    } else {
        r.v[0] = __ldg(p);
    }
    return r;
}

template <int V>
__device__ __forceinline__ Vec<V> vzero() {
    Vec<V> r;
#pragma unroll
    for (int k = 0; k < V; ++k) r.v[k] = 0.0f;
    return r;
}

template <int V>
__device__ __forceinline__ void vstore(float* p, const Vec<V>& a) {
    if constexpr (V == 4)
        stg_stream(reinterpret_cast<float4*>(p), make_float4(a.v[0], a.v[1], a.v[2], a.v[3]));
    else
        *p = a.v[0];
}

// Loads row `iy` at columns ix-1, ix, ix+1 for channel offset `ch` (zero when padded).
template <int V>
__device__ __forceinline__ void load_row(const float* __restrict__ xb, int h, int w, int c, int iy, int ix, int ch,
                                         Vec<V> (&row)[3]) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const int xx = ix + k - 1;
        row[k] = (iy >= 0 && iy < h && xx >= 0 && xx < w) ? vload<V>(xb + ((int64_t)iy * w + xx) * c + ch)
                                                          : vzero<V>();
    }
}

template <int V>
__device__ __forceinline__ Vec<V> taps(const Vec<V> (&win)[3][3], const Vec<V> (&wt)[9], const Vec<V>& bias,
                                       bool top, bool bottom, bool left, bool right) {
    Vec<V> acc = bias;
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
        if ((ky == 0 && !top) || (ky == 2 && !bottom)) continue;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            if ((kx == 0 && !left) || (kx == 2 && !right)) continue;
#pragma unroll
            for (int k = 0; k < V; ++k) acc.v[k] = fmaf(wt[ky * 3 + kx].v[k], win[ky][kx].v[k], acc.v[k]);
        }
    }
    return acc;
}

// grid: x = output channel-vector blocks, y = x-position blocks, z = item × strip.
// The CTA's taps and bias sit in shared memory (read with warp broadcasts).
template <int V, int EPI, int RB>
__global__ void __launch_bounds__(kDwThreads, 4) dw3x3_kernel(const float* __restrict__ x, int h, int w, int c,
                                                           const float* __restrict__ weight,
                                                           const float* __restrict__ bias, float* __restrict__ out,
                                                           int qb, int strips, int rows) {
    constexpr bool kGlu = EPI == MBX_EPILOGUE_GLU_SILU;
    constexpr int kSets = kGlu ? 2 : 1;  // value (and gate) channel sets
    __shared__ Vec<V> s_w[kSets][9][kDwQuads];
    __shared__ Vec<V> s_b[kSets][kDwQuads];
    const int c_out = kGlu ? c / 2 : c;
    const int cvo = c_out / V;
    const int xb = kDwThreads / qb;
    const int t = threadIdx.x;
    // Stage the taps of this CTA's channel vectors.
    for (int e = t; e < kSets * 10 * qb; e += kDwThreads) {
        const int set = e / (10 * qb), rem = e % (10 * qb), tap = rem / qb, qq = rem % qb;
        const int qv = blockIdx.x * qb + qq;
        if (qv < cvo) {
            const int ch = set * c_out + qv * V;
            if (tap < 9)
                s_w[set][tap][qq] = vload<V>(weight + tap * c + ch);
            else
                s_b[set][qq] = vload<V>(bias + ch);
        }
    }
    __syncthreads();
    if (t >= qb * xb) return;
    const int qq = t % qb;
    const int qv = blockIdx.x * qb + qq;
    const int ox = blockIdx.y * xb + t / qb;
    if (qv >= cvo || ox >= w) return;
    const int b = blockIdx.z / strips;
    const int y0 = (blockIdx.z % strips) * rows;
    const int y1 = min(y0 + rows, h);
    const int ch = qv * V;
    const float* xb_ = x + (int64_t)b * h * w * c;

    // Blocks of RB output rows: their RB + 2 input rows are loaded together (all loads in
    // flight at once, no register rotation), then the RB rows are computed; the two rows
    // shared with the next block come from L1.
    const bool left = ox > 0, right = ox + 1 < w;
    for (int y = y0; y < y1; y += RB) {
        Vec<V> in[kSets][RB + 2][3];
#pragma unroll
        for (int set = 0; set < kSets; ++set)
#pragma unroll
            for (int rr = 0; rr < RB + 2; ++rr) load_row<V>(xb_, h, w, c, y - 1 + rr, ox, set * c_out + ch, in[set][rr]);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            if (y + r >= y1) break;
            const bool top = y + r > 0, bottom = y + r + 1 < h;
            Vec<V> acc[kSets];
#pragma unroll
            for (int set = 0; set < kSets; ++set) {
                const Vec<V>(&win)[3][3] = *reinterpret_cast<const Vec<V>(*)[3][3]>(&in[set][r]);
                Vec<V> wt[9];
#pragma unroll
                for (int k = 0; k < 9; ++k) wt[k] = s_w[set][k][qq];
                acc[set] = taps<V>(win, wt, s_b[set][qq], top, bottom, left, right);
            }
            Vec<V> res = acc[0];
            if constexpr (EPI == MBX_EPILOGUE_RELU) {
#pragma unroll
                for (int k = 0; k < V; ++k) res.v[k] = fmaxf(res.v[k], 0.0f);
            } else if constexpr (kGlu) {
#pragma unroll
                for (int k = 0; k < V; ++k) res.v[k] = acc[0].v[k] * dev_silu(acc[kSets - 1].v[k]);
            }
            vstore<V>(out + (((int64_t)b * h + y + r) * w + ox) * c_out + ch, res);
        }
    }
}


// ---------------------------------------------------------------- TMA-tiled variant
// A tile is 16 × 16 output pixels of 32 channels (both channel sets for GLU): one TMA box
// {32, 18, 18, 1} per set brings it with its halo, read once from global memory (the box's zero
// fill past the map is never used: padding taps are skipped as above). Persistent CTAs walk tiles
// tt = blockIdx.x, blockIdx.x + gridDim.x, ... (channel block fastest, then tile, then item)
// through a two-stage ring: tile i + 1's boxes land while tile i is computed, so the memory pipe
// stays busy (one CTA per SM with the GLU's two sets, two otherwise). Each thread walks 8 output
// rows of one 4-channel vector at one x, sliding a 3-row window through shared memory; its taps
// and bias sit in registers, reloaded when the tile's channel block changes.
constexpr int kTT = 16;                                           // tile side (output pixels)
constexpr int kTC = 32;                                           // channels per tile
constexpr int kTH = kTT + 2;                                      // halo tile side
constexpr int kTileThreads = 256;                                 // 8 vectors × 16 columns × 2 row groups
constexpr uint32_t kSetBytes = (uint32_t)kTH * kTH * kTC * 4;    // 41472
constexpr int kStages = 2;
constexpr long long kDwWaitLimit = 4ll << 30;                     // clock cycles (about 2 s)

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool dw_landed(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

struct DwTiles {
    int cblocks, tiles_x, tiles_xy;
    int64_t total;
    __device__ __forceinline__ void at(int64_t tt, int& cb, int& y0, int& x0, int& item) const {
        cb = (int)(tt % cblocks);
        const int64_t rest = tt / cblocks;
        const int tile = (int)(rest % tiles_xy);
        item = (int)(rest / tiles_xy);
        const int ty = tile / tiles_x;
        y0 = ty * kTT;
        x0 = (tile - ty * tiles_x) * kTT;
    }
};

// PRO: GroupNorm prologue, the input read as [SiLU](x*pro_scale[item,c] + pro_shift[item,c]).
template <int EPI, bool PRO>
__global__ void __launch_bounds__(kTileThreads) dw3x3_tma_kernel(const __grid_constant__ CUtensorMap map, int h,
                                                                 int w, int c, const float* __restrict__ weight,
                                                                 const float* __restrict__ bias,
                                                                 const float* __restrict__ pro_scale,
                                                                 const float* __restrict__ pro_shift, int pro_silu,
                                                                 float* __restrict__ out, DwTiles tiles, int* err) {
    constexpr bool kGlu = EPI == MBX_EPILOGUE_GLU_SILU;
    constexpr int kSets = kGlu ? 2 : 1;
    constexpr uint32_t kStageBytes = (uint32_t)kSets * kSetBytes;
    extern __shared__ __align__(1024) float ring[];  // [stage][set][kTH][kTH][kTC]
    __shared__ __align__(8) uint64_t bars[kStages];
    const int c_out = kGlu ? c / 2 : c;
    const uint32_t bar0 = smem_addr(&bars[0]);
    auto bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto stage_ptr = [&](int s) { return ring + (size_t)s * (kStageBytes / 4); };
    // Thread 0: arms stage s for tile tt and issues its boxes.
    auto issue = [&](int s, int64_t tt) {
        int cb, y0, x0, item;
        tiles.at(tt, cb, y0, x0, item);
        asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar(s)),
                     "r"(kStageBytes)
                     : "memory");
#pragma unroll
        for (int set = 0; set < kSets; ++set)
            asm volatile(
                "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
                "%3, %4, %5}], [%6];" ::"r"(smem_addr(stage_ptr(s) + set * kTH * kTH * kTC)),
                "l"(reinterpret_cast<uint64_t>(&map)), "r"(cb * kTC + set * c_out), "r"(x0 - 1), "r"(y0 - 1),
                "r"(item), "r"(bar(s))
                : "memory");
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(s)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int s = 0; s < kStages; ++s) {
            const int64_t tt = blockIdx.x + (int64_t)s * gridDim.x;
            if (tt < tiles.total) issue(s, tt);
        }
    }
    __syncthreads();
    // Thread mapping: channel quad j, column xl, row group rg (8 rows each); a thread holds both
    // GLU sets (splitting them over a lane pair, to halve the registers and double the warps, was
    // slower: the gate shuffles and the doubled SiLU work cost more than the extra warps gained).
    const int j = threadIdx.x & 7, xl = (threadIdx.x >> 3) & 15, rg = threadIdx.x >> 7;
    Vec<4> wt[kSets][9], bs[kSets];
    int cb_loaded = -1;
    int it = 0;
    for (int64_t tt = blockIdx.x; tt < tiles.total; tt += gridDim.x, ++it) {
        const int s = it & 1;
        const uint32_t parity = (uint32_t)((it >> 1) & 1);
        // Bounded wait for the boxes; on timeout (any thread's) the error is recorded and the CTA
        // writes nothing more. Thread 0 then keeps waiting, bounded again, for the boxes it issued
        // (this tile's and the next one's), so the CTA does not retire under a pending copy.
        {
            const long long t0 = clock64();
            int timed_out = 0;
            while (!dw_landed(bar(s), parity)) {
                if (clock64() - t0 > kDwWaitLimit) {
                    timed_out = 1;
                    break;
                }
            }
            if (__syncthreads_or(timed_out)) {
                if (threadIdx.x == 0) {
                    if (atomicCAS(err, 0, kErrWaitTimeout) == 0) err[1] = kKDepthwise;
                    const long long t1 = clock64();
                    while (!dw_landed(bar(s), parity) && clock64() - t1 <= kDwWaitLimit) {
                    }
                    if (tt + gridDim.x < tiles.total) {
                        const uint32_t p1 = (uint32_t)(((it + 1) >> 1) & 1);
                        while (!dw_landed(bar(s ^ 1), p1) && clock64() - t1 <= 2 * kDwWaitLimit) {
                        }
                    }
                }
                return;
            }
        }
        int cb, y0, x0, item;
        tiles.at(tt, cb, y0, x0, item);
        const int c0 = cb * kTC;
        float* tile = stage_ptr(s);
        if constexpr (PRO) {
            // GroupNorm prologue on the landed window, in place, at in-image pixels of real channels
            // (the padding taps are skipped below and channels past c are never stored, so their
            // zero fill stays). Same arithmetic as the GroupNorm apply kernel: fmaf(x, scale, shift),
            // then SiLU.
            const int q4 = threadIdx.x & 7;
#pragma unroll
            for (int set = 0; set < kSets; ++set) {
                const int cc = c0 + set * c_out + 4 * q4;
                if (cc >= c) continue;
                const float4 sc = __ldg(reinterpret_cast<const float4*>(pro_scale + (int64_t)item * c + cc));
                const float4 sh = __ldg(reinterpret_cast<const float4*>(pro_shift + (int64_t)item * c + cc));
                float* base = tile + set * kTH * kTH * kTC + 4 * q4;
                for (int px = threadIdx.x >> 3; px < kTH * kTH; px += kTileThreads / 8) {
                    const int row = px / kTH, col = px - row * kTH;
                    const int gy = y0 - 1 + row, gx = x0 - 1 + col;
                    if (gy < 0 || gy >= h || gx < 0 || gx >= w) continue;
                    float4* e = reinterpret_cast<float4*>(base + px * kTC);
                    float4 t = *e;
                    t = make_float4(fmaf(t.x, sc.x, sh.x), fmaf(t.y, sc.y, sh.y), fmaf(t.z, sc.z, sh.z),
                                    fmaf(t.w, sc.w, sh.w));
                    if (pro_silu) t = make_float4(dev_silu(t.x), dev_silu(t.y), dev_silu(t.z), dev_silu(t.w));
                    *e = t;
                }
            }
            __syncthreads();
        }
        const int ch = c0 + 4 * j, ox = x0 + xl;
        if (ch < c_out && ox < w) {
            // All taps of this thread's channel quad (both GLU sets) stay in registers while the
            // channel block stays the same.
            if (cb != cb_loaded) {
#pragma unroll
                for (int set = 0; set < kSets; ++set) {
#pragma unroll
                    for (int k = 0; k < 9; ++k) wt[set][k] = vload<4>(weight + k * c + set * c_out + ch);
                    bs[set] = vload<4>(bias + set * c_out + ch);
                }
                cb_loaded = cb;
            }
            const bool left = ox > 0, right = ox + 1 < w;
            auto at = [&](int set, int row, int col) -> Vec<4> {
                const float4 f =
                    *reinterpret_cast<const float4*>(tile + (((set * kTH + row) * kTH + col) * kTC + 4 * j));
                Vec<4> r;
                r.v[0] = f.x;
                r.v[1] = f.y;
                r.v[2] = f.z;
                r.v[3] = f.w;
                return r;
            };
            const int r_begin = rg * (kTT / 2), r_end = min(r_begin + kTT / 2, h - y0);
            Vec<4> win[kSets][3][3];
#pragma unroll
            for (int set = 0; set < kSets; ++set)
#pragma unroll
                for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                    for (int k = 0; k < 3; ++k) win[set][rr][k] = at(set, r_begin + rr, xl + k);
            // Fully unrolled, so the window's rotation below is register renaming, not moves.
#pragma unroll
            for (int rr = 0; rr < kTT / 2; ++rr) {
                const int r = r_begin + rr;
                if (r >= r_end) break;
                const int oy = y0 + r;
#pragma unroll
                for (int set = 0; set < kSets; ++set)
#pragma unroll
                    for (int k = 0; k < 3; ++k) win[set][2][k] = at(set, r + 2, xl + k);
                const bool top = oy > 0, bottom = oy + 1 < h;
                Vec<4> acc[kSets];
#pragma unroll
                for (int set = 0; set < kSets; ++set)
                    acc[set] = taps<4>(win[set], wt[set], bs[set], top, bottom, left, right);
                Vec<4> res = acc[0];
                if constexpr (EPI == MBX_EPILOGUE_RELU) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) res.v[k] = fmaxf(res.v[k], 0.0f);
                } else if constexpr (kGlu) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) res.v[k] = acc[0].v[k] * dev_silu(acc[kSets - 1].v[k]);
                }
                vstore<4>(out + (((int64_t)item * h + oy) * w + ox) * c_out + ch, res);
#pragma unroll
                for (int set = 0; set < kSets; ++set)
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        win[set][0][k] = win[set][1][k];
                        win[set][1][k] = win[set][2][k];
                    }
            }
        }
        // Every thread's reads (and the prologue's writes) of this stage are ordered before the
        // next boxes land in it (an async-proxy write), then thread 0 re-arms the stage.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (threadIdx.x == 0 && tt + (int64_t)kStages * gridDim.x < tiles.total)
            issue(s, tt + (int64_t)kStages * gridDim.x);
    }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

void launch_depthwise3x3(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                         const float* weight, const float* bias, int epilogue, float* out, const float* pro_scale,
                         const float* pro_shift, bool pro_silu) {
    MBX_REQUIRE(h < (1 << 20) && w < (1 << 20) && c < (1 << 20), "depthwise: dimension too large");
    MBX_REQUIRE((pro_scale == nullptr) == (pro_shift == nullptr), "depthwise: prologue needs scale and shift");
    const bool pro = pro_scale != nullptr;
    const int64_t c_out = epilogue == MBX_EPILOGUE_GLU_SILU ? c / 2 : c;
    const bool vec = c % 4 == 0 && c_out % 4 == 0 && aligned16(x) && aligned16(out) && aligned16(weight) &&
                     aligned16(bias);
    // TMA-tiled kernel where the halo box fits inside the map and one channel box inside c.
    if (vec && c >= kTC && h >= kTH && w >= kTH && n < 65536 && h < (1 << 20) && w < (1 << 20) &&
        (!pro || (aligned16(pro_scale) && aligned16(pro_shift)))) {
        const int64_t tiles_x = (w + kTT - 1) / kTT, tiles_y = (h + kTT - 1) / kTT;
        const int64_t cblocks = (c_out + kTC - 1) / kTC;
        if (tiles_x * tiles_y < 65536 && cblocks < 65536) {
            CUtensorMap map;
            const uint64_t dims[4] = {(uint64_t)c, (uint64_t)w, (uint64_t)h, (uint64_t)n};
            const uint64_t strides[3] = {(uint64_t)c * 4, (uint64_t)(w * c) * 4, (uint64_t)(h * w * c) * 4};
            const uint32_t box[4] = {(uint32_t)kTC, (uint32_t)kTH, (uint32_t)kTH, 1};
            encode_tensor_map_f32(&map, x, 4, dims, strides, box, false);
            DwTiles tiles{(int)cblocks, (int)tiles_x, (int)(tiles_x * tiles_y), cblocks * tiles_x * tiles_y * n};
            auto launch = [&](auto kern, int sets) {
                const int smem = kStages * sets * (int)kSetBytes;
                ensure_smem_limit(reinterpret_cast<const void*>(kern), smem, "depthwise smem attribute");
                int per_sm = 0;
                check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTileThreads, smem),
                           "depthwise occupancy");
                const int64_t grid = std::min<int64_t>(tiles.total, (int64_t)ctx->sm_count * std::max(per_sm, 1));
                kern<<<(unsigned)grid, kTileThreads, smem, ctx->stream>>>(map, (int)h, (int)w, (int)c, weight, bias,
                                                                          pro_scale, pro_shift, pro_silu ? 1 : 0, out,
                                                                          tiles, ctx->dev_err);
            };
            if (pro) {
                if (epilogue == MBX_EPILOGUE_NONE) launch(dw3x3_tma_kernel<MBX_EPILOGUE_NONE, true>, 1);
                else if (epilogue == MBX_EPILOGUE_RELU) launch(dw3x3_tma_kernel<MBX_EPILOGUE_RELU, true>, 1);
                else launch(dw3x3_tma_kernel<MBX_EPILOGUE_GLU_SILU, true>, 2);
            } else {
                if (epilogue == MBX_EPILOGUE_NONE) launch(dw3x3_tma_kernel<MBX_EPILOGUE_NONE, false>, 1);
                else if (epilogue == MBX_EPILOGUE_RELU) launch(dw3x3_tma_kernel<MBX_EPILOGUE_RELU, false>, 1);
                else launch(dw3x3_tma_kernel<MBX_EPILOGUE_GLU_SILU, false>, 2);
            }
            after_launch(ctx, "depthwise3x3");
            return;
        }
    }
    if (pro) {
        // Shapes the tiled kernel does not take: the GroupNorm goes to scratch first.
        PoolBuf normed(ctx, size_t(n * h * w * c) * sizeof(float));
        launch_gn_apply(ctx, x, n, h * w, c, pro_scale, pro_shift, pro_silu, nullptr, normed.as<float>());
        launch_depthwise3x3(ctx, normed.as<float>(), n, h, w, c, weight, bias, epilogue, out);
        return;
    }
    const int V = vec ? 4 : 1;
    const int64_t cvo = c_out / V;
    const int qb = (int)std::min<int64_t>(cvo, kDwQuads);
    const int xb = kDwThreads / qb;
    const int rows = strip_rows(h);
    const int64_t strips = (h + rows - 1) / rows;
    MBX_REQUIRE(n * strips < (int64_t(1) << 31) && (cvo + qb - 1) / qb < (int64_t(1) << 31),
                "depthwise: grid too large");
    MBX_REQUIRE((w + xb - 1) / xb < 65536 && n * strips < 65536 * 32768LL, "depthwise: grid too large");
    dim3 grid((unsigned)((cvo + qb - 1) / qb), (unsigned)((w + xb - 1) / xb), (unsigned)(n * strips));
    MBX_REQUIRE(grid.z <= 65535, "depthwise: too many row strips (n * ceil(h / strip rows) must be <= 65535)");
    const int hh = (int)h, ww = (int)w, cc = (int)c, st = (int)strips;
#define MBX_DW(VV, EE)                                                                                      \
    dw3x3_kernel<VV, EE, EE == MBX_EPILOGUE_GLU_SILU ? 1 : 4><<<grid, kDwThreads, 0, ctx->stream>>>( \
        x, hh, ww, cc, weight, bias, out, qb, st, rows)
    if (V == 4) {
        if (epilogue == MBX_EPILOGUE_NONE) MBX_DW(4, MBX_EPILOGUE_NONE);
        else if (epilogue == MBX_EPILOGUE_RELU) MBX_DW(4, MBX_EPILOGUE_RELU);
        else MBX_DW(4, MBX_EPILOGUE_GLU_SILU);
    } else {
        if (epilogue == MBX_EPILOGUE_NONE) MBX_DW(1, MBX_EPILOGUE_NONE);
        else if (epilogue == MBX_EPILOGUE_RELU) MBX_DW(1, MBX_EPILOGUE_RELU);
        else MBX_DW(1, MBX_EPILOGUE_GLU_SILU);
    }
#undef MBX_DW
    after_launch(ctx, "depthwise3x3");
}

}  // namespace mbx
