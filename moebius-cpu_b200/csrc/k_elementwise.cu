// Streaming elementwise kernels: SiLU, residual add, bias + timestep
// broadcast add, channel concat. HBM-bound; 128-bit loads/stores whenever the
// pointers are 16-byte aligned and the channel counts are multiples of 4,
// grid-stride loops sized to a few waves of the 148 SMs.
#include <algorithm>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kThreads = 256;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__global__ void silu_vec4(float4* x, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 v = x[i];
        v.x = dev_silu(v.x);
        v.y = dev_silu(v.y);
        v.z = dev_silu(v.z);
        v.w = dev_silu(v.w);
        x[i] = v;
    }
}

__global__ void silu_scalar(float* x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = dev_silu(x[i]);
}

__global__ void add_vec4(const float4* a, const float4* b, float4* out, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 u = ldg_stream(a + i), v = ldg_stream(b + i);
        u.x += v.x;
        u.y += v.y;
        u.z += v.z;
        u.w += v.w;
        stg_stream(out + i, u);
    }
}

__global__ void add_scalar(const float* a, const float* b, float* out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

// out = (x + bias[c]) + temb[item, c]; V = 4 (float4 over channels) or 1.
// grid.y = item; each thread keeps one channel vector and walks pixels.
template <int V>
__global__ void __launch_bounds__(256) bias_temb_kernel(const float* __restrict__ x, int64_t hw, int c,
                                                        const float* __restrict__ bias,
                                                        const float* __restrict__ temb, float* out) {
    const int cv = c / V;
    const int64_t item = blockIdx.y;
    ChanStationary m;
    if (!m.init(cv)) return;
    for (int j = m.j; j < cv; j += blockDim.x) {
        // (x + bias) + temb, in that order: keep both addends separate.
        float bv[V], tv[V];
#pragma unroll
        for (int k = 0; k < V; ++k) {
            bv[k] = bias ? __ldg(bias + j * V + k) : 0.0f;
            tv[k] = temb ? __ldg(temb + item * c + j * V + k) : 0.0f;
        }
        const float* xi = x + item * hw * c + (int64_t)j * V;
        float* oi = out + item * hw * c + (int64_t)j * V;
#pragma unroll 4
        for (int64_t p = m.p0; p < hw; p += m.step) {
            if constexpr (V == 4) {
                float4 v = ldg_stream(reinterpret_cast<const float4*>(xi + p * c));
                if (bias) {
                    v.x = v.x + bv[0];
                    v.y = v.y + bv[1];
                    v.z = v.z + bv[2];
                    v.w = v.w + bv[3];
                }
                if (temb) {
                    v.x = v.x + tv[0];
                    v.y = v.y + tv[1];
                    v.z = v.z + tv[2];
                    v.w = v.w + tv[3];
                }
                stg_stream(reinterpret_cast<float4*>(oi + p * c), v);
            } else {
                float v = xi[p * c];
                if (bias) v = v + bv[0];
                if (temb) v = v + tv[0];
                oi[p * c] = v;
            }
        }
        if (cv <= (int)blockDim.x) break;
    }
}

template <int V>
__global__ void concat_kernel(const float* __restrict__ a, int64_t ca, const float* __restrict__ b, int64_t cb,
                              float* __restrict__ out, int64_t total_v) {
    const int64_t cav = ca / V, cbv = cb / V, cov = cav + cbv;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total_v;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = i / cov, j = i % cov;
        if constexpr (V == 4) {
            const float4 v = j < cav ? ldg_stream(reinterpret_cast<const float4*>(a) + p * cav + j)
                                     : ldg_stream(reinterpret_cast<const float4*>(b) + p * cbv + (j - cav));
            stg_stream(reinterpret_cast<float4*>(out) + i, v);
        } else {
            out[i] = j < cav ? a[p * cav + j] : b[p * cbv + (j - cav)];
        }
    }
}

}  // namespace

void launch_silu_inplace(mbx_ctx* ctx, float* x, int64_t len) {
    if (aligned16(x) && len % 4 == 0) {
        silu_vec4<<<grid_for(ctx, len / 4, kThreads), kThreads, 0, ctx->stream>>>(reinterpret_cast<float4*>(x),
                                                                                   len / 4);
    } else {
        silu_scalar<<<grid_for(ctx, len, kThreads), kThreads, 0, ctx->stream>>>(x, len);
    }
    after_launch(ctx, "silu");
}

void launch_add(mbx_ctx* ctx, const float* a, const float* b, float* out, int64_t len) {
    if (aligned16(a) && aligned16(b) && aligned16(out) && len % 4 == 0) {
        add_vec4<<<grid_for(ctx, len / 4, kThreads), kThreads, 0, ctx->stream>>>(
            reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(out),
            len / 4);
    } else {
        add_scalar<<<grid_for(ctx, len, kThreads), kThreads, 0, ctx->stream>>>(a, b, out, len);
    }
    after_launch(ctx, "add");
}

void launch_bias_temb_add(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* bias,
                          const float* temb, float* out) {
    MBX_REQUIRE(n < 65536 && c < (1 << 24), "bias_temb_add: too many items or channels");
    const bool vec = c % 4 == 0 && aligned16(x) && aligned16(out) && (!bias || aligned16(bias)) &&
                     (!temb || aligned16(temb));
    const int cv = (int)(vec ? c / 4 : c);
    const int rows = cv <= kThreads ? kThreads / cv : 1;
    const int64_t per_item = (hw + rows - 1) / rows;
    const int64_t want = std::max<int64_t>(1, (int64_t)ctx->sm_count * 8 / n);
    dim3 grid((unsigned)std::min<int64_t>(per_item, want), (unsigned)n);
    if (vec)
        bias_temb_kernel<4><<<grid, kThreads, 0, ctx->stream>>>(x, hw, (int)c, bias, temb, out);
    else
        bias_temb_kernel<1><<<grid, kThreads, 0, ctx->stream>>>(x, hw, (int)c, bias, temb, out);
    after_launch(ctx, "bias_temb_add");
}

void launch_concat(mbx_ctx* ctx, const float* a, int64_t ca, const float* b, int64_t cb, int64_t pixels,
                   float* out) {
    const int64_t total = pixels * (ca + cb);
    const bool vec = ca % 4 == 0 && cb % 4 == 0 && (ca == 0 || aligned16(a)) && (cb == 0 || aligned16(b)) &&
                     aligned16(out);
    if (vec) {
        concat_kernel<4><<<grid_for(ctx, total / 4, kThreads), kThreads, 0, ctx->stream>>>(a, ca, b, cb, out,
                                                                                           total / 4);
    } else {
        concat_kernel<1><<<grid_for(ctx, total, kThreads), kThreads, 0, ctx->stream>>>(a, ca, b, cb, out, total);
    }
    after_launch(ctx, "concat_channels");
}

}  // namespace mbx
