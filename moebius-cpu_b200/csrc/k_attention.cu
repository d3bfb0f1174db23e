// Pieces of the VAE mid-block attention and of the decoder's latent/image
// scaling (reference src/vae/mod.rs:240-293, src/vae/decoder.rs:81,97):
//
//  * softmax_rows: in-place softmax(scale·row) per row with probabilities
//    below e^flush set to zero (the reference flushes below e^-40, :273-293).
//  * split_to_param: an activation matrix B used as the tensor-core GEMM's
//    second operand (q·kᵀ, p·v) is rounded into TF32 high/low parts in the
//    K-major, zero-padded layout of a conv weight (either from B stored
//    [n × k] row-major, or transposed from [k × n]).
//  * scale_add: out = x·mul + add.
#include <cfloat>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int kSoftmaxThreads = 512;

__device__ __forceinline__ float block_reduce(float v, float* sh, bool is_max) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, u) : v + u;
    }
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float r = is_max ? -FLT_MAX : 0.0f;
    for (int i = 0; i < nw; ++i) r = is_max ? fmaxf(r, sh[i]) : r + sh[i];
    return r;
}

// One CTA per row; the row (≤ 16 K floats here) streams through registers twice.
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_rows_kernel(float* __restrict__ x, int64_t n, float scale,
                                                                       float flush) {
    __shared__ float sh[kSoftmaxThreads / 32];
    float* row = x + (int64_t)blockIdx.x * n;
    float m = -FLT_MAX;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, row[i]);
    m = block_reduce(m, sh, true);
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float a = (row[i] - m) * scale;
        const float e = a < flush ? 0.0f : expf(a);
        row[i] = e;
        s += e;
    }
    s = block_reduce(s, sh, false);
    const float inv = 1.0f / s;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) row[i] *= inv;
}

__device__ __forceinline__ float tf32_rn(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// hi/lo [rows_pad × k_pad]: row o, column i = B(o, i) (0 in the padding).
__global__ void split_to_param_kernel(const float* __restrict__ b, int64_t n, int64_t k, int b_is_kn, int64_t rows_pad,
                                      int64_t k_pad, float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t total = rows_pad * k_pad;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e / k_pad, i = e % k_pad;
        float v = 0.0f;
        if (o < n && i < k) v = b_is_kn ? b[i * n + o] : b[o * k + i];
        const float h = tf32_rn(v);
        hi[e] = h;
        lo[e] = tf32_rn(v - h);
    }
}

__global__ void scale_add_kernel(const float* __restrict__ x, int64_t len, float mul, float add,
                                 float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < len; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = fmaf(x[i], mul, add);
}

}  // namespace

void launch_softmax_rows(mbx_ctx* ctx, float* x, int64_t rows, int64_t n, float scale, float flush) {
    MBX_REQUIRE(rows < (int64_t(1) << 31), "softmax: too many rows");
    softmax_rows_kernel<<<(unsigned)rows, kSoftmaxThreads, 0, ctx->stream>>>(x, n, scale, flush);
    after_launch(ctx, "softmax_rows");
}

void launch_split_to_param(mbx_ctx* ctx, const float* b, int64_t n, int64_t k, bool b_is_kn, mbx_param* p) {
    split_to_param_kernel<<<grid_for(ctx, int64_t(p->cout_pad) * p->cin_pad, 256), 256, 0, ctx->stream>>>(
        b, n, k, b_is_kn ? 1 : 0, p->cout_pad, p->cin_pad, p->hi, p->lo);
    after_launch(ctx, "split_to_param");
}

void launch_scale_add(mbx_ctx* ctx, const float* x, int64_t len, float mul, float add, float* out) {
    scale_add_kernel<<<grid_for(ctx, len, 256), 256, 0, ctx->stream>>>(x, len, mul, add, out);
    after_launch(ctx, "scale_add");
}

}  // namespace mbx
