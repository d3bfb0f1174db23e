// General strided f32 matmul c (+)= A·B (reference gemm::matmul with MatRef
// views, src/engine/gemm.rs:25-132). Serves the small strided contractions of
// the engine's callers (λ layers, attention score bands) whose operands are
// views with arbitrary element strides; the dense convolutions use the
// tensor-core path in k_conv_tc.cu. 64×64 output tiles, 16-deep K slabs
// staged in shared memory, 4×4 outputs per thread, f32 FMA.
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) matmul_simt_kernel(float* __restrict__ c, const float* __restrict__ a,
                                                          int64_t m, int64_t k, int64_t a_rs, int64_t a_cs,
                                                          const float* __restrict__ b, int64_t n, int64_t b_rs,
                                                          int64_t b_cs, bool accumulate) {
    __shared__ float as[TK][TM + 4];
    __shared__ float bs[TK][TN + 4];
    const int t = threadIdx.x;
    const int tr = t / 16, tc = t % 16;  // 16×16 threads, 4×4 outputs each
    const int64_t i0 = (int64_t)blockIdx.y * TM, j0 = (int64_t)blockIdx.x * TN;
    float acc[4][4] = {};
    for (int64_t p0 = 0; p0 < k; p0 += TK) {
        for (int e = t; e < TM * TK; e += 256) {
            const int ii = e / TK, pp = e % TK;
            const int64_t i = i0 + ii, p = p0 + pp;
            as[pp][ii] = (i < m && p < k) ? a[i * a_rs + p * a_cs] : 0.0f;
        }
        for (int e = t; e < TN * TK; e += 256) {
            const int jj = e % TN, pp = e / TN;
            const int64_t j = j0 + jj, p = p0 + pp;
            bs[pp][jj] = (j < n && p < k) ? b[p * b_rs + j * b_cs] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int pp = 0; pp < TK; ++pp) {
            float av[4], bv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) av[r] = as[pp][tr * 4 + r];
#pragma unroll
            for (int q = 0; q < 4; ++q) bv[q] = bs[pp][tc * 4 + q];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[r][q] = fmaf(av[r], bv[q], acc[r][q]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t i = i0 + tr * 4 + r, j = j0 + tc * 4 + q;
            if (i < m && j < n) {
                float* dst = c + i * n + j;
                *dst = accumulate ? *dst + acc[r][q] : acc[r][q];
            }
        }
}

}  // namespace

void launch_matmul_simt(mbx_ctx* ctx, float* c, const float* a, int64_t m, int64_t k, int64_t a_rs, int64_t a_cs,
                        const float* b, int64_t n, int64_t b_rs, int64_t b_cs, bool accumulate) {
    MBX_REQUIRE((m + TM - 1) / TM < 65536, "matmul: too many rows");
    dim3 grid((unsigned)((n + TN - 1) / TN), (unsigned)((m + TM - 1) / TM));
    matmul_simt_kernel<<<grid, 256, 0, ctx->stream>>>(c, a, m, k, a_rs, a_cs, b, n, b_rs, b_cs, accumulate);
    after_launch(ctx, "matmul");
}

}  // namespace mbx
