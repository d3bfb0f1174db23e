// Device-side helpers shared by the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mbx {

// x·σ(x) = x / (1 + e^−x), the reference's SiLU (src/engine/math.rs:34-36),
// evaluated with the hardware exponential and the approximate divide (within
// a few ulp); e^−x overflowing to +inf gives the correctly signed zero limit.
__device__ __forceinline__ float dev_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Loads of data read once (the read-only path); stores are plain so the
// result stays in L2 for the consumer kernel that usually follows.
template <class T>
__device__ __forceinline__ T ldg_stream(const T* p) {
    return __ldg(p);
}

template <class T>
__device__ __forceinline__ void stg_stream(T* p, const T& v) {
    *p = v;
}

// Thread mapping for per-item, per-channel streaming kernels over one item of
// hw pixels × cv channel vectors: each thread keeps one channel vector j (so its
// per-channel operands live in registers) and walks pixels p, p + rows_step, ...
// Returns false for threads with no channel vector (cv does not divide the block).
struct ChanStationary {
    int j;          // channel vector of this thread
    int64_t p0;     // first pixel
    int64_t step;   // pixel stride
    __device__ __forceinline__ bool init(int cv) {
        if (cv <= (int)blockDim.x) {
            const int rows = blockDim.x / cv;
            const int r = threadIdx.x / cv;
            if (r >= rows) return false;
            j = threadIdx.x - r * cv;
            p0 = (int64_t)blockIdx.x * rows + r;
            step = (int64_t)gridDim.x * rows;
        } else {
            j = threadIdx.x;  // caller loops j += blockDim.x
            p0 = blockIdx.x;
            step = gridDim.x;
        }
        return true;
    }
};

__device__ __forceinline__ float4 f4_fma(float4 a, float4 b, float4 c) {
    return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}

}  // namespace mbx
