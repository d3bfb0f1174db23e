// Device-side helpers shared by the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mbx {

// x·σ(x) = x / (1 + e^−x), the reference's SiLU (src/engine/math.rs:34-36),
// evaluated with the hardware exponential; e^−x overflowing to +inf gives
// the correctly signed zero limit.
__device__ __forceinline__ float dev_silu(float x) { return x / (1.0f + __expf(-x)); }

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

__device__ __forceinline__ float4 f4_fma(float4 a, float4 b, float4 c) {
    return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}

}  // namespace mbx
