// The C ABI of moebius-cuda: context, memory pool, params and the kernel
// entry points. Argument checks mirror the reference engine's asserts; the
// kernels themselves live in k_*.cu.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "mbx_internal.h"

namespace {

thread_local std::string g_last_error;

int32_t set_error(int32_t code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

// Runs `f`, converting exceptions into status codes (src/ffi.rs:90-103 convention).
template <class F>
int32_t guard(F&& f) {
    try {
        f();
        return MBX_OK;
    } catch (const mbx::Error& e) {
        return set_error(e.code, e.what());
    } catch (const std::bad_alloc&) {
        return set_error(MBX_ERR_OUT_OF_MEMORY, "host allocation failed");
    } catch (const std::exception& e) {
        return set_error(MBX_ERR_INTERNAL, std::string("internal error: ") + e.what());
    } catch (...) {
        return set_error(MBX_ERR_INTERNAL, "internal error");
    }
}

void require_ctx(const mbx_ctx* ctx) { MBX_REQUIRE(ctx != nullptr, "null context"); }

void use_device(const mbx_ctx* ctx) { mbx::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice"); }

void require_ptr(const void* p, const char* what) {
    MBX_REQUIRE(p != nullptr, std::string("null pointer: ") + what);
}

// IEEE binary16 -> binary32 (exact).
float half_bits_to_float(uint16_t h) {
    uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            do {
                man <<= 1;
                ++e;
            } while (!(man & 0x400u));
            bits = sign | uint32_t(127 - 15 - e) << 23 | (man & 0x3ffu) << 13;
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | man << 13;
    } else {
        bits = sign | (exp + 127 - 15) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Nearest TF32 value (ties to even) as an f32 with the low 13 mantissa bits
// clear: the tensor core reads it exactly, and rounding keeps the 3xTF32
// split unbiased (the same rule as the kernel's A-operand split).
inline float tf32_rn(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    b = (b + 0xfffu + ((b >> 13) & 1u)) & 0xffffe000u;
    float r;
    std::memcpy(&r, &b, 4);
    return r;
}

}  // namespace

namespace mbx {

Pool::~Pool() {
    for (auto& kv : free_) cudaFree(kv.second);
    for (auto& kv : used_) cudaFree(kv.first);
}

void* Pool::alloc(size_t bytes) {
    std::lock_guard<std::mutex> lock(mu_);
    if (bytes == 0) bytes = 256;
    bytes = (bytes + 511) & ~size_t(511);
    // Best fit (Scratch::tensor_for, src/engine/mod.rs:61-66 / best_fit :104-117):
    // the smallest cached block that holds `bytes`, unless it wastes more than half.
    auto it = free_.lower_bound(bytes);
    if (it != free_.end() && it->first <= 2 * bytes + (size_t(1) << 20)) {
        void* p = it->second;
        size_t sz = it->first;
        free_.erase(it);
        cached_ -= sz;
        used_[p] = sz;
        in_use_ += sz;
        return p;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        // Give cached memory back and retry once.
        for (auto& kv : free_) cudaFree(kv.second);
        free_.clear();
        cached_ = 0;
        e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            fail(MBX_ERR_OUT_OF_MEMORY, "device allocation of " + std::to_string(bytes) + " bytes failed");
        }
    }
    used_[p] = bytes;
    in_use_ += bytes;
    return p;
}

void Pool::free(void* p) {
    std::lock_guard<std::mutex> lock(mu_);
    auto it = used_.find(p);
    if (it == used_.end()) fail(MBX_ERR_INVALID_ARGUMENT, "mbx_free: pointer not from this context's pool");
    // Most recently freed first among equal sizes (still warm in L2).
    free_.emplace_hint(free_.lower_bound(it->second), it->second, p);
    cached_ += it->second;
    in_use_ -= it->second;
    used_.erase(it);
}

void Pool::release_below(size_t min_bytes) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto it = free_.begin(); it != free_.end();) {
        if (it->first < min_bytes) {
            cudaFree(it->second);
            cached_ -= it->first;
            it = free_.erase(it);
        } else {
            ++it;
        }
    }
}

void record_error(int32_t code, const char* msg) { set_error(code, msg); }

void ensure_smem_limit(const void* kernel, int bytes, const char* what) {
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, int> set;  // (device, kernel) -> limit set
    std::lock_guard<std::mutex> lock(mu);
    int& have = set[{device, kernel}];
    if (have >= bytes) return;
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
    have = bytes;
}


}  // namespace mbx

using mbx::check_cuda;

extern "C" {

uint32_t mbx_abi_version(void) { return MBX_ABI_VERSION; }

const char* mbx_last_error(void) { return g_last_error.c_str(); }

int32_t mbx_ctx_create(int32_t device, mbx_ctx** out) {
    return guard([&] {
        require_ptr(out, "out");
        *out = nullptr;
        int count = 0;
        cudaError_t e = cudaGetDeviceCount(&count);
        if (e != cudaSuccess || count == 0) {
            (void)cudaGetLastError();
            mbx::fail(MBX_ERR_UNSUPPORTED_DEVICE, "no CUDA device available");
        }
        MBX_REQUIRE(device >= 0 && device < count, "device index out of range");
        cudaDeviceProp prop;
        check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10 || prop.minor != 0)
            mbx::fail(MBX_ERR_UNSUPPORTED_DEVICE, std::string("moebius-cuda needs an sm_100 GPU (B200); device is ") +
                                                      prop.name + " sm_" + std::to_string(prop.major) +
                                                      std::to_string(prop.minor));
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
        auto* ctx = new mbx_ctx();
        ctx->device = device;
        ctx->sm_count = prop.multiProcessorCount;
        try {
            check_cuda(cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking), "cudaStreamCreate");
            ctx->stream = ctx->own_stream;
            check_cuda(cudaMalloc(&ctx->dev_err, 4 * sizeof(int)), "cudaMalloc(dev_err)");
            check_cuda(cudaMemset(ctx->dev_err, 0, 4 * sizeof(int)), "cudaMemset(dev_err)");
            ctx->pool = new mbx::Pool(device);
        } catch (...) {
            if (ctx->dev_err) cudaFree(ctx->dev_err);
            if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
            delete ctx;
            throw;
        }
        *out = ctx;
    });
}

void mbx_ctx_destroy(mbx_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    delete ctx->pool;
    cudaFree(ctx->dev_err);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
}

int32_t mbx_ctx_set_stream(mbx_ctx* ctx, void* stream) {
    return guard([&] {
        require_ctx(ctx);
        ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    });
}

void* mbx_ctx_stream(mbx_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

uint64_t mbx_ctx_launch_count(const mbx_ctx* ctx) { return ctx ? ctx->launches : 0; }

int32_t mbx_ctx_synchronize(mbx_ctx* ctx) {
    return guard([&] {
        require_ctx(ctx);
        use_device(ctx);
        check_cuda(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        int rec[4];
        check_cuda(cudaMemcpy(rec, ctx->dev_err, sizeof(rec), cudaMemcpyDeviceToHost), "read device error record");
        if (rec[0] != mbx::kErrNone) {
            check_cuda(cudaMemset(ctx->dev_err, 0, sizeof(rec)), "clear device error record");
            mbx::fail(MBX_ERR_TIMEOUT, "device wait timed out (kernel " + std::to_string(rec[1]) + ", site " +
                                           std::to_string(rec[2]) + ")");
        }
    });
}

int32_t mbx_selftest_wait_timeout(mbx_ctx* ctx, int64_t cycles) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(cycles >= 1 && cycles <= (int64_t(1) << 32), "cycles must be in [1, 2^32]");
        use_device(ctx);
        mbx::launch_wait_probe(ctx, cycles);
    });
}

int32_t mbx_alloc(mbx_ctx* ctx, size_t bytes, void** out) {
    return guard([&] {
        require_ctx(ctx);
        require_ptr(out, "out");
        use_device(ctx);
        *out = ctx->pool->alloc(bytes);
    });
}

int32_t mbx_free(mbx_ctx* ctx, void* ptr) {
    return guard([&] {
        require_ctx(ctx);
        if (ptr) ctx->pool->free(ptr);
    });
}

int32_t mbx_pool_release_below(mbx_ctx* ctx, size_t min_bytes) {
    return guard([&] {
        require_ctx(ctx);
        use_device(ctx);
        check_cuda(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        ctx->pool->release_below(min_bytes);
    });
}

int32_t mbx_pool_stats(const mbx_ctx* ctx, size_t* cached_bytes, size_t* in_use_bytes) {
    return guard([&] {
        require_ctx(ctx);
        if (cached_bytes) *cached_bytes = ctx->pool->cached_bytes();
        if (in_use_bytes) *in_use_bytes = ctx->pool->in_use_bytes();
    });
}

int32_t mbx_host_alloc(size_t bytes, void** out) {
    return guard([&] {
        require_ptr(out, "out");
        *out = nullptr;
        check_cuda(cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocDefault), "cudaHostAlloc");
    });
}

int32_t mbx_host_free(void* ptr) {
    return guard([&] {
        if (ptr) check_cuda(cudaFreeHost(ptr), "cudaFreeHost");
    });
}

static int32_t memcpy_kind(mbx_ctx* ctx, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind) {
    return guard([&] {
        require_ctx(ctx);
        if (bytes == 0) return;
        require_ptr(dst, "dst");
        require_ptr(src, "src");
        use_device(ctx);
        check_cuda(cudaMemcpyAsync(dst, src, bytes, kind, ctx->stream), "cudaMemcpyAsync");
    });
}

int32_t mbx_memcpy_h2d(mbx_ctx* ctx, void* dst, const void* src, size_t bytes) {
    return memcpy_kind(ctx, dst, src, bytes, cudaMemcpyHostToDevice);
}
int32_t mbx_memcpy_d2h(mbx_ctx* ctx, void* dst, const void* src, size_t bytes) {
    return memcpy_kind(ctx, dst, src, bytes, cudaMemcpyDeviceToHost);
}
int32_t mbx_memcpy_d2d(mbx_ctx* ctx, void* dst, const void* src, size_t bytes) {
    return memcpy_kind(ctx, dst, src, bytes, cudaMemcpyDeviceToDevice);
}

int32_t mbx_param_create(mbx_ctx* ctx, const void* host_data, int32_t dtype, int64_t c_out, int64_t taps,
                         int64_t c_in, mbx_param** out) {
    return guard([&] {
        require_ctx(ctx);
        require_ptr(host_data, "host_data");
        require_ptr(out, "out");
        *out = nullptr;
        MBX_REQUIRE(dtype == MBX_DTYPE_F32 || dtype == MBX_DTYPE_F16, "dtype must be MBX_DTYPE_F32 or MBX_DTYPE_F16");
        MBX_REQUIRE(taps == 1 || taps == 9, "taps must be 1 (1x1) or 9 (3x3)");
        MBX_REQUIRE(c_out > 0 && c_in > 0, "c_out and c_in must be positive");
        MBX_REQUIRE(c_in <= (1 << 16) && c_out <= (1 << 16), "channel count too large");
        use_device(ctx);
        auto* p = new mbx_param();
        p->dtype = dtype;
        p->c_out = c_out;
        p->taps = taps;
        p->c_in = c_in;
        p->cin_pad = int((c_in + 31) / 32 * 32);
        p->bn = mbx::choose_bn(c_out, dtype == MBX_DTYPE_F32);
        p->cout_pad = int((c_out + p->bn - 1) / p->bn * p->bn);
        const size_t kdim = size_t(taps) * p->cin_pad;
        const size_t elems = size_t(p->cout_pad) * kdim;
        std::vector<float> hi(elems, 0.0f), lo;
        if (dtype == MBX_DTYPE_F32) lo.assign(elems, 0.0f);
        for (int64_t o = 0; o < c_out; ++o)
            for (int64_t t = 0; t < taps; ++t)
                for (int64_t i = 0; i < c_in; ++i) {
                    const size_t src = (size_t(o) * taps + t) * c_in + i;
                    const size_t dst = size_t(o) * kdim + size_t(t) * p->cin_pad + i;
                    if (dtype == MBX_DTYPE_F16) {
                        hi[dst] = half_bits_to_float(static_cast<const uint16_t*>(host_data)[src]);
                    } else {
                        const float v = static_cast<const float*>(host_data)[src];
                        hi[dst] = tf32_rn(v);
                        lo[dst] = tf32_rn(v - hi[dst]);
                    }
                }
        try {
            check_cuda(cudaMalloc(&p->hi, elems * 4), "cudaMalloc(param hi)");
            check_cuda(cudaMemcpy(p->hi, hi.data(), elems * 4, cudaMemcpyHostToDevice), "upload param hi");
            if (!lo.empty()) {
                check_cuda(cudaMalloc(&p->lo, elems * 4), "cudaMalloc(param lo)");
                check_cuda(cudaMemcpy(p->lo, lo.data(), elems * 4, cudaMemcpyHostToDevice), "upload param lo");
            }
            mbx::encode_param_tmaps(p);
        } catch (...) {
            cudaFree(p->hi);
            cudaFree(p->lo);
            delete p;
            throw;
        }
        *out = p;
    });
}

void mbx_param_destroy(mbx_ctx* ctx, mbx_param* p) {
    if (!p) return;
    if (ctx) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
    }
    cudaFree(p->hi);
    cudaFree(p->lo);
    delete p;
}

int32_t mbx_param_info(const mbx_param* p, int64_t* c_out, int64_t* taps, int64_t* c_in, int32_t* dtype) {
    return guard([&] {
        MBX_REQUIRE(p != nullptr, "null param");
        if (c_out) *c_out = p->c_out;
        if (taps) *taps = p->taps;
        if (c_in) *c_in = p->c_in;
        if (dtype) *dtype = p->dtype;
    });
}

int32_t mbx_silu_inplace(mbx_ctx* ctx, float* x, int64_t len) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(len >= 0, "negative length");
        if (len == 0) return;
        require_ptr(x, "x");
        use_device(ctx);
        mbx::launch_silu_inplace(ctx, x, len);
    });
}

int32_t mbx_add_inplace(mbx_ctx* ctx, float* a, const float* b, int64_t len) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(len >= 0, "negative length");
        if (len == 0) return;
        require_ptr(a, "a");
        require_ptr(b, "b");
        use_device(ctx);
        mbx::launch_add(ctx, a, b, a, len);
    });
}

int32_t mbx_bias_temb_add(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* bias,
                          const float* temb, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0 && c > 0, "bad shape");
        if (n * hw == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::launch_bias_temb_add(ctx, x, n, hw, c, bias, temb, out);
    });
}

int32_t mbx_concat_channels(mbx_ctx* ctx, const float* a, int64_t ca, const float* b, int64_t cb, int64_t pixels,
                            float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(ca >= 0 && cb >= 0 && pixels >= 0, "bad shape");
        if (pixels == 0 || ca + cb == 0) return;
        require_ptr(out, "out");
        MBX_REQUIRE(ca == 0 || a, "null a");
        MBX_REQUIRE(cb == 0 || b, "null b");
        MBX_REQUIRE(out != a && out != b, "concat_channels: out must alias neither input");
        use_device(ctx);
        mbx::launch_concat(ctx, a, ca, b, cb, pixels, out);
    });
}

static void check_gn(int64_t n, int64_t h, int64_t w, int64_t c, int64_t groups) {
    MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && c > 0, "bad shape");
    MBX_REQUIRE(groups > 0 && c % groups == 0, "channels not divisible by groups");
    MBX_REQUIRE(c <= 8192, "GroupNorm supports at most 8192 channels");
    MBX_REQUIRE(groups <= 1024, "GroupNorm supports at most 1024 groups");
}

static void gn_affine_impl(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t groups,
                           float eps, const float* gamma, const float* beta, const float* add, float* scale,
                           float* shift) {
    const int64_t hw = h * w;
    mbx::PoolBuf part(ctx, size_t(n) * mbx::gn_chunks(hw) * groups * 2 * sizeof(double));
    mbx::launch_gn_partials(ctx, x, n, hw, c, groups, add, part.as<double>());
    mbx::launch_gn_finalize(ctx, part.as<double>(), n, hw, c, groups, eps, gamma, beta, add, scale, shift);
}

int32_t mbx_group_norm_affine(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                              int64_t groups, float eps, const float* gamma, const float* beta, const float* add,
                              float* scale_out, float* shift_out) {
    return guard([&] {
        require_ctx(ctx);
        check_gn(n, h, w, c, groups);
        if (n == 0) return;
        MBX_REQUIRE(h * w > 0, "GroupNorm over an empty image");
        require_ptr(x, "x");
        require_ptr(gamma, "gamma");
        require_ptr(beta, "beta");
        require_ptr(scale_out, "scale_out");
        require_ptr(shift_out, "shift_out");
        use_device(ctx);
        gn_affine_impl(ctx, x, n, h, w, c, groups, eps, gamma, beta, add, scale_out, shift_out);
    });
}

int32_t mbx_group_norm_apply(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* scale,
                             const float* shift, int32_t silu, const float* residual, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0 && c > 0, "bad shape");
        if (n * hw == 0) return;
        require_ptr(x, "x");
        require_ptr(scale, "scale");
        require_ptr(shift, "shift");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::launch_gn_apply(ctx, x, n, hw, c, scale, shift, silu != 0, residual, out);
    });
}

int32_t mbx_group_norm_forward(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                               int64_t groups, float eps, const float* gamma, const float* beta, const float* add,
                               int32_t silu, float* out) {
    return guard([&] {
        require_ctx(ctx);
        check_gn(n, h, w, c, groups);
        if (n == 0) return;
        MBX_REQUIRE(h * w > 0, "GroupNorm over an empty image");
        require_ptr(x, "x");
        require_ptr(gamma, "gamma");
        require_ptr(beta, "beta");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::PoolBuf ss(ctx, size_t(n) * c * 2 * sizeof(float));
        float* scale = ss.as<float>();
        float* shift = scale + n * c;
        gn_affine_impl(ctx, x, n, h, w, c, groups, eps, gamma, beta, add, scale, shift);
        mbx::launch_gn_apply(ctx, x, n, h * w, c, scale, shift, silu != 0, nullptr, out);
    });
}

int32_t mbx_layer_norm(mbx_ctx* ctx, const float* x, int64_t tokens, int64_t c, const float* gamma,
                       const float* beta, float eps, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(tokens >= 0 && c > 0, "bad shape");
        MBX_REQUIRE(c <= 8192, "LayerNorm supports at most 8192 channels");
        if (tokens == 0) return;
        require_ptr(x, "x");
        require_ptr(gamma, "gamma");
        require_ptr(beta, "beta");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::launch_layer_norm(ctx, x, tokens, c, gamma, beta, eps, out);
    });
}

int32_t mbx_depthwise3x3(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                         const float* weight, const float* bias, int32_t epilogue, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && c > 0, "bad shape");
        MBX_REQUIRE(epilogue == MBX_EPILOGUE_NONE || epilogue == MBX_EPILOGUE_RELU ||
                        epilogue == MBX_EPILOGUE_GLU_SILU,
                    "unknown epilogue");
        MBX_REQUIRE(epilogue != MBX_EPILOGUE_GLU_SILU || c % 2 == 0, "GLU needs an even channel count");
        if (n * h * w == 0) return;
        require_ptr(x, "x");
        require_ptr(weight, "weight");
        require_ptr(bias, "bias");
        require_ptr(out, "out");
        MBX_REQUIRE(out != x, "depthwise3x3: out must not alias x");
        use_device(ctx);
        mbx::launch_depthwise3x3(ctx, x, n, h, w, c, weight, bias, epilogue, out);
    });
}

int32_t mbx_depthwise3x3_fused(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                               const float* pro_scale, const float* pro_shift, int32_t pro_silu,
                               const float* weight, const float* bias, int32_t epilogue, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && c > 0, "bad shape");
        MBX_REQUIRE(epilogue == MBX_EPILOGUE_NONE || epilogue == MBX_EPILOGUE_RELU ||
                        epilogue == MBX_EPILOGUE_GLU_SILU,
                    "unknown epilogue");
        MBX_REQUIRE(epilogue != MBX_EPILOGUE_GLU_SILU || c % 2 == 0, "GLU needs an even channel count");
        if (n * h * w == 0) return;
        require_ptr(x, "x");
        require_ptr(pro_scale, "pro_scale");
        require_ptr(pro_shift, "pro_shift");
        require_ptr(weight, "weight");
        require_ptr(bias, "bias");
        require_ptr(out, "out");
        MBX_REQUIRE(out != x, "depthwise3x3: out must not alias x");
        use_device(ctx);
        mbx::launch_depthwise3x3(ctx, x, n, h, w, c, weight, bias, epilogue, out, pro_scale, pro_shift,
                                 pro_silu != 0);
    });
}

int32_t mbx_conv1x1(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param* weight, const float* bias, const float* residual, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(weight != nullptr, "null weight");
        MBX_REQUIRE(weight->taps == 1, "Conv1x1 needs a 1x1 (taps = 1) weight");
        MBX_REQUIRE(weight->c_in == c_in, "Conv1x1 input channels");
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0, "bad shape");
        if (n * h * w == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        MBX_REQUIRE(out != x, "conv1x1: out must not alias x");

        use_device(ctx);
        mbx::ConvShape s{n, h, w, c_in, h, w, 1, 0, 0, 0};
        mbx::launch_conv_tc(ctx, x, s, weight, bias, nullptr, nullptr, false, residual, out);
    });
}

int32_t mbx_conv1x1_fused(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                          const mbx_param* weight, const float* bias, const float* pro_scale,
                          const float* pro_shift, int32_t pro_silu, const float* residual, int32_t act,
                          float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(weight != nullptr, "null weight");
        MBX_REQUIRE(weight->taps == 1, "Conv1x1 needs a 1x1 (taps = 1) weight");
        MBX_REQUIRE(weight->c_in == c_in, "Conv1x1 input channels");
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0, "bad shape");
        MBX_REQUIRE((pro_scale == nullptr) == (pro_shift == nullptr), "prologue needs both scale and shift");
        MBX_REQUIRE(act == MBX_ACT_NONE || act == MBX_ACT_SILU, "unknown activation");
        if (n * h * w == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        MBX_REQUIRE(out != x, "conv1x1: out must not alias x");
        use_device(ctx);
        mbx::ConvShape s{n, h, w, c_in, h, w, 1, 0, 0, 0};
        mbx::launch_conv_tc(ctx, x, s, weight, bias, pro_scale, pro_shift, pro_silu != 0, residual, out, act);
    });
}

int32_t mbx_conv3x3_output_hw(int64_t h, int64_t w, int64_t stride, const int64_t pad[4], int32_t upsample2x,
                              int64_t* ho, int64_t* wo) {
    return guard([&] {
        require_ptr(pad, "pad");
        require_ptr(ho, "ho");
        require_ptr(wo, "wo");
        MBX_REQUIRE(stride >= 1 && stride <= 2, "stride must be 1 or 2");
        for (int i = 0; i < 4; ++i) MBX_REQUIRE(pad[i] >= 0 && pad[i] <= 2, "padding must be in [0, 2]");
        const int64_t up = upsample2x ? 2 : 1;
        const int64_t hh = h * up + pad[0] + pad[2] - 3, ww = w * up + pad[1] + pad[3] - 3;
        MBX_REQUIRE(hh >= 0 && ww >= 0, "input smaller than the 3x3 window");
        *ho = hh / stride + 1;
        *wo = ww / stride + 1;
    });
}

int32_t mbx_conv3x3(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                    const mbx_param* weight, const float* bias, int64_t stride, const int64_t pad[4],
                    int32_t upsample2x, const float* pro_scale, const float* pro_shift, int32_t pro_silu,
                    const float* residual, float* out) {
    int64_t ho = 0, wo = 0;
    int32_t st = mbx_conv3x3_output_hw(h, w, stride, pad, upsample2x, &ho, &wo);
    if (st != MBX_OK) return st;
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(weight != nullptr, "null weight");
        MBX_REQUIRE(weight->taps == 9, "Conv3x3 needs a 3x3 (taps = 9) weight");
        MBX_REQUIRE(weight->c_in == c_in, "Conv3x3 input channels");
        MBX_REQUIRE(n >= 0 && h >= 1 && w >= 1, "bad shape");
        MBX_REQUIRE((pro_scale == nullptr) == (pro_shift == nullptr), "prologue needs both scale and shift");
        if (n == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        MBX_REQUIRE(out != x, "conv3x3: out must not alias x");
        MBX_REQUIRE((h << (upsample2x ? 1 : 0)) < (1 << 14) && (w << (upsample2x ? 1 : 0)) < (1 << 14),
                    "conv3x3: image side must be below 16384 (after the optional upsample)");
        use_device(ctx);
        mbx::ConvShape s{n, h, w, c_in, ho, wo, int(stride), int(pad[0]), int(pad[1]), upsample2x ? 1 : 0};
        mbx::launch_conv_tc(ctx, x, s, weight, bias, pro_scale, pro_shift, pro_silu != 0, residual, out);
    });
}

int32_t mbx_conv_group_norm_affine(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in,
                                   const mbx_param* weight, const float* bias, int64_t stride, const int64_t pad[4],
                                   int32_t upsample2x, const float* pro_scale, const float* pro_shift,
                                   int32_t pro_silu, const float* residual, int32_t act, float* out, int64_t groups,
                                   float eps, const float* gamma, const float* beta, const float* add,
                                   float* scale_out, float* shift_out) {
    int64_t ho = h, wo = w;
    if (weight && weight->taps == 9) {
        const int32_t st = mbx_conv3x3_output_hw(h, w, stride, pad, upsample2x, &ho, &wo);
        if (st != MBX_OK) return st;
    }
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(weight != nullptr, "null weight");
        MBX_REQUIRE(weight->c_in == c_in, "conv input channels");
        MBX_REQUIRE(weight->taps == 9 || (stride == 1 && !upsample2x), "a 1x1 conv takes stride 1 and no upsample");
        MBX_REQUIRE(n >= 0 && h >= 1 && w >= 1, "bad shape");
        MBX_REQUIRE((pro_scale == nullptr) == (pro_shift == nullptr), "prologue needs both scale and shift");
        MBX_REQUIRE(act == MBX_ACT_NONE || act == MBX_ACT_SILU, "unknown activation");
        check_gn(n, ho, wo, weight->c_out, groups);
        if (n == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        require_ptr(gamma, "gamma");
        require_ptr(beta, "beta");
        require_ptr(scale_out, "scale_out");
        require_ptr(shift_out, "shift_out");
        MBX_REQUIRE(out != x, "conv: out must not alias x");
        if (weight->taps == 9)
            MBX_REQUIRE((h << (upsample2x ? 1 : 0)) < (1 << 14) && (w << (upsample2x ? 1 : 0)) < (1 << 14),
                        "conv3x3: image side must be below 16384 (after the optional upsample)");
        use_device(ctx);
        const int64_t c_out = weight->c_out;
        const mbx::ConvShape s = weight->taps == 9
                                     ? mbx::ConvShape{n, h, w, c_in, ho, wo, int(stride), int(pad[0]), int(pad[1]),
                                                      upsample2x ? 1 : 0}
                                     : mbx::ConvShape{n, h, w, c_in, h, w, 1, 0, 0, 0};
        if (mbx::conv_gn_fusable(s, c_out)) {
            // Statistics gathered by the conv's epilogue, folded, then the usual finalize.
            mbx::PoolBuf tiles(ctx, size_t(mbx::conv_gn_part_floats(s, c_out)) * sizeof(float));
            mbx::launch_conv_tc(ctx, x, s, weight, bias, pro_scale, pro_shift, pro_silu != 0, residual, out, act,
                                tiles.as<float>(), add);
            const int64_t hw = ho * wo;
            mbx::PoolBuf part(ctx, size_t(n) * mbx::gn_chunks(hw) * groups * 2 * sizeof(double));
            mbx::launch_gn_fold_tiles(ctx, tiles.as<float>(), n, hw, c_out, groups, part.as<double>());
            mbx::launch_gn_finalize(ctx, part.as<double>(), n, hw, c_out, groups, eps, gamma, beta, add, scale_out,
                                    shift_out);
        } else {
            // Output maps that are not a multiple of 256 pixels (or c_out % 4 != 0): a separate pass.
            mbx::launch_conv_tc(ctx, x, s, weight, bias, pro_scale, pro_shift, pro_silu != 0, residual, out, act);
            gn_affine_impl(ctx, out, n, ho, wo, c_out, groups, eps, gamma, beta, add, scale_out, shift_out);
        }
    });
}

int32_t mbx_softmax_rows(mbx_ctx* ctx, float* x, int64_t rows, int64_t n, float scale, float flush) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(rows >= 0 && n >= 0, "bad shape");
        if (rows == 0 || n == 0) return;
        require_ptr(x, "x");
        use_device(ctx);
        mbx::launch_softmax_rows(ctx, x, rows, n, scale, flush);
    });
}

int32_t mbx_gemm(mbx_ctx* ctx, float* c, const float* a, int64_t m, int64_t k, const float* b, int64_t n,
                 int32_t b_is_kn, const float* bias, const float* residual) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(m >= 0 && n > 0 && k > 0, "bad shape");
        MBX_REQUIRE(n <= (1 << 20) && k <= (1 << 20), "gemm: n or k too large");
        if (m == 0) return;
        require_ptr(c, "c");
        require_ptr(a, "a");
        require_ptr(b, "b");
        MBX_REQUIRE(c != a && c != b, "gemm: c must alias neither a nor b");
        use_device(ctx);
        // B becomes a transient tensor-core operand: TF32 hi/lo, K-major, zero padded.
        mbx_param p;
        p.dtype = MBX_DTYPE_F32;
        p.c_out = n;
        p.taps = 1;
        p.c_in = k;
        p.cin_pad = int((k + 31) / 32 * 32);
        p.bn = mbx::choose_bn(n, true);
        p.cout_pad = int((n + p.bn - 1) / p.bn * p.bn);
        const size_t elems = size_t(p.cout_pad) * p.cin_pad;
        mbx::PoolBuf hi(ctx, elems * 4), lo(ctx, elems * 4);
        p.hi = hi.as<float>();
        p.lo = lo.as<float>();
        mbx::launch_split_to_param(ctx, b, n, k, b_is_kn != 0, &p);
        mbx::encode_param_tmaps(&p);
        mbx::ConvShape s{1, m, 1, k, m, 1, 1, 0, 0, 0};
        mbx::launch_conv_tc(ctx, a, s, &p, bias, nullptr, nullptr, false, residual, c);
    });
}

int32_t mbx_scale_add(mbx_ctx* ctx, const float* x, int64_t len, float mul, float add, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(len >= 0, "negative length");
        if (len == 0) return;
        require_ptr(x, "x");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::launch_scale_add(ctx, x, len, mul, add, out);
    });
}

int32_t mbx_lambda_content(mbx_ctx* ctx, const float* keys, int64_t key_stride, const float* values,
                           int64_t value_stride, int64_t items, int64_t rows, int64_t k, int64_t vd,
                           float* lambda_out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(items >= 0 && rows >= 1 && k >= 1 && vd >= 1, "bad shape");
        MBX_REQUIRE(key_stride >= k && value_stride >= vd, "row strides smaller than the widths");
        if (items == 0) return;
        require_ptr(keys, "keys");
        require_ptr(values, "values");
        require_ptr(lambda_out, "lambda_out");
        use_device(ctx);
        const int64_t chunks = mbx::lambda_chunks(rows);
        mbx::PoolBuf pmax(ctx, size_t(items * chunks * k) * 4), psum(ctx, size_t(items * chunks * k) * 4);
        mbx::PoolBuf plam(ctx, size_t(items * chunks * k * vd) * 4);
        mbx::launch_lambda_content(ctx, keys, key_stride, values, value_stride, items, rows, k, vd,
                                   pmax.as<float>(), plam.as<float>(), psum.as<float>(), lambda_out);
    });
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

int32_t mbx_self_lambda_position(mbx_ctx* ctx, const float* q, const float* lambda_c, const float* a,
                                 int64_t a_stride, const float* v, int64_t v_stride, int64_t n, int64_t h,
                                 int64_t w, int64_t k, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 1 && w >= 1, "bad shape");
        MBX_REQUIRE(k >= 8 && k % 8 == 0, "self lambda: head width must be a positive multiple of 8");
        MBX_REQUIRE(a_stride >= 228 && a_stride % 4 == 0, "self lambda: a_stride must be >= 228 and a multiple of 4");
        MBX_REQUIRE(v_stride >= k && v_stride % 4 == 0, "self lambda: v_stride must be >= k and a multiple of 4");
        MBX_REQUIRE(h < (1 << 20) && w < (1 << 20), "self lambda: map too large");
        if (n == 0) return;
        for (const void* p : {(const void*)q, (const void*)lambda_c, (const void*)a, (const void*)v, (const void*)out})
            require_ptr(p, "operand");
        MBX_REQUIRE(aligned16(q) && aligned16(a) && aligned16(v) && aligned16(out),
                    "self lambda: q, a, v and out must be 16-byte aligned");
        MBX_REQUIRE(out != q && out != a, "self lambda: out must alias neither q nor a");
        use_device(ctx);
        mbx::launch_self_position(ctx, q, lambda_c, a, a_stride, v, v_stride, n, h, w, k, out);
    });
}

int32_t mbx_cross_lambda_position(mbx_ctx* ctx, const float* q, const float* e_table, const float* lambda_c,
                                  const float* v_table, int64_t branch_period, int64_t n, int64_t hw, int64_t k,
                                  float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 1, "bad shape");
        MBX_REQUIRE(k >= 8 && k % 8 == 0, "cross lambda: head width must be a positive multiple of 8");
        MBX_REQUIRE(branch_period >= 1 && branch_period <= 1024, "cross lambda: bad branch period");
        if (n == 0) return;
        for (const void* p : {(const void*)q, (const void*)e_table, (const void*)lambda_c, (const void*)v_table,
                              (const void*)out})
            require_ptr(p, "operand");
        MBX_REQUIRE(aligned16(q) && aligned16(e_table) && aligned16(out),
                    "cross lambda: q, e_table and out must be 16-byte aligned");
        MBX_REQUIRE(out != q, "cross lambda: out must not alias q");
        use_device(ctx);
        mbx::launch_cross_position(ctx, q, e_table, lambda_c, v_table, branch_period, n, hw, k, out);
    });
}

int32_t mbx_inpaint_prepare(mbx_ctx* ctx, const uint8_t* image, const uint8_t* mask, int64_t n, int64_t h,
                            int64_t w, int64_t channels, float* images_out, uint8_t* bin_out, float* mask_lat,
                            int32_t* nonempty_out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 8 && w >= 8 && h % 8 == 0 && w % 8 == 0,
                    "inpaint: image sides must be positive multiples of 8");
        MBX_REQUIRE(channels == 3 || channels == 4, "image must be RGB or RGBA");
        if (n == 0) return;
        for (const void* p : {(const void*)image, (const void*)mask, (const void*)images_out, (const void*)bin_out,
                              (const void*)mask_lat})
            require_ptr(p, "operand");
        use_device(ctx);
        mbx::launch_inpaint_prepare(ctx, image, mask, n, h, w, (int)channels, images_out, bin_out, mask_lat,
                                    nonempty_out);
    });
}

int32_t mbx_vae_sample(mbx_ctx* ctx, const float* moments, const float* noise, int64_t pixels, float scale,
                       float* z) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(pixels >= 0, "bad shape");
        if (pixels == 0) return;
        require_ptr(moments, "moments");
        require_ptr(noise, "noise");
        require_ptr(z, "z");
        use_device(ctx);
        mbx::launch_vae_sample(ctx, moments, noise, pixels, scale, z);
    });
}

int32_t mbx_latents_init(mbx_ctx* ctx, const float* z_pairs, const float* noise_init, const float* noise_offset,
                         int64_t n, int64_t hw, float noise_offset_scale, float sqrt_alpha,
                         float sqrt_one_minus_alpha, int32_t pure_noise, float* x) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0, "bad shape");
        if (n * hw == 0) return;
        MBX_REQUIRE(pure_noise || z_pairs != nullptr, "null pointer: z_pairs");
        require_ptr(noise_init, "noise_init");
        require_ptr(noise_offset, "noise_offset");
        require_ptr(x, "x");
        use_device(ctx);
        mbx::launch_latents_init(ctx, z_pairs, noise_init, noise_offset, n, hw, noise_offset_scale, sqrt_alpha,
                                 sqrt_one_minus_alpha, pure_noise != 0, x);
    });
}

int32_t mbx_unet_input(mbx_ctx* ctx, const float* x, const float* mask_lat, const float* z_pairs, int64_t n,
                       int64_t hw, int64_t copies, float* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0, "bad shape");
        MBX_REQUIRE(copies == 1 || copies == 2, "copies must be 1 or 2");
        if (n * hw == 0) return;
        for (const void* p : {(const void*)x, (const void*)mask_lat, (const void*)z_pairs, (const void*)out})
            require_ptr(p, "operand");
        use_device(ctx);
        mbx::launch_unet_input(ctx, x, mask_lat, z_pairs, n, hw, (int)copies, out);
    });
}

int32_t mbx_cfg_ddim_step(mbx_ctx* ctx, const float* eps, int64_t n, int64_t hw, int64_t copies, float guidance,
                          const float coef[4], float* x) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0, "bad shape");
        MBX_REQUIRE(copies == 1 || copies == 2, "copies must be 1 or 2");
        require_ptr(coef, "coef");
        if (n * hw == 0) return;
        require_ptr(eps, "eps");
        require_ptr(x, "x");
        use_device(ctx);
        mbx::launch_cfg_ddim(ctx, eps, n, hw * 4, (int)copies, guidance, coef, x);
    });
}

int32_t mbx_gaussian_blur_u8(mbx_ctx* ctx, const uint8_t* in, int64_t n, int64_t h, int64_t w, float radius,
                             uint8_t* scratch, uint8_t* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0, "bad shape");
        MBX_REQUIRE(h <= 16384 && w <= 16384, "blur: sides above 16384");
        if (n * h * w == 0) return;
        require_ptr(in, "in");
        require_ptr(out, "out");
        use_device(ctx);
        if (radius > 0.0f) require_ptr(scratch, "scratch");
        mbx::gaussian_blur(ctx, in, n, h, w, radius, scratch, out);
    });
}

int32_t mbx_feather_paste(mbx_ctx* ctx, const float* result, const uint8_t* blurred, uint8_t* image, int64_t n,
                          int64_t h, int64_t w, int64_t channels, const int32_t* nonempty) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0, "bad shape");
        MBX_REQUIRE(channels == 3 || channels == 4, "image must be RGB or RGBA");
        if (n * h * w == 0) return;
        require_ptr(result, "result");
        require_ptr(blurred, "blurred");
        require_ptr(image, "image");
        use_device(ctx);
        mbx::launch_feather_paste(ctx, result, blurred, image, n * h * w, h * w, (int)channels, nonempty);
    });
}

int32_t mbx_cfg_dpm_step(mbx_ctx* ctx, const float* eps, int64_t n, int64_t hw, int64_t copies, float guidance,
                         const float coef[5], int32_t order, float* x, float* x0_prev) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && hw >= 0, "bad shape");
        MBX_REQUIRE(copies == 1 || copies == 2, "copies must be 1 (cond only) or 2 (uncond, cond)");
        MBX_REQUIRE(order >= 0 && order <= 2, "order must be 0, 1 or 2");
        if (n * hw == 0) return;
        require_ptr(eps, "eps");
        require_ptr(coef, "coef");
        require_ptr(x, "x");
        if (order > 0) require_ptr(x0_prev, "x0_prev");
        use_device(ctx);
        mbx::launch_cfg_dpm(ctx, eps, n, hw * 4, (int)copies, guidance, coef, order, x, x0_prev);
    });
}

int32_t mbx_crop_window(uint32_t bx, uint32_t by, uint32_t bw, uint32_t bh, uint32_t width, uint32_t height,
                        int64_t model_side, int64_t window[3], mbx_rect* source) {
    return guard([&] {
        MBX_REQUIRE(window != nullptr, "null argument");
        MBX_REQUIRE(width > 0 && height > 0 && model_side > 0, "empty image");
        MBX_REQUIRE(bw > 0 && bh > 0 && (uint64_t)bx + bw <= width && (uint64_t)by + bh <= height,
                    "mask bbox outside the image");
        const mbx::CropWindow c = mbx::crop_window(bx, by, bw, bh, width, height, model_side);
        window[0] = c.x;
        window[1] = c.y;
        window[2] = c.side;
        if (source) *source = mbx::source_rect(c, width, height);
    });
}

int32_t mbx_lanczos_table(int64_t in_size, int64_t out_size, int32_t* bounds, int32_t* coeffs, int64_t* ksize) {
    return guard([&] {
        MBX_REQUIRE(ksize != nullptr, "null argument");
        MBX_REQUIRE(in_size > 0 && out_size > 0 && in_size <= (1 << 20) && out_size <= (1 << 20), "bad sizes");
        MBX_REQUIRE(!bounds || coeffs, "coeffs must accompany bounds");
        mbx::lanczos_table(in_size, out_size, bounds, coeffs, ksize);
    });
}

int32_t mbx_mask_dilate(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t mask_stride,
                        int64_t k, uint8_t* scratch, uint8_t* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && mask_stride >= w && k >= 0, "bad shape");
        if (n * h * w == 0) return;
        require_ptr(mask, "mask");
        require_ptr(out, "out");
        if (k > 1) require_ptr(scratch, "scratch");
        use_device(ctx);
        mbx::launch_mask_dilate(ctx, mask, n, h, w, mask_stride, k, scratch, out);
    });
}

int32_t mbx_mask_bbox(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t mask_stride,
                      int32_t* box) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && h > 0 && w > 0 && mask_stride >= w, "bad shape");
        MBX_REQUIRE(h * w < INT32_MAX, "mask too large");
        if (n == 0) return;
        require_ptr(mask, "mask");
        require_ptr(box, "box");
        MBX_REQUIRE(n <= 65535, "at most 65535 masks per call");
        use_device(ctx);
        mbx::launch_mask_bbox(ctx, mask, n, h, w, mask_stride, box);
    });
}

namespace {
void require_region(int64_t stride, int64_t channels, int64_t mask_stride, int64_t origin_x, int64_t origin_y,
                    int64_t region_w, int64_t region_h, int64_t width, int64_t height) {
    MBX_REQUIRE(channels == 3 || channels == 4, "image must be RGB or RGBA");
    MBX_REQUIRE(width > 0 && height > 0, "empty image");
    MBX_REQUIRE(region_w > 0 && region_h > 0 && origin_x >= 0 && origin_y >= 0 && origin_x + region_w <= width &&
                    origin_y + region_h <= height,
                "region outside the image");
    MBX_REQUIRE(stride >= region_w * channels && mask_stride >= region_w,
                "buffer smaller than width, height and stride imply");
}
}  // namespace

int32_t mbx_window_to_model(mbx_ctx* ctx, const uint8_t* image, int64_t stride, int64_t channels,
                            const uint8_t* mask, int64_t mask_stride, int64_t origin_x, int64_t origin_y,
                            int64_t region_w, int64_t region_h, int64_t width, int64_t height, int64_t win_x,
                            int64_t win_y, int64_t side, int64_t model_side, uint8_t* rgb_out, uint8_t* bin_out) {
    return guard([&] {
        require_ctx(ctx);
        require_region(stride, channels, mask_stride, origin_x, origin_y, region_w, region_h, width, height);
        MBX_REQUIRE(side > 0 && model_side > 0 && side <= (1 << 16) && model_side <= (1 << 16), "bad window");
        // Edge replication reads the window's part inside the image: the region must hold it.
        const int64_t sx0 = std::max<int64_t>(win_x, 0), sy0 = std::max<int64_t>(win_y, 0);
        const int64_t sx1 = std::min<int64_t>(win_x + side, width), sy1 = std::min<int64_t>(win_y + side, height);
        MBX_REQUIRE(sx1 > sx0 && sy1 > sy0, "window outside the image");
        MBX_REQUIRE(sx0 >= origin_x && sy0 >= origin_y && sx1 <= origin_x + region_w && sy1 <= origin_y + region_h,
                    "region does not cover the window's part inside the image");
        require_ptr(image, "image");
        require_ptr(mask, "mask");
        require_ptr(rgb_out, "rgb_out");
        require_ptr(bin_out, "bin_out");
        use_device(ctx);
        // Clamped coordinates stay inside [sx0, sx1) x [sy0, sy1), which the region covers.
        mbx::launch_window_to_model(ctx, image, stride, channels, mask, mask_stride, origin_x, origin_y, width, height,
                                    win_x, win_y, side, model_side, rgb_out, bin_out);
    });
}

int32_t mbx_model_to_window(mbx_ctx* ctx, const float* rgb, int64_t n, int64_t model_side, int64_t side,
                            uint8_t* out) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(n >= 0 && model_side > 0 && side > 0 && side <= (1 << 16) && model_side <= (1 << 16),
                    "bad shape");
        if (n == 0) return;
        require_ptr(rgb, "rgb");
        require_ptr(out, "out");
        use_device(ctx);
        mbx::launch_model_to_window(ctx, rgb, n, model_side, side, out);
    });
}

int32_t mbx_paste(mbx_ctx* ctx, uint8_t* image, int64_t n, int64_t stride, int64_t channels, const uint8_t* mask,
                  int64_t mask_stride, int64_t origin_x, int64_t origin_y, int64_t region_w, int64_t region_h,
                  int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, const uint8_t* result,
                  uint32_t mode, const int32_t* active) {
    return guard([&] {
        require_ctx(ctx);
        require_region(stride, channels, mask_stride, origin_x, origin_y, region_w, region_h, width, height);
        MBX_REQUIRE(mode >= 1 && mode <= 3, "paste mode must be NONE (1), FEATHER (2) or FEATHER_COMPENSATE (3)");
        MBX_REQUIRE(n >= 0 && side > 0 && side <= (1 << 16), "bad shape");
        MBX_REQUIRE(n <= 65535, "at most 65535 images per call");
        if (n == 0) return;
        require_ptr(image, "image");
        require_ptr(mask, "mask");
        require_ptr(result, "result");
        use_device(ctx);
        mbx::launch_paste(ctx, image, n, stride, channels, mask, mask_stride, origin_x, origin_y, region_w, region_h,
                          width, height, win_x, win_y, side, result, mode, active);
    });
}

int32_t mbx_matmul(mbx_ctx* ctx, float* c, const float* a, int64_t m, int64_t k, int64_t a_row_stride,
                   int64_t a_col_stride, const float* b, int64_t n, int64_t b_row_stride, int64_t b_col_stride,
                   int32_t accumulate) {
    return guard([&] {
        require_ctx(ctx);
        MBX_REQUIRE(m >= 0 && n >= 0 && k >= 0, "bad shape");
        MBX_REQUIRE(a_row_stride >= 0 && a_col_stride >= 0 && b_row_stride >= 0 && b_col_stride >= 0,
                    "negative stride");
        if (m == 0 || n == 0) return;
        require_ptr(c, "c");
        MBX_REQUIRE(k == 0 || (a && b), "null operand");
        use_device(ctx);
        mbx::launch_matmul_simt(ctx, c, a, m, k, a_row_stride, a_col_stride, b, n, b_row_stride, b_col_stride,
                                accumulate != 0);
    });
}

}  // extern "C"
