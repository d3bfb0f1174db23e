// Host-side engine above the kernel ABI: the reference's callers of its engine
// layer (src/unet/*, src/vae/*, src/scheduler.rs, src/pipeline.rs) re-built in
// C++ on the mbx_* entry points. Internal to libmoebius_cuda.so.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "mbx_internal.h"

namespace mbx {
namespace eng {

// Raises the status of a failed mbx_* call (with its message) as an exception.
void ck(int32_t status);

// NHWC f32 activation on the device, from the context's stream-ordered pool (the
// reference's Tensor + Scratch pair, src/engine/tensor.rs:12-34, src/engine/mod.rs:25-117).
class Tensor {
public:
    Tensor() = default;
    Tensor(mbx_ctx* ctx, int64_t n, int64_t h, int64_t w, int64_t c);
    ~Tensor();
    Tensor(Tensor&& o) noexcept { *this = std::move(o); }
    Tensor& operator=(Tensor&& o) noexcept;
    Tensor(const Tensor&) = delete;
    Tensor& operator=(const Tensor&) = delete;
    // A non-owning view of caller memory (never freed here).
    static Tensor view(mbx_ctx* ctx, float* p, int64_t n, int64_t h, int64_t w, int64_t c);

    float* data() const { return p_; }
    float* item(int64_t i) const { return p_ + i * h * w * c; }
    int64_t size() const { return n * h * w * c; }
    int64_t pixels() const { return n * h * w; }
    explicit operator bool() const { return p_ != nullptr; }
    mbx_ctx* ctx() const { return ctx_; }

    int64_t n = 0, h = 0, w = 0, c = 0;

private:
    mbx_ctx* ctx_ = nullptr;
    Pool* pool_ = nullptr;  // the pool the block came from (a graph runner may swap the context's pool)
    float* p_ = nullptr;
};

// Long-lived device array (weights, constants): cudaMalloc'd, freed on destruction.
class DevBuf {
public:
    DevBuf() = default;
    explicit DevBuf(size_t bytes);
    DevBuf(const void* host, size_t bytes);  // upload (synchronous)
    ~DevBuf();
    DevBuf(DevBuf&& o) noexcept { *this = std::move(o); }
    DevBuf& operator=(DevBuf&& o) noexcept;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    float* f() const { return static_cast<float*>(p_); }
    void* get() const { return p_; }
    size_t bytes() const { return bytes_; }

private:
    void* p_ = nullptr;
    size_t bytes_ = 0;
};

// A dense conv / linear weight in its stored precision (mbx_param).
class Param {
public:
    Param() = default;
    Param(mbx_ctx* ctx, const void* host, int32_t dtype, int64_t c_out, int64_t taps, int64_t c_in);
    ~Param();
    Param(Param&& o) noexcept { *this = std::move(o); }
    Param& operator=(Param&& o) noexcept;
    Param(const Param&) = delete;
    Param& operator=(const Param&) = delete;
    const mbx_param* get() const { return p_; }
    int64_t c_out() const { return p_ ? p_->c_out : 0; }
    int64_t c_in() const { return p_ ? p_->c_in : 0; }
    int64_t taps() const { return p_ ? p_->taps : 0; }

private:
    mbx_ctx* ctx_ = nullptr;
    mbx_param* p_ = nullptr;
};

// One safetensors file held in memory.
struct StTensor {
    std::string dtype;  // "F32" | "F16"
    std::vector<int64_t> shape;
    const uint8_t* data = nullptr;
    size_t bytes = 0;
};

class StFile {
public:
    explicit StFile(const std::string& path);
    const StTensor* find(const std::string& name) const;
    std::string metadata(const std::string& key) const;

private:
    std::vector<uint8_t> buf_;
    std::map<std::string, StTensor> tensors_;
    std::map<std::string, std::string> meta_;
};

// Prefix-scoped, shape-checked access to the converted weights (reference
// src/unet/load.rs:14-98). Dense weights keep their stored precision.
class Loader {
public:
    Loader(mbx_ctx* ctx, const StFile* f, std::string prefix) : ctx_(ctx), f_(f), prefix_(std::move(prefix)) {}
    Loader sub(const std::string& name) const { return Loader(ctx_, f_, key(name)); }
    std::string key(const std::string& leaf) const { return prefix_.empty() ? leaf : prefix_ + "." + leaf; }
    bool has(const std::string& name) const { return f_->find(key(name)) != nullptr; }
    std::vector<int64_t> shape(const std::string& name) const;
    // Any stored tensor widened to host f32, checked against `shape`.
    std::vector<float> f32s(const std::string& name, const std::vector<int64_t>& shape) const;
    DevBuf vec(const std::string& name, int64_t len) const;
    // `<name>` [c_out, c_in] (taps 1) or [c_out, 3, 3, c_in] (taps 9).
    Param param(const std::string& name, int64_t c_out, int64_t taps, int64_t c_in) const;
    // Raw stored tensor (for weights concatenated at load).
    const StTensor& raw(const std::string& name, const std::vector<int64_t>& shape) const;
    mbx_ctx* ctx() const { return ctx_; }

private:
    mbx_ctx* ctx_;
    const StFile* f_;
    std::string prefix_;
};

// A 1×1 or 3×3 conv with its bias (Conv1x1 / Conv3x3, src/engine/conv.rs:17-106).
struct Conv {
    Param w;
    DevBuf b;
    int64_t c_in = 0, c_out = 0;
    int stride = 1;
    int64_t pad[4] = {1, 1, 1, 1};
    bool up = false;
    static Conv load1x1(const Loader& l, const std::string& name, int64_t c_in, int64_t c_out, bool bias);
    static Conv load3x3(const Loader& l, const std::string& name, int64_t c_in, int64_t c_out);
};

struct GroupNormP {
    DevBuf gamma, beta;
    int64_t c = 0, groups = 32;
    float eps = 1e-5f;
    static GroupNormP load(const Loader& l, const std::string& name, int64_t c, float eps);
};

// Conv helpers on the kernel ABI. `out` is allocated here.
Tensor conv1x1(const Tensor& x, const Conv& cv, const float* residual = nullptr, const float* pro_scale = nullptr,
               const float* pro_shift = nullptr, bool pro_silu = false, int act = MBX_ACT_NONE);
Tensor conv3x3(const Tensor& x, const Conv& cv, const float* pro_scale = nullptr, const float* pro_shift = nullptr,
               bool pro_silu = false, const float* residual = nullptr);
// GroupNorm affine (per-item scale/shift [n, c]); `add` [n, c] or null.
void gn_affine(const Tensor& x, const GroupNormP& g, const float* add, Tensor& scale, Tensor& shift);

// The GroupNorm that will consume a conv's output: the conv gathers its statistics in its epilogue
// (mbx_conv_group_norm_affine) and fills scale / shift, so the output is not read again for them.
struct NextNorm {
    const GroupNormP* g = nullptr;
    const float* add = nullptr;  // [n, c] or null (the resnets' time embedding)
    Tensor* scale = nullptr;
    Tensor* shift = nullptr;
};
Tensor conv_gn(const Tensor& x, const Conv& cv, const NextNorm& next, const float* residual = nullptr,
               const float* pro_scale = nullptr, const float* pro_shift = nullptr, bool pro_silu = false);

uint16_t f32_to_f16(float v);
float f16_to_f32(uint16_t h);

}  // namespace eng
}  // namespace mbx
