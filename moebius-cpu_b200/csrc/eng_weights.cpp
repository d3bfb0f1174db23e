// Engine support: device tensors, weight parameters and the safetensors reader
// (the format of the reference's converted weights, src/weights.rs).
#include <cstdio>
#include <cstring>
#include <fstream>

#include "eng.h"

namespace mbx {
namespace eng {

void ck(int32_t status) {
    if (status != MBX_OK) throw Error(status, mbx_last_error());
}

// ---------------------------------------------------------------- Tensor

Tensor::Tensor(mbx_ctx* ctx, int64_t n_, int64_t h_, int64_t w_, int64_t c_)
    : n(n_), h(h_), w(w_), c(c_), ctx_(ctx), pool_(ctx->pool) {
    MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && c >= 0, "negative tensor shape");
    const size_t bytes = size_t(size()) * sizeof(float);
    p_ = bytes ? static_cast<float*>(pool_->alloc(bytes)) : nullptr;
}

Tensor Tensor::view(mbx_ctx* ctx, float* p, int64_t n, int64_t h, int64_t w, int64_t c) {
    Tensor t;
    t.ctx_ = ctx;
    t.pool_ = nullptr;
    t.p_ = p;
    t.n = n;
    t.h = h;
    t.w = w;
    t.c = c;
    return t;
}

Tensor::~Tensor() {
    if (p_ && pool_) {
        try {
            pool_->free(p_);
        } catch (...) {
        }
    }
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this != &o) {
        if (p_ && pool_) {
            try {
                pool_->free(p_);
            } catch (...) {
            }
        }
        ctx_ = o.ctx_;
        pool_ = o.pool_;
        p_ = o.p_;
        n = o.n;
        h = o.h;
        w = o.w;
        c = o.c;
        o.p_ = nullptr;
    }
    return *this;
}

// ---------------------------------------------------------------- DevBuf

DevBuf::DevBuf(size_t bytes) : bytes_(bytes) {
    if (bytes) check_cuda(cudaMalloc(&p_, bytes), "cudaMalloc (weights)");
}

DevBuf::DevBuf(const void* host, size_t bytes) : DevBuf(bytes) {
    if (bytes) check_cuda(cudaMemcpy(p_, host, bytes, cudaMemcpyHostToDevice), "weight upload");
}

DevBuf::~DevBuf() {
    if (p_) cudaFree(p_);
}

DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
    if (this != &o) {
        if (p_) cudaFree(p_);
        p_ = o.p_;
        bytes_ = o.bytes_;
        o.p_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

// ---------------------------------------------------------------- Param

Param::Param(mbx_ctx* ctx, const void* host, int32_t dtype, int64_t c_out, int64_t taps, int64_t c_in) : ctx_(ctx) {
    ck(mbx_param_create(ctx, host, dtype, c_out, taps, c_in, &p_));
}

Param::~Param() {
    if (p_) mbx_param_destroy(ctx_, p_);
}

Param& Param::operator=(Param&& o) noexcept {
    if (this != &o) {
        if (p_) mbx_param_destroy(ctx_, p_);
        ctx_ = o.ctx_;
        p_ = o.p_;
        o.p_ = nullptr;
    }
    return *this;
}

// ---------------------------------------------------------------- f16

float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
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

// Round-to-nearest-even f32 → f16 (used only for values that came from f16).
uint16_t f32_to_f16(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    const uint32_t sign = (b >> 16) & 0x8000u;
    const int32_t exp = int32_t((b >> 23) & 0xffu) - 127 + 15;
    uint32_t man = b & 0x7fffffu;
    if (((b >> 23) & 0xffu) == 0xffu) return uint16_t(sign | 0x7c00u | (man ? 0x200u : 0u));
    if (exp >= 0x1f) return uint16_t(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return uint16_t(sign);
        man |= 0x800000u;
        const int shift = 14 - exp;
        uint32_t r = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return uint16_t(sign | r);
    }
    uint32_t r = (uint32_t(exp) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return uint16_t(sign | r);
}

// ---------------------------------------------------------------- safetensors

namespace {

// Minimal JSON reader for the safetensors header: objects, arrays, strings,
// integers (all the header holds).
struct Json {
    const char* s;
    const char* e;
    void ws() {
        while (s < e && (*s == ' ' || *s == '\n' || *s == '\r' || *s == '\t')) ++s;
    }
    void expect(char c) {
        ws();
        if (s >= e || *s != c) fail(MBX_ERR_WEIGHTS, std::string("safetensors header: expected '") + c + "'");
        ++s;
    }
    bool peek(char c) {
        ws();
        return s < e && *s == c;
    }
    std::string str() {
        expect('"');
        std::string out;
        while (s < e && *s != '"') {
            if (*s == '\\') {
                ++s;
                if (s >= e) break;
                switch (*s) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (e - s < 5) fail(MBX_ERR_WEIGHTS, "safetensors header: bad escape");
                        const unsigned cp = (unsigned)std::stoul(std::string(s + 1, s + 5), nullptr, 16);
                        out += cp < 0x80 ? char(cp) : '?';
                        s += 4;
                        break;
                    }
                    default: out += *s;
                }
                ++s;
            } else {
                out += *s++;
            }
        }
        expect('"');
        return out;
    }
    int64_t integer() {
        ws();
        const char* b = s;
        if (s < e && (*s == '-' || *s == '+')) ++s;
        while (s < e && *s >= '0' && *s <= '9') ++s;
        if (b == s) fail(MBX_ERR_WEIGHTS, "safetensors header: expected an integer");
        return std::stoll(std::string(b, s));
    }
    std::vector<int64_t> int_array() {
        std::vector<int64_t> v;
        expect('[');
        if (peek(']')) {
            ++s;
            return v;
        }
        for (;;) {
            v.push_back(integer());
            if (peek(',')) {
                ++s;
                continue;
            }
            expect(']');
            return v;
        }
    }
};

}  // namespace

StFile::StFile(const std::string& path) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) fail(MBX_ERR_IO, "cannot open " + path);
    const std::streamsize size = in.tellg();
    in.seekg(0);
    buf_.resize(size_t(size));
    if (size < 8 || !in.read(reinterpret_cast<char*>(buf_.data()), size)) fail(MBX_ERR_IO, "cannot read " + path);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | buf_[size_t(i)];
    if (hlen > uint64_t(size) - 8) fail(MBX_ERR_WEIGHTS, path + ": bad safetensors header length");
    const uint8_t* data = buf_.data() + 8 + hlen;
    const size_t data_len = size_t(size) - 8 - size_t(hlen);
    Json j{reinterpret_cast<const char*>(buf_.data() + 8), reinterpret_cast<const char*>(buf_.data() + 8 + hlen)};
    j.expect('{');
    if (j.peek('}')) return;
    for (;;) {
        const std::string name = j.str();
        j.expect(':');
        j.expect('{');
        if (name == "__metadata__") {
            if (!j.peek('}')) {
                for (;;) {
                    const std::string k = j.str();
                    j.expect(':');
                    meta_[k] = j.str();
                    if (j.peek(',')) {
                        ++j.s;
                        continue;
                    }
                    break;
                }
            }
            j.expect('}');
        } else {
            StTensor t;
            std::vector<int64_t> off;
            for (;;) {
                const std::string k = j.str();
                j.expect(':');
                if (k == "dtype")
                    t.dtype = j.str();
                else if (k == "shape")
                    t.shape = j.int_array();
                else if (k == "data_offsets")
                    off = j.int_array();
                else
                    fail(MBX_ERR_WEIGHTS, path + ": unexpected key " + k);
                if (j.peek(',')) {
                    ++j.s;
                    continue;
                }
                break;
            }
            j.expect('}');
            if (off.size() != 2 || off[0] < 0 || off[1] < off[0] || size_t(off[1]) > data_len)
                fail(MBX_ERR_WEIGHTS, path + ": bad data_offsets for " + name);
            t.data = data + off[0];
            t.bytes = size_t(off[1] - off[0]);
            int64_t count = 1;
            for (int64_t d : t.shape) count *= d;
            const size_t esz = t.dtype == "F32" ? 4 : (t.dtype == "F16" ? 2 : 0);
            if (!esz) fail(MBX_ERR_WEIGHTS, path + ": " + name + " has unsupported dtype " + t.dtype);
            if (size_t(count) * esz != t.bytes) fail(MBX_ERR_WEIGHTS, path + ": size mismatch for " + name);
            tensors_[name] = std::move(t);
        }
        if (j.peek(',')) {
            ++j.s;
            continue;
        }
        j.expect('}');
        break;
    }
}

const StTensor* StFile::find(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

std::string StFile::metadata(const std::string& key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? std::string() : it->second;
}

// ---------------------------------------------------------------- Loader

namespace {
std::string shape_str(const std::vector<int64_t>& s) {
    std::string o = "[";
    for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
    return o + "]";
}
}  // namespace

std::vector<int64_t> Loader::shape(const std::string& name) const {
    const StTensor* t = f_->find(key(name));
    if (!t) fail(MBX_ERR_WEIGHTS, "missing tensor " + key(name));
    return t->shape;
}

const StTensor& Loader::raw(const std::string& name, const std::vector<int64_t>& shape) const {
    const StTensor* t = f_->find(key(name));
    if (!t) fail(MBX_ERR_WEIGHTS, "missing tensor " + key(name));
    if (t->shape != shape)
        fail(MBX_ERR_WEIGHTS, key(name) + " has shape " + shape_str(t->shape) + ", expected " + shape_str(shape));
    return *t;
}

std::vector<float> Loader::f32s(const std::string& name, const std::vector<int64_t>& shape) const {
    const StTensor& t = raw(name, shape);
    std::vector<float> out(t.bytes / (t.dtype == "F32" ? 4 : 2));
    if (t.dtype == "F32") {
        std::memcpy(out.data(), t.data, t.bytes);
    } else {
        for (size_t i = 0; i < out.size(); ++i) {
            uint16_t hb;
            std::memcpy(&hb, t.data + 2 * i, 2);
            out[i] = f16_to_f32(hb);
        }
    }
    return out;
}

DevBuf Loader::vec(const std::string& name, int64_t len) const {
    const std::vector<float> v = f32s(name, {len});
    return DevBuf(v.data(), v.size() * 4);
}

Param Loader::param(const std::string& name, int64_t c_out, int64_t taps, int64_t c_in) const {
    const std::vector<int64_t> shape =
        taps == 1 ? std::vector<int64_t>{c_out, c_in} : std::vector<int64_t>{c_out, 3, 3, c_in};
    const StTensor& t = raw(name, shape);
    std::vector<uint8_t> host(t.data, t.data + t.bytes);  // aligned copy
    return Param(ctx_, host.data(), t.dtype == "F16" ? MBX_DTYPE_F16 : MBX_DTYPE_F32, c_out, taps, c_in);
}

Conv Conv::load1x1(const Loader& l, const std::string& name, int64_t c_in, int64_t c_out, bool bias) {
    Conv cv;
    const Loader s = l.sub(name);
    cv.w = s.param("weight", c_out, 1, c_in);
    if (bias) cv.b = s.vec("bias", c_out);
    cv.c_in = c_in;
    cv.c_out = c_out;
    return cv;
}

Conv Conv::load3x3(const Loader& l, const std::string& name, int64_t c_in, int64_t c_out) {
    Conv cv;
    const Loader s = l.sub(name);
    cv.w = s.param("weight", c_out, 9, c_in);
    cv.b = s.vec("bias", c_out);
    cv.c_in = c_in;
    cv.c_out = c_out;
    return cv;
}

GroupNormP GroupNormP::load(const Loader& l, const std::string& name, int64_t c, float eps) {
    if (c % 32 != 0) fail(MBX_ERR_WEIGHTS, l.key(name) + ": channels not divisible by 32 groups");
    GroupNormP g;
    const Loader s = l.sub(name);
    g.gamma = s.vec("weight", c);
    g.beta = s.vec("bias", c);
    g.c = c;
    g.eps = eps;
    return g;
}

// ---------------------------------------------------------------- op helpers

Tensor conv1x1(const Tensor& x, const Conv& cv, const float* residual, const float* pro_scale, const float* pro_shift,
               bool pro_silu, int act) {
    Tensor out(x.ctx(), x.n, x.h, x.w, cv.c_out);
    ck(mbx_conv1x1_fused(x.ctx(), x.data(), x.n, x.h, x.w, x.c, cv.w.get(), cv.b.f(), pro_scale, pro_shift,
                         pro_silu ? 1 : 0, residual, act, out.data()));
    return out;
}

Tensor conv3x3(const Tensor& x, const Conv& cv, const float* pro_scale, const float* pro_shift, bool pro_silu,
               const float* residual) {
    int64_t ho = 0, wo = 0;
    ck(mbx_conv3x3_output_hw(x.h, x.w, cv.stride, cv.pad, cv.up ? 1 : 0, &ho, &wo));
    Tensor out(x.ctx(), x.n, ho, wo, cv.c_out);
    ck(mbx_conv3x3(x.ctx(), x.data(), x.n, x.h, x.w, x.c, cv.w.get(), cv.b.f(), cv.stride, cv.pad, cv.up ? 1 : 0,
                   pro_scale, pro_shift, pro_silu ? 1 : 0, residual, out.data()));
    return out;
}

Tensor conv_gn(const Tensor& x, const Conv& cv, const NextNorm& next, const float* residual, const float* pro_scale,
               const float* pro_shift, bool pro_silu) {
    int64_t ho = x.h, wo = x.w;
    if (cv.w.taps() == 9) ck(mbx_conv3x3_output_hw(x.h, x.w, cv.stride, cv.pad, cv.up ? 1 : 0, &ho, &wo));
    Tensor out(x.ctx(), x.n, ho, wo, cv.c_out);
    *next.scale = Tensor(x.ctx(), x.n, 1, 1, cv.c_out);
    *next.shift = Tensor(x.ctx(), x.n, 1, 1, cv.c_out);
    ck(mbx_conv_group_norm_affine(x.ctx(), x.data(), x.n, x.h, x.w, x.c, cv.w.get(), cv.b.f(), cv.stride, cv.pad,
                                  cv.up ? 1 : 0, pro_scale, pro_shift, pro_silu ? 1 : 0, residual, MBX_ACT_NONE,
                                  out.data(), next.g->groups, next.g->eps, next.g->gamma.f(), next.g->beta.f(),
                                  next.add, next.scale->data(), next.shift->data()));
    return out;
}

void gn_affine(const Tensor& x, const GroupNormP& g, const float* add, Tensor& scale, Tensor& shift) {
    scale = Tensor(x.ctx(), x.n, 1, 1, x.c);
    shift = Tensor(x.ctx(), x.n, 1, 1, x.c);
    ck(mbx_group_norm_affine(x.ctx(), x.data(), x.n, x.h, x.w, x.c, g.groups, g.eps, g.gamma.f(), g.beta.f(), add,
                             scale.data(), shift.data()));
}

}  // namespace eng
}  // namespace mbx
