// The inpainting pipeline (reference src/pipeline.rs, src/scheduler.rs,
// src/preset.rs, src/ffi.rs) for batches of inpaints on one GPU, and the
// engine's C ABI (include/moebius_cuda_engine.h).
//
// Per batch of n inpaints (the reference runs one at a time):
//   prepare (8-bit → model RGB, masks) → VAE encode of [image, masked] × n →
//   starting latents → per DDIM timestep: UNet input, one UNet call at batch 2n
//   (replayed from a CUDA graph captured once per batch size), guidance +
//   DDIM update → VAE decode → Pillow blur of the mask → feathered paste.
// Everything stays on the device between the input copy and the output copy.
#include <cmath>
#include <cstring>
#include <string>

#include "../../include/moebius_cuda_engine.h"
#include "eng_models.h"

namespace mbx {
namespace eng {
namespace {

// ---------------------------------------------------------------- DDIM (src/scheduler.rs:19-98)

constexpr int kTrainSteps = 1000;

std::vector<float> alphas_cumprod() {
    // torch: linspace(√β0, √β1, 1000, f32)² → cumprod(1 − β) in f32; torch's CPU linspace
    // fills the two halves from opposite ends (src/scheduler.rs:155-169).
    const float start = (float)std::sqrt(0.00085), end = (float)std::sqrt(0.012);
    const int n = kTrainSteps;
    const float step = (end - start) / (float)(n - 1);
    std::vector<float> out((size_t)n);
    float acc = 1.0f;
    for (int i = 0; i < n; ++i) {
        const float s = i < n / 2 ? start + step * (float)i : end - step * (float)(n - 1 - i);
        acc *= 1.0f - s * s;
        out[size_t(i)] = acc;
    }
    return out;
}

struct Ddim {
    std::vector<float> ac;
    int step_ratio = 0;
    std::vector<int64_t> timesteps;
    bool pure_noise_start = false;

    Ddim(int steps, double strength, bool trailing) : ac(alphas_cumprod()) {
        MBX_REQUIRE(steps >= 1 && steps <= kTrainSteps, "steps must be 1..=1000");
        step_ratio = kTrainSteps / steps;
        std::vector<int64_t> all;
        for (int i = 0; i < steps; ++i) {
            if (trailing) {
                const double r = (double)kTrainSteps / (double)steps;
                all.push_back((int64_t)std::round((double)kTrainSteps - (double)i * r) - 1);
            } else {
                all.push_back((int64_t)(steps - 1 - i) * step_ratio);
            }
        }
        const int64_t init = std::min<int64_t>((int64_t)((double)steps * strength), steps);
        timesteps.assign(all.begin() + (steps - init), all.end());
        pure_noise_start = strength >= 1.0;
    }
    // {√(1−ᾱ_t), √ᾱ_t, √ᾱ_prev, √(1−ᾱ_prev)} with ᾱ_prev = 1 past the start.
    void step_coef(int64_t t, float coef[4]) const {
        const float a_t = ac[size_t(t)];
        const float a_prev = t >= step_ratio ? ac[size_t(t - step_ratio)] : 1.0f;
        coef[0] = std::sqrt(1.0f - a_t);
        coef[1] = std::sqrt(a_t);
        coef[2] = std::sqrt(a_prev);
        coef[3] = std::sqrt(1.0f - a_prev);
    }
};

// Standard normal samples for the seeded path: SplitMix64 → Box-Muller in f64.
struct Normal {
    uint64_t s;
    bool has = false;
    double spare = 0.0;
    explicit Normal(uint64_t seed) : s(seed) {}
    uint64_t next() {
        uint64_t z = (s += 0x9e3779b97f4a7c15ull);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    }
    double uniform() { return ((double)(next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
    float operator()() {
        if (has) {
            has = false;
            return (float)spare;
        }
        const double r = std::sqrt(-2.0 * std::log(uniform())), th = 6.283185307179586 * uniform();
        spare = r * std::sin(th);
        has = true;
        return (float)(r * std::cos(th));
    }
};

struct ExactParams {
    int steps = 20;
    double strength = 0.99;
    float guidance = 2.5f;
    float noise_offset = 0.0357f;
};

// src/preset.rs:312-338 (Exact) with the caller's overrides (src/ffi.rs).
ExactParams resolve(const mbx_inpaint_params* p) {
    ExactParams e;
    if (!p) return e;
    MBX_REQUIRE(p->preset == MBX_PRESET_EXACT, "only the Exact preset is built in this library");
    MBX_REQUIRE(p->paste == MBX_PASTE_DEFAULT || p->paste == MBX_PASTE_FEATHER,
                "only the Feather paste (the Exact default) is built in this library");
    MBX_REQUIRE(p->mask_dilate == 0, "mask dilation is not built in this library");
    if (p->steps) {
        MBX_REQUIRE(p->steps <= 1000, "steps must be 1..=1000");
        e.steps = (int)p->steps;
    }
    if (p->guidance > 0.0f) e.guidance = p->guidance;
    return e;
}

}  // namespace

// One UNet batch size with its CUDA graph: the input, timestep and output
// buffers and every temporary come from a private pool that lives as long as
// the graph, so nothing the graph touches is ever handed to other work.
struct UNetRunner {
    std::unique_ptr<Pool> pool;
    Tensor x, sin, eps;
    int period = 2;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;  // kernel launches per replay

    ~UNetRunner() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
    }
};

}  // namespace eng
}  // namespace mbx

using namespace mbx;
using namespace mbx::eng;

struct mbx_engine {
    mbx_ctx* ctx = nullptr;
    std::unique_ptr<UNet> unet;
    std::unique_ptr<Vae> vae;
    std::map<std::pair<int64_t, int>, std::unique_ptr<UNetRunner>> runners;
    int64_t vae_chunk = 16;  // items per VAE call (bounds the 512² feature maps)

    ~mbx_engine() {
        runners.clear();
        vae.reset();
        unet.reset();
        if (ctx) mbx_ctx_destroy(ctx);
    }

    int64_t latent() const { return unet->shape().latent; }
    int64_t side() const { return unet->shape().latent * 8; }

    // Temporarily routes the context's allocations to `p`.
    struct PoolSwap {
        mbx_ctx* ctx;
        Pool* saved;
        PoolSwap(mbx_ctx* c, Pool* p) : ctx(c), saved(c->pool) { c->pool = p; }
        ~PoolSwap() { ctx->pool = saved; }
    };

    UNetRunner& runner(int64_t items, int period) {
        auto& slot = runners[{items, period}];
        if (slot) return *slot;
        auto r = std::make_unique<UNetRunner>();
        r->pool = std::make_unique<Pool>(ctx->device);
        r->period = period;
        const int64_t L = latent();
        {
            PoolSwap swap(ctx, r->pool.get());
            r->x = Tensor(ctx, items, L, L, kUnetIn);
            r->sin = Tensor(ctx, items, 1, 1, unet->shape().time_proj);
            r->eps = Tensor(ctx, items, L, L, kUnetOut);
            check_cuda(cudaMemsetAsync(r->x.data(), 0, size_t(r->x.size()) * 4, ctx->stream), "runner init");
            check_cuda(cudaMemsetAsync(r->sin.data(), 0, size_t(r->sin.size()) * 4, ctx->stream), "runner init");
            {  // eager pass: fills the private pool and sets every kernel attribute
                Tensor o = unet->forward(r->x, r->sin.data(), period);
            }
            check_cuda(cudaStreamSynchronize(ctx->stream), "UNet warm-up");
            const uint64_t before = ctx->launches;
            check_cuda(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeRelaxed), "graph capture");
            try {
                Tensor o = unet->forward(r->x, r->sin.data(), period);
                check_cuda(cudaMemcpyAsync(r->eps.data(), o.data(), size_t(o.size()) * 4, cudaMemcpyDeviceToDevice,
                                           ctx->stream),
                           "graph output");
            } catch (...) {
                cudaGraph_t g = nullptr;
                cudaStreamEndCapture(ctx->stream, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            check_cuda(cudaStreamEndCapture(ctx->stream, &r->graph), "graph capture");
            check_cuda(cudaGraphInstantiate(&r->exec, r->graph, 0), "graph instantiate");
            r->kernels = ctx->launches - before;
        }
        slot = std::move(r);
        return *slot;
    }

    void launch(UNetRunner& r) {
        check_cuda(cudaGraphLaunch(r.exec, ctx->stream), "UNet graph launch");
        ctx->launches += r.kernels;
    }

    // Device-buffer batch inpaint (src/pipeline.rs:215-373 for n inpaints at once).
    void inpaint_device(uint8_t* pixels, const uint8_t* masks, int64_t n, int64_t S, int64_t ch,
                        const mbx_inpaint_params* params, const float* noise_vae, const float* noise_init,
                        const float* noise_offset, mbx_progress_fn progress, void* user) {
        const ExactParams ep = resolve(params);
        MBX_REQUIRE(S == side(), "images must be " + std::to_string(side()) + " x " + std::to_string(side()) +
                                     " (the model size; crop-window resampling is not part of this library)");
        MBX_REQUIRE(ch == 3 || ch == 4, "image must be RGB or RGBA");
        if (n == 0) return;
        const int64_t L = latent(), lhw = L * L;
        auto report = [&](uint32_t stage, uint32_t done, uint32_t total) {
            if (!progress) return;
            check_cuda(cudaStreamSynchronize(ctx->stream), "progress");
            if (progress(user, stage, done, total) != 0) fail(MBX_ERR_CANCELLED, "cancelled");
        };

        // Seeded noise when none is given (NoiseSet::sample order: vae_img, vae_masked, init, offset).
        std::vector<float> hv, hi, ho;
        Tensor dv, di, dof;
        if (!noise_vae && !noise_init && !noise_offset) {
            const uint64_t seed = params ? params->seed : 0;
            hv.resize(size_t(2 * n * lhw * 4));
            hi.resize(size_t(n * lhw * 4));
            ho.resize(size_t(n * 4));
            for (int64_t i = 0; i < n; ++i) {
                Normal g(seed + (uint64_t)i);
                for (int part = 0; part < 2; ++part)
                    for (int64_t e = 0; e < lhw * 4; ++e) hv[size_t((2 * i + part) * lhw * 4 + e)] = g();
                for (int64_t e = 0; e < lhw * 4; ++e) hi[size_t(i * lhw * 4 + e)] = g();
                for (int e = 0; e < 4; ++e) ho[size_t(i * 4 + e)] = g();
            }
            dv = Tensor(ctx, 2 * n, L, L, 4);
            di = Tensor(ctx, n, L, L, 4);
            dof = Tensor(ctx, n, 1, 1, 4);
            check_cuda(cudaMemcpyAsync(dv.data(), hv.data(), hv.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
            check_cuda(cudaMemcpyAsync(di.data(), hi.data(), hi.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
            check_cuda(cudaMemcpyAsync(dof.data(), ho.data(), ho.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
            noise_vae = dv.data();
            noise_init = di.data();
            noise_offset = dof.data();
        }
        MBX_REQUIRE(noise_vae && noise_init && noise_offset, "give all three noise tensors or none");

        // 2-5: model inputs and masks (pipeline.rs:234-252).
        report(0, 0, 1);
        Tensor images(ctx, 2 * n, S, S, 3);
        PoolBuf bin(ctx, size_t(n * S * S)), flags(ctx, size_t(n) * 4);
        Tensor mask_lat(ctx, n, L, L, 1);
        ck(mbx_inpaint_prepare(ctx, pixels, masks, n, S, S, ch, images.data(), bin.as<uint8_t>(), mask_lat.data(),
                               flags.as<int32_t>()));
        // 4: VAE encode of [image, masked] per inpaint (pipeline.rs:276-289).
        Tensor z(ctx, 2 * n, L, L, 4);
        for (int64_t b0 = 0; b0 < 2 * n; b0 += vae_chunk) {
            const int64_t b = std::min(vae_chunk, 2 * n - b0);
            Tensor zi = vae->encode(Tensor::view(ctx, images.item(b0), b, S, S, 3), noise_vae + b0 * lhw * 4);
            check_cuda(cudaMemcpyAsync(z.item(b0), zi.data(), size_t(zi.size()) * 4, cudaMemcpyDeviceToDevice,
                                       ctx->stream),
                       "latents");
        }
        images = Tensor();
        report(0, 1, 1);

        // 6-7: starting latents.
        const Ddim ddim(ep.steps, ep.strength, false);
        const std::vector<int64_t>& ts = ddim.timesteps;
        Tensor x(ctx, n, L, L, 4);
        {
            const float a0 = ddim.ac[size_t(ts.empty() ? 0 : ts[0])];
            ck(mbx_latents_init(ctx, z.data(), noise_init, noise_offset, n, lhw, ep.noise_offset, std::sqrt(a0),
                                std::sqrt(1.0f - a0), ddim.pure_noise_start ? 1 : 0, x.data()));
        }

        // 8: denoise (pipeline.rs:313-345), CFG at batch 2n.
        if (!ts.empty()) {
            UNetRunner& r = runner(2 * n, 2);
            const int64_t tp = unet->shape().time_proj;
            float* host_sin = nullptr;
            check_cuda(cudaHostAlloc((void**)&host_sin, ts.size() * size_t(2 * n * tp) * 4, cudaHostAllocDefault),
                       "timestep table");
            struct HostFree {
                float* p;
                mbx_ctx* ctx;
                ~HostFree() {
                    cudaStreamSynchronize(ctx->stream);
                    cudaFreeHost(p);
                }
            } host_free{host_sin, ctx};
            std::vector<float> one((size_t)tp);
            for (size_t i = 0; i < ts.size(); ++i) {
                unet->sinusoid(ts[i], one.data());
                for (int64_t it = 0; it < 2 * n; ++it)
                    std::memcpy(host_sin + (i * size_t(2 * n) + size_t(it)) * size_t(tp), one.data(), size_t(tp) * 4);
            }
            for (size_t i = 0; i < ts.size(); ++i) {
                check_cuda(cudaMemcpyAsync(r.sin.data(), host_sin + i * size_t(2 * n * tp), size_t(2 * n * tp) * 4,
                                           cudaMemcpyHostToDevice, ctx->stream),
                           "timestep embedding");
                ck(mbx_unet_input(ctx, x.data(), mask_lat.data(), z.data(), n, lhw, 2, r.x.data()));
                launch(r);
                float coef[4];
                ddim.step_coef(ts[i], coef);
                ck(mbx_cfg_ddim_step(ctx, r.eps.data(), n, lhw, 2, ep.guidance, coef, x.data()));
                report(1, (uint32_t)(i + 1), (uint32_t)ts.size());
            }
        }
        z = Tensor();
        mask_lat = Tensor();

        // 9: decode; 10: 8-bit result and feathered paste (pipeline.rs:355-372, blend.rs:174-215).
        report(2, 0, 1);
        Tensor dec(ctx, n, S, S, 3);
        for (int64_t b0 = 0; b0 < n; b0 += vae_chunk) {
            const int64_t b = std::min(vae_chunk, n - b0);
            Tensor di2 = vae->decode(Tensor::view(ctx, x.item(b0), b, L, L, 4));
            check_cuda(cudaMemcpyAsync(dec.item(b0), di2.data(), size_t(di2.size()) * 4, cudaMemcpyDeviceToDevice,
                                       ctx->stream),
                       "decoded images");
        }
        report(2, 1, 1);
        PoolBuf blurred(ctx, size_t(n * S * S)), scratch(ctx, size_t(n * S * S));
        ck(mbx_gaussian_blur_u8(ctx, bin.as<uint8_t>(), n, S, S, 3.0f, scratch.as<uint8_t>(), blurred.as<uint8_t>()));
        ck(mbx_feather_paste(ctx, dec.data(), blurred.as<uint8_t>(), pixels, n, S, S, ch, flags.as<int32_t>()));
    }

    void inpaint_host(uint8_t* pixels, const uint8_t* masks, int64_t n, int64_t S, int64_t ch,
                      const mbx_inpaint_params* params, const float* nv, const float* ni, const float* no,
                      mbx_progress_fn progress, void* user) {
        const int64_t L = latent();
        PoolBuf dp(ctx, size_t(n * S * S * ch)), dm(ctx, size_t(n * S * S));
        check_cuda(cudaMemcpyAsync(dp.p, pixels, size_t(n * S * S * ch), cudaMemcpyHostToDevice, ctx->stream), "pixels");
        check_cuda(cudaMemcpyAsync(dm.p, masks, size_t(n * S * S), cudaMemcpyHostToDevice, ctx->stream), "masks");
        Tensor dv, di, dof;
        if (nv || ni || no) {
            MBX_REQUIRE(nv && ni && no, "give all three noise tensors or none");
            dv = Tensor(ctx, 2 * n, L, L, 4);
            di = Tensor(ctx, n, L, L, 4);
            dof = Tensor(ctx, n, 1, 1, 4);
            check_cuda(cudaMemcpyAsync(dv.data(), nv, size_t(dv.size()) * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
            check_cuda(cudaMemcpyAsync(di.data(), ni, size_t(di.size()) * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
            check_cuda(cudaMemcpyAsync(dof.data(), no, size_t(dof.size()) * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
        }
        inpaint_device(dp.as<uint8_t>(), dm.as<uint8_t>(), n, S, ch, params, dv ? dv.data() : nullptr,
                       di ? di.data() : nullptr, dof ? dof.data() : nullptr, progress, user);
        check_cuda(cudaMemcpyAsync(pixels, dp.p, size_t(n * S * S * ch), cudaMemcpyDeviceToHost, ctx->stream), "pixels");
        check_cuda(cudaStreamSynchronize(ctx->stream), "inpaint");
    }
};

namespace {

template <class F>
int32_t eguard(F&& f) {
    try {
        f();
        return MBX_OK;
    } catch (const mbx::Error& e) {
        mbx::record_error(e.code, e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        mbx::record_error(MBX_ERR_OUT_OF_MEMORY, "host allocation failed");
        return MBX_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        mbx::record_error(MBX_ERR_INTERNAL, (std::string("internal error: ") + e.what()).c_str());
        return MBX_ERR_INTERNAL;
    } catch (...) {
        mbx::record_error(MBX_ERR_INTERNAL, "internal error");
        return MBX_ERR_INTERNAL;
    }
}

void require_engine(const mbx_engine* e) { MBX_REQUIRE(e != nullptr && e->ctx != nullptr, "null engine"); }

void use(const mbx_engine* e) { check_cuda(cudaSetDevice(e->ctx->device), "cudaSetDevice"); }

}  // namespace

extern "C" {

int32_t mbx_engine_create(const char* weights_dir, int32_t device, mbx_engine** out) {
    return eguard([&] {
        MBX_REQUIRE(weights_dir != nullptr && out != nullptr, "null argument");
        *out = nullptr;
        auto e = std::make_unique<mbx_engine>();
        ck(mbx_ctx_create(device, &e->ctx));
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
        const std::string dir(weights_dir);
        {
            const StFile uf(dir + "/unet.safetensors");
            e->unet = std::make_unique<UNet>(e->ctx, uf);
        }
        {
            const StFile vf(dir + "/vae.safetensors");
            e->vae = std::make_unique<Vae>(e->ctx, vf);
        }
        check_cuda(cudaStreamSynchronize(e->ctx->stream), "engine load");
        *out = e.release();
    });
}

void mbx_engine_destroy(mbx_engine* engine) {
    if (!engine) return;
    cudaSetDevice(engine->ctx ? engine->ctx->device : 0);
    if (engine->ctx) cudaStreamSynchronize(engine->ctx->stream);
    delete engine;
}

int32_t mbx_engine_set_stream(mbx_engine* engine, void* stream) {
    return eguard([&] {
        require_engine(engine);
        // Graphs were captured on the old stream; they replay on any stream, but their
        // private pools assume stream order, so the old stream is drained first.
        check_cuda(cudaStreamSynchronize(engine->ctx->stream), "cudaStreamSynchronize");
        ck(mbx_ctx_set_stream(engine->ctx, stream));
    });
}

uint64_t mbx_engine_launch_count(const mbx_engine* engine) { return engine && engine->ctx ? engine->ctx->launches : 0; }

int32_t mbx_engine_info(const mbx_engine* engine, int64_t* latent_side, int64_t* image_side, int64_t widths[3]) {
    return eguard([&] {
        require_engine(engine);
        if (latent_side) *latent_side = engine->latent();
        if (image_side) *image_side = engine->side();
        if (widths)
            for (int i = 0; i < 3; ++i) widths[i] = engine->unet->shape().ch[i];
    });
}

int32_t mbx_inpaint(mbx_engine* engine, uint8_t* pixels, uint32_t width, uint32_t height, uint32_t stride,
                    uint32_t channels, const uint8_t* mask, uint32_t mask_stride, const mbx_inpaint_params* params,
                    mbx_progress_fn progress, void* user, mbx_rect* changed) {
    return eguard([&] {
        require_engine(engine);
        if (changed) *changed = mbx_rect{0, 0, 0, 0};
        MBX_REQUIRE(pixels != nullptr && mask != nullptr, "null argument");
        MBX_REQUIRE(channels == 3 || channels == 4, "image must be RGB or RGBA");
        MBX_REQUIRE(width > 0 && height > 0, "empty image");
        MBX_REQUIRE(stride >= width * channels && mask_stride >= width,
                    "buffer smaller than width, height and stride imply");
        (void)resolve(params);
        use(engine);
        const int64_t S = engine->side();
        MBX_REQUIRE(width == S && height == S, "image must be " + std::to_string(S) + " x " + std::to_string(S) +
                                                   " (the model size; crop-window resampling is not part of this library)");
        // Tightly packed copies; an empty mask changes nothing (src/pipeline.rs:202-204).
        std::vector<uint8_t> px(size_t(S * S * channels)), mk(size_t(S * S));
        bool any = false;
        for (int64_t y = 0; y < S; ++y) {
            std::memcpy(px.data() + y * S * channels, pixels + y * stride, size_t(S * channels));
            std::memcpy(mk.data() + y * S, mask + y * mask_stride, size_t(S));
            for (int64_t x = 0; x < S && !any; ++x) any = mk[size_t(y * S + x)] >= 128;
        }
        if (!any) return;
        engine->inpaint_host(px.data(), mk.data(), 1, S, channels, params, nullptr, nullptr, nullptr, progress, user);
        for (int64_t y = 0; y < S; ++y) std::memcpy(pixels + y * stride, px.data() + y * S * channels, size_t(S * channels));
        if (changed) *changed = mbx_rect{0, 0, (uint32_t)S, (uint32_t)S};
    });
}

int32_t mbx_inpaint_batch(mbx_engine* engine, uint8_t* pixels, const uint8_t* masks, int64_t n, uint32_t side,
                          uint32_t channels, const mbx_inpaint_params* params, const float* noise_vae,
                          const float* noise_init, const float* noise_offset, int32_t device_buffers,
                          mbx_progress_fn progress, void* user) {
    return eguard([&] {
        require_engine(engine);
        MBX_REQUIRE(n >= 0, "negative batch");
        if (n == 0) return;
        MBX_REQUIRE(pixels != nullptr && masks != nullptr, "null argument");
        use(engine);
        if (device_buffers)
            engine->inpaint_device(pixels, masks, n, side, channels, params, noise_vae, noise_init, noise_offset,
                                   progress, user);
        else
            engine->inpaint_host(pixels, masks, n, side, channels, params, noise_vae, noise_init, noise_offset,
                                 progress, user);
    });
}

int32_t mbx_engine_unet_forward(mbx_engine* engine, const float* x, int64_t items, int64_t timestep, int32_t cfg,
                                float* eps) {
    return eguard([&] {
        require_engine(engine);
        MBX_REQUIRE(items >= 0, "negative batch");
        MBX_REQUIRE(timestep >= 0 && timestep < kTrainSteps, "timestep must be 0..1000");
        if (items == 0) return;
        MBX_REQUIRE(x != nullptr && eps != nullptr, "null argument");
        use(engine);
        mbx_ctx* ctx = engine->ctx;
        const int64_t L = engine->latent(), tp = engine->unet->shape().time_proj;
        std::vector<float> one((size_t)tp), all((size_t)(items * tp));
        engine->unet->sinusoid(timestep, one.data());
        for (int64_t i = 0; i < items; ++i) std::memcpy(all.data() + i * tp, one.data(), size_t(tp) * 4);
        Tensor sin(ctx, items, 1, 1, tp);
        check_cuda(cudaMemcpyAsync(sin.data(), all.data(), all.size() * 4, cudaMemcpyHostToDevice, ctx->stream),
                   "timestep embedding");
        Tensor o = engine->unet->forward(Tensor::view(ctx, const_cast<float*>(x), items, L, L, kUnetIn), sin.data(),
                                         cfg ? 2 : 1);
        check_cuda(cudaMemcpyAsync(eps, o.data(), size_t(o.size()) * 4, cudaMemcpyDeviceToDevice, ctx->stream), "eps");
        check_cuda(cudaStreamSynchronize(ctx->stream), "unet");
    });
}

int32_t mbx_engine_vae_encode(mbx_engine* engine, const float* images, const float* noise, int64_t b, int64_t h,
                              int64_t w, float* z) {
    return eguard([&] {
        require_engine(engine);
        MBX_REQUIRE(b >= 0 && h > 0 && w > 0 && h % 8 == 0 && w % 8 == 0, "bad shape");
        if (b == 0) return;
        MBX_REQUIRE(images && noise && z, "null argument");
        use(engine);
        mbx_ctx* ctx = engine->ctx;
        Tensor o = engine->vae->encode(Tensor::view(ctx, const_cast<float*>(images), b, h, w, 3), noise);
        check_cuda(cudaMemcpyAsync(z, o.data(), size_t(o.size()) * 4, cudaMemcpyDeviceToDevice, ctx->stream), "z");
    });
}

int32_t mbx_engine_vae_decode(mbx_engine* engine, const float* latents, int64_t b, int64_t h, int64_t w,
                              float* out) {
    return eguard([&] {
        require_engine(engine);
        MBX_REQUIRE(b >= 0 && h > 0 && w > 0, "bad shape");
        if (b == 0) return;
        MBX_REQUIRE(latents && out, "null argument");
        use(engine);
        mbx_ctx* ctx = engine->ctx;
        Tensor o = engine->vae->decode(Tensor::view(ctx, const_cast<float*>(latents), b, h, w, 4));
        check_cuda(cudaMemcpyAsync(out, o.data(), size_t(o.size()) * 4, cudaMemcpyDeviceToDevice, ctx->stream), "out");
    });
}

int32_t mbx_ddim_timesteps(uint32_t steps, double strength, int32_t trailing, int64_t* out, int64_t* count) {
    return eguard([&] {
        MBX_REQUIRE(out != nullptr && count != nullptr, "null argument");
        const Ddim d((int)steps, strength, trailing != 0);
        for (size_t i = 0; i < d.timesteps.size(); ++i) out[i] = d.timesteps[i];
        *count = (int64_t)d.timesteps.size();
    });
}

int32_t mbx_ddim_alphas_cumprod(float* out) {
    return eguard([&] {
        MBX_REQUIRE(out != nullptr, "null argument");
        const std::vector<float> a = alphas_cumprod();
        std::memcpy(out, a.data(), a.size() * 4);
    });
}

}  // extern "C"
