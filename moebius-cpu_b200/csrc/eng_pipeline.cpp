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
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
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

// Resolved inpaint parameters (reference InpaintParams, src/preset.rs:32-83).
struct Params {
    int steps = 20;
    double strength = 0.99;
    bool trailing = false;
    bool dpm = false;         // Solver::DpmPp2M (else Ddim)
    float guidance = 2.5f;
    float noise_offset = 0.0357f;
    uint64_t seed = 0;
    int cfg_steps = -1;       // CFG for the first cfg_steps steps only (-1: every step)
    bool roi_encode = false;
    uint32_t paste = MBX_PASTE_FEATHER;
    uint32_t mask_dilate = 0;
};

// Preset defaults with the caller's overrides (src/preset.rs:55-83, src/ffi.rs:248-271).
Params resolve(const mbx_inpaint_params* p) {
    Params e;
    if (!p) return e;
    if (p->preset == MBX_PRESET_FAST) {  // Preset::Fast: 10 trailing DPM++(2M) steps, CFG for 3, ROI encode
        e.steps = 10;
        e.trailing = true;
        e.dpm = true;
        e.cfg_steps = 3;
        e.roi_encode = true;
    } else {
        MBX_REQUIRE(p->preset == MBX_PRESET_EXACT, "unknown preset " + std::to_string(p->preset));
    }
    if (p->steps) {
        MBX_REQUIRE(p->steps <= 1000, "steps must be 1..=1000, got " + std::to_string(p->steps));
        e.steps = (int)p->steps;
    }
    if (p->guidance > 0.0f) e.guidance = p->guidance;
    e.seed = p->seed;
    e.mask_dilate = p->mask_dilate;
    switch (p->paste) {
        case MBX_PASTE_DEFAULT:
            break;
        case MBX_PASTE_NONE:
        case MBX_PASTE_FEATHER:
        case MBX_PASTE_FEATHER_COMPENSATE:
            e.paste = p->paste;
            break;
        default:
            fail(MBX_ERR_INVALID_ARGUMENT, "unknown paste mode " + std::to_string(p->paste));
    }
    return e;
}

// (α_t, σ_t, λ_t = ln α_t − ln σ_t) in f64 (src/scheduler.rs:100-105).
void dpm_abl(const Ddim& d, int64_t t, double& alpha, double& sigma, double& lambda) {
    const double a = (double)d.ac[size_t(t)];
    alpha = std::sqrt(a);
    sigma = std::sqrt(1.0 - a);
    lambda = std::log(alpha) - std::log(sigma);
}

// Coefficients of DPM-Solver++(2M) step i (Dpm2M::step, src/scheduler.rs:121-151) given whether the
// solver holds the previous step's data prediction (and its λ): coef = {σ, 1/α, σ_n/σ, φ or c0, c1}.
void dpm_step_coef(const Ddim& d, size_t i, bool has_prev, double lambda_prev, float coef[5], int* order) {
    const std::vector<int64_t>& ts = d.timesteps;
    double alpha, sigma, lambda;
    dpm_abl(d, ts[i], alpha, sigma, lambda);
    coef[0] = (float)sigma;
    coef[1] = (float)(1.0 / alpha);
    coef[2] = coef[3] = coef[4] = 0.0f;
    if (i + 1 >= ts.size()) {
        *order = 0;
        return;
    }
    double an, sn, ln;
    dpm_abl(d, ts[i + 1], an, sn, ln);
    const double h = ln - lambda;
    coef[2] = (float)(sn / sigma);
    const double phi = an * (1.0 - std::exp(-h));
    if (!has_prev) {
        *order = 1;
        coef[3] = (float)phi;
    } else {
        const double r = (lambda - lambda_prev) / h;
        *order = 2;
        coef[3] = (float)(phi * (1.0 + 0.5 / r));
        coef[4] = (float)(phi * 0.5 / r);
    }
}

// The latent bbox of mask_lat > 0.5 grown by `margin` and clamped (src/vae/mod.rs:64-78).
struct LatRect {
    int64_t x = 0, y = 0, w = 0, h = 0;
    bool empty = true;
};

LatRect roi_window(const float* m, int64_t L, int64_t margin) {
    int64_t x0 = L, y0 = L, x1 = -1, y1 = -1;
    for (int64_t i = 0; i < L * L; ++i)
        if (m[i] > 0.5f) {
            const int64_t y = i / L, x = i % L;
            x0 = std::min(x0, x);
            y0 = std::min(y0, y);
            x1 = std::max(x1, x);
            y1 = std::max(y1, y);
        }
    LatRect r;
    if (x1 < 0) return r;
    x0 = std::max<int64_t>(x0 - margin, 0);
    y0 = std::max<int64_t>(y0 - margin, 0);
    x1 = std::min(x1 + margin, L - 1);
    y1 = std::min(y1 + margin, L - 1);
    r.x = x0;
    r.y = y0;
    r.w = x1 - x0 + 1;
    r.h = y1 - y0 + 1;
    r.empty = false;
    return r;
}

constexpr int64_t kRoiMargin = 8;  // src/vae/mod.rs:60

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
    DevBuf sin_table;        // [1000][time_proj]: the timestep embedding of every train step

    // The embeddings on the device, built on first use, so a denoising loop copies them on the
    // device and never waits for the host.
    const float* sinusoids() {
        if (!sin_table.get()) {
            const int64_t tp = unet->shape().time_proj;
            std::vector<float> h(size_t(kTrainSteps * tp));
            for (int64_t t = 0; t < kTrainSteps; ++t) unet->sinusoid(t, h.data() + t * tp);
            sin_table = DevBuf(h.data(), h.size() * 4);
        }
        return sin_table.f();
    }

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

    using Report = std::function<void(uint32_t, uint32_t, uint32_t)>;

    Report reporter(mbx_progress_fn progress, void* user) {
        return [this, progress, user](uint32_t stage, uint32_t done, uint32_t total) {
            if (!progress) return;
            check_cuda(cudaStreamSynchronize(ctx->stream), "progress");
            if (progress(user, stage, done, total) != 0) fail(MBX_ERR_CANCELLED, "cancelled");
        };
    }

    // The caller's noise, or seeded noise (NoiseSet::sample order per inpaint: vae_img,
    // vae_masked, init, offset; inpaint i uses seed + i) uploaded into `keep`.
    struct Noise {
        Tensor v, i, o;
        const float* vae = nullptr;
        const float* init = nullptr;
        const float* offset = nullptr;
    };

    Noise noise_for(int64_t n, uint64_t seed, const float* nv, const float* ni, const float* no) {
        Noise z;
        if (nv || ni || no) {
            MBX_REQUIRE(nv && ni && no, "give all three noise tensors or none");
            z.vae = nv;
            z.init = ni;
            z.offset = no;
            return z;
        }
        const int64_t lhw = latent() * latent();
        std::vector<float> hv(size_t(2 * n * lhw * 4)), hi(size_t(n * lhw * 4)), ho(size_t(n * 4));
        for (int64_t i = 0; i < n; ++i) {
            Normal g(seed + (uint64_t)i);
            for (int part = 0; part < 2; ++part)
                for (int64_t e = 0; e < lhw * 4; ++e) hv[size_t((2 * i + part) * lhw * 4 + e)] = g();
            for (int64_t e = 0; e < lhw * 4; ++e) hi[size_t(i * lhw * 4 + e)] = g();
            for (int e = 0; e < 4; ++e) ho[size_t(i * 4 + e)] = g();
        }
        const int64_t L = latent();
        z.v = Tensor(ctx, 2 * n, L, L, 4);
        z.i = Tensor(ctx, n, L, L, 4);
        z.o = Tensor(ctx, n, 1, 1, 4);
        // Pageable sources: each copy has read its host buffer when the call returns.
        check_cuda(cudaMemcpyAsync(z.v.data(), hv.data(), hv.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
        check_cuda(cudaMemcpyAsync(z.i.data(), hi.data(), hi.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
        check_cuda(cudaMemcpyAsync(z.o.data(), ho.data(), ho.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "noise");
        z.vae = z.v.data();
        z.init = z.i.data();
        z.offset = z.o.data();
        return z;
    }

    // 4: VAE encode into z [2n] = (z_img, z_masked) per inpaint (pipeline.rs:255-289). images holds
    // [image_0, masked_0, image_1, ...]. ROI encode: z_masked from the masked image alone and z_img =
    // z_masked with the latents near the mask replaced by an encode of the image window around it.
    void encode(const Tensor& images, const float* noise_vae, const Tensor& mask_lat, int64_t n, bool roi,
                Tensor& z) {
        const int64_t S = side(), L = latent(), lhw = L * L;
        auto put = [&](const Tensor& t, int64_t item) {
            check_cuda(cudaMemcpyAsync(z.item(item), t.data(), size_t(t.size()) * 4, cudaMemcpyDeviceToDevice,
                                       ctx->stream),
                       "latents");
        };
        if (!roi) {
            for (int64_t b0 = 0; b0 < 2 * n; b0 += vae_chunk) {
                const int64_t b = std::min(vae_chunk, 2 * n - b0);
                put(vae->encode(Tensor::view(ctx, images.item(b0), b, S, S, 3), noise_vae + b0 * lhw * 4), b0);
            }
            return;
        }
        std::vector<float> ml(size_t(n * lhw));
        check_cuda(cudaMemcpyAsync(ml.data(), mask_lat.data(), ml.size() * 4, cudaMemcpyDeviceToHost, ctx->stream),
                   "latent masks");
        check_cuda(cudaStreamSynchronize(ctx->stream), "latent masks");
        for (int64_t i = 0; i < n; ++i) {
            const float* mi = ml.data() + i * lhw;
            const LatRect r = roi_window(mi, L, kRoiMargin);
            if (r.empty || (r.w == L && r.h == L)) {  // no window: both images whole
                put(vae->encode(Tensor::view(ctx, images.item(2 * i), 2, S, S, 3), noise_vae + 2 * i * lhw * 4),
                    2 * i);
                continue;
            }
            {
                Tensor zm = vae->encode(Tensor::view(ctx, images.item(2 * i + 1), 1, S, S, 3),
                                        noise_vae + (2 * i + 1) * lhw * 4);
                put(zm, 2 * i + 1);
                put(zm, 2 * i);
            }
            Tensor crop(ctx, 1, 8 * r.h, 8 * r.w, 3), cn(ctx, 1, r.h, r.w, 4);
            check_cuda(cudaMemcpy2DAsync(crop.data(), size_t(8 * r.w * 3) * 4,
                                         images.item(2 * i) + (8 * r.y * S + 8 * r.x) * 3, size_t(S * 3) * 4,
                                         size_t(8 * r.w * 3) * 4, size_t(8 * r.h), cudaMemcpyDeviceToDevice,
                                         ctx->stream),
                       "ROI crop");
            check_cuda(cudaMemcpy2DAsync(cn.data(), size_t(r.w * 4) * 4, noise_vae + (2 * i * lhw + r.y * L + r.x) * 4,
                                         size_t(L * 4) * 4, size_t(r.w * 4) * 4, size_t(r.h), cudaMemcpyDeviceToDevice,
                                         ctx->stream),
                       "ROI noise");
            Tensor part = vae->encode(crop, cn.data());
            // The window's border latents see zero padding: only the part nearer the mask is kept.
            const LatRect in = roi_window(mi, L, kRoiMargin / 2);
            check_cuda(cudaMemcpy2DAsync(z.item(2 * i) + (in.y * L + in.x) * 4, size_t(L * 4) * 4,
                                         part.data() + ((in.y - r.y) * r.w + (in.x - r.x)) * 4, size_t(r.w * 4) * 4,
                                         size_t(in.w * 4) * 4, size_t(in.h), cudaMemcpyDeviceToDevice, ctx->stream),
                       "ROI latents");
        }
    }

    // Steps 2-9 for n model-size inputs on the device: images8 [n][S][S][ch], masks [n][S][S]
    // (>= 128 inpaints). Returns the decoded images [n][S][S][3] in [0, 1]; flags[i] = 1 when
    // mask i has a masked pixel. src/pipeline.rs:215-366 for n inpaints at once.
    Tensor run_model(const uint8_t* images8, int64_t ch, const uint8_t* masks, int64_t n, const Params& ep,
                     const Noise& noise, int32_t* flags, const Report& report) {
        const int64_t S = side(), L = latent(), lhw = L * L;
        // 2-5: model inputs and masks (pipeline.rs:234-252).
        report(0, 0, 1);
        Tensor images(ctx, 2 * n, S, S, 3);
        Tensor mask_lat(ctx, n, L, L, 1);
        {
            PoolBuf bin(ctx, size_t(n * S * S));
            ck(mbx_inpaint_prepare(ctx, images8, masks, n, S, S, ch, images.data(), bin.as<uint8_t>(),
                                   mask_lat.data(), flags));
        }
        Tensor z(ctx, 2 * n, L, L, 4);
        encode(images, noise.vae, mask_lat, n, ep.roi_encode, z);
        images = Tensor();
        report(0, 1, 1);

        // 6-7: starting latents.
        const Ddim ddim(ep.steps, ep.strength, ep.trailing);
        const std::vector<int64_t>& ts = ddim.timesteps;
        Tensor x(ctx, n, L, L, 4);
        {
            const float a0 = ddim.ac[size_t(ts.empty() ? 0 : ts[0])];
            ck(mbx_latents_init(ctx, z.data(), noise.init, noise.offset, n, lhw, ep.noise_offset, std::sqrt(a0),
                                std::sqrt(1.0f - a0), ddim.pure_noise_start ? 1 : 0, x.data()));
        }

        // 8: denoise (pipeline.rs:313-346): CFG at batch 2n for the first cfg_steps steps (all of
        // them by default), conditional-only at batch n after; DDIM or DPM-Solver++(2M).
        if (!ts.empty()) {
            const int64_t tp = unet->shape().time_proj;
            const float* table = sinusoids();
            Tensor x0_prev;
            if (ep.dpm) x0_prev = Tensor(ctx, n, L, L, 4);
            bool has_prev = false;
            double lambda_prev = 0.0;
            for (size_t i = 0; i < ts.size(); ++i) {
                const bool cfg = ep.cfg_steps < 0 || (int64_t)i < ep.cfg_steps;
                const int copies = cfg ? 2 : 1;
                UNetRunner& r = runner(copies * n, copies);
                launch_broadcast_rows(ctx, table + ts[i] * tp, tp, copies * n, r.sin.data());
                ck(mbx_unet_input(ctx, x.data(), mask_lat.data(), z.data(), n, lhw, copies, r.x.data()));
                launch(r);
                if (!ep.dpm) {
                    float coef[4];
                    ddim.step_coef(ts[i], coef);
                    ck(mbx_cfg_ddim_step(ctx, r.eps.data(), n, lhw, copies, ep.guidance, coef, x.data()));
                } else {
                    if (ep.cfg_steps == (int64_t)i) has_prev = false;  // guidance switched off: restart
                    float coef[5];
                    int order = 0;
                    dpm_step_coef(ddim, i, has_prev, lambda_prev, coef, &order);
                    ck(mbx_cfg_dpm_step(ctx, r.eps.data(), n, lhw, copies, ep.guidance, coef, order, x.data(),
                                        x0_prev.data()));
                    double a, sg;
                    dpm_abl(ddim, ts[i], a, sg, lambda_prev);
                    has_prev = true;
                }
                report(1, (uint32_t)(i + 1), (uint32_t)ts.size());
            }
        }
        z = Tensor();
        mask_lat = Tensor();

        // 9: decode (pipeline.rs:355-366).
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
        return dec;
    }

    // Device-buffer batch inpaint of model-size images, each used whole (src/pipeline.rs:163-373
    // for n inpaints at once; a model-size window is its own source rectangle, crop.rs:11-14).
    void inpaint_device(uint8_t* pixels, const uint8_t* masks, int64_t n, int64_t S, int64_t ch,
                        const mbx_inpaint_params* params, const float* noise_vae, const float* noise_init,
                        const float* noise_offset, mbx_progress_fn progress, void* user) {
        const Params ep = resolve(params);
        MBX_REQUIRE(S == side(), "images must be " + std::to_string(side()) + " x " + std::to_string(side()) +
                                     " (the model size) in the batch call; mbx_inpaint takes any size");
        MBX_REQUIRE(ch == 3 || ch == 4, "image must be RGB or RGBA");
        if (n == 0) return;
        const Noise noise = noise_for(n, ep.seed, noise_vae, noise_init, noise_offset);
        const uint8_t* m = masks;
        PoolBuf dilated;
        if (ep.mask_dilate > 0) {  // pipeline.rs:191-197
            dilated = PoolBuf(ctx, size_t(n * S * S));
            PoolBuf scratch(ctx, size_t(n * S * S));
            ck(mbx_mask_dilate(ctx, masks, n, S, S, S, ep.mask_dilate, scratch.as<uint8_t>(), dilated.as<uint8_t>()));
            m = dilated.as<uint8_t>();
        }
        PoolBuf flags(ctx, size_t(n) * 4);
        Tensor dec = run_model(pixels, ch, m, n, ep, noise, flags.as<int32_t>(), reporter(progress, user));
        // 10: 8-bit result and the paste; an empty mask leaves its image untouched (pipeline.rs:198-200).
        PoolBuf res(ctx, size_t(n * S * S * 3));
        ck(mbx_model_to_window(ctx, dec.data(), n, S, S, res.as<uint8_t>()));
        dec = Tensor();
        ck(mbx_paste(ctx, pixels, n, S * ch, ch, m, S, 0, 0, S, S, S, S, 0, 0, S, res.as<uint8_t>(), ep.paste,
                     flags.as<int32_t>()));
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

    // One host image of any size (src/pipeline.rs:163-213): dilation, bbox, square crop window,
    // Lanczos3 to the model size, the model, Lanczos3 back, paste. Only the source rectangle plus
    // the blur margin travels to the device and only the source rectangle comes back; nothing is
    // written before the last cancellation point. Returns the changed rectangle.
    mbx_rect inpaint_any(uint8_t* pixels, int64_t w, int64_t h, int64_t stride, int64_t ch, const uint8_t* mask,
                         int64_t mask_stride, const mbx_inpaint_params* params, const float* nv, const float* ni,
                         const float* no, mbx_progress_fn progress, void* user) {
        const Params ep = resolve(params);
        const int64_t S = side();
        PoolBuf dm(ctx, size_t(w * h));
        check_cuda(cudaMemcpy2DAsync(dm.p, size_t(w), mask, size_t(mask_stride), size_t(w), size_t(h),
                                     cudaMemcpyHostToDevice, ctx->stream),
                   "mask");
        const uint8_t* m = dm.as<uint8_t>();
        PoolBuf dilated;
        if (ep.mask_dilate > 0) {
            dilated = PoolBuf(ctx, size_t(w * h));
            PoolBuf scratch(ctx, size_t(w * h));
            ck(mbx_mask_dilate(ctx, m, 1, h, w, w, ep.mask_dilate, scratch.as<uint8_t>(), dilated.as<uint8_t>()));
            m = dilated.as<uint8_t>();
        }
        int32_t hb[4];
        {
            PoolBuf box(ctx, 16);
            ck(mbx_mask_bbox(ctx, m, 1, h, w, w, box.as<int32_t>()));
            check_cuda(cudaMemcpyAsync(hb, box.p, 16, cudaMemcpyDeviceToHost, ctx->stream), "bbox");
            check_cuda(cudaStreamSynchronize(ctx->stream), "bbox");
        }
        if (hb[2] < 0) return mbx_rect{0, 0, 0, 0};  // empty mask: nothing to do (pipeline.rs:198-200)
        const CropWindow c = crop_window(hb[0], hb[1], hb[2] - hb[0] + 1, hb[3] - hb[1] + 1, w, h, S);
        const mbx_rect src = source_rect(c, w, h);
        const int64_t margin = 16;  // the paste's blur margin (blend.rs:102)
        const int64_t rx0 = std::max<int64_t>(src.x - margin, 0), ry0 = std::max<int64_t>(src.y - margin, 0);
        const int64_t rx1 = std::min<int64_t>(src.x + src.width + margin, w);
        const int64_t ry1 = std::min<int64_t>(src.y + src.height + margin, h);
        const int64_t rw = rx1 - rx0, rh = ry1 - ry0;
        PoolBuf img(ctx, size_t(rw * rh * ch));
        check_cuda(cudaMemcpy2DAsync(img.p, size_t(rw * ch), pixels + ry0 * stride + rx0 * ch, size_t(stride),
                                     size_t(rw * ch), size_t(rh), cudaMemcpyHostToDevice, ctx->stream),
                   "pixels");
        const uint8_t* mr = m + ry0 * w + rx0;
        PoolBuf rgb8(ctx, size_t(S * S * 3)), bin8(ctx, size_t(S * S));
        ck(mbx_window_to_model(ctx, img.as<uint8_t>(), rw * ch, ch, mr, w, rx0, ry0, rw, rh, w, h, c.x, c.y, c.side, S,
                               rgb8.as<uint8_t>(), bin8.as<uint8_t>()));
        const Noise noise = noise_for(1, ep.seed, nv, ni, no);
        PoolBuf flags(ctx, 4);
        Tensor dec = run_model(rgb8.as<uint8_t>(), 3, bin8.as<uint8_t>(), 1, ep, noise, flags.as<int32_t>(),
                               reporter(progress, user));
        PoolBuf res(ctx, size_t(c.side * c.side * 3));
        ck(mbx_model_to_window(ctx, dec.data(), 1, S, c.side, res.as<uint8_t>()));
        dec = Tensor();
        ck(mbx_paste(ctx, img.as<uint8_t>(), 1, rw * ch, ch, mr, w, rx0, ry0, rw, rh, w, h, c.x, c.y, c.side,
                     res.as<uint8_t>(), ep.paste, nullptr));
        check_cuda(cudaMemcpy2DAsync(pixels + src.y * stride + src.x * ch, size_t(stride),
                                     img.as<uint8_t>() + ((src.y - ry0) * rw + (src.x - rx0)) * ch, size_t(rw * ch),
                                     size_t(src.width * ch), size_t(src.height), cudaMemcpyDeviceToHost, ctx->stream),
                   "pixels");
        check_cuda(cudaStreamSynchronize(ctx->stream), "inpaint");
        return src;
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

int32_t mbx_inpaint_with_noise(mbx_engine* engine, uint8_t* pixels, uint32_t width, uint32_t height, uint32_t stride,
                               uint32_t channels, const uint8_t* mask, uint32_t mask_stride,
                               const mbx_inpaint_params* params, const float* noise_vae, const float* noise_init,
                               const float* noise_offset, mbx_progress_fn progress, void* user, mbx_rect* changed) {
    return eguard([&] {
        require_engine(engine);
        if (changed) *changed = mbx_rect{0, 0, 0, 0};
        // Argument checks in the reference's order (src/ffi.rs:207-214, src/pipeline.rs:172-190).
        MBX_REQUIRE(pixels != nullptr && mask != nullptr, "null argument");
        MBX_REQUIRE(width > 0 && height > 0 && (uint64_t)stride >= (uint64_t)width * channels && mask_stride >= width,
                    "bad dimensions or stride");
        MBX_REQUIRE(channels == 3 || channels == 4, "image must be RGB or RGBA");
        (void)resolve(params);
        MBX_REQUIRE(!noise_vae == !noise_init && !noise_vae == !noise_offset, "give all three noise tensors or none");
        use(engine);
        mbx_ctx* ctx = engine->ctx;
        const int64_t L = engine->latent();
        Tensor dv, di, dof;
        if (noise_vae) {
            dv = Tensor(ctx, 2, L, L, 4);
            di = Tensor(ctx, 1, L, L, 4);
            dof = Tensor(ctx, 1, 1, 1, 4);
            check_cuda(cudaMemcpyAsync(dv.data(), noise_vae, size_t(dv.size()) * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "noise");
            check_cuda(cudaMemcpyAsync(di.data(), noise_init, size_t(di.size()) * 4, cudaMemcpyHostToDevice, ctx->stream),
                       "noise");
            check_cuda(cudaMemcpyAsync(dof.data(), noise_offset, size_t(dof.size()) * 4, cudaMemcpyHostToDevice,
                                       ctx->stream),
                       "noise");
        }
        const mbx_rect r = engine->inpaint_any(pixels, width, height, stride, channels, mask, mask_stride, params,
                                               dv ? dv.data() : nullptr, di ? di.data() : nullptr,
                                               dof ? dof.data() : nullptr, progress, user);
        if (changed) *changed = r;
    });
}

int32_t mbx_inpaint(mbx_engine* engine, uint8_t* pixels, uint32_t width, uint32_t height, uint32_t stride,
                    uint32_t channels, const uint8_t* mask, uint32_t mask_stride, const mbx_inpaint_params* params,
                    mbx_progress_fn progress, void* user, mbx_rect* changed) {
    return mbx_inpaint_with_noise(engine, pixels, width, height, stride, channels, mask, mask_stride, params, nullptr,
                                  nullptr, nullptr, progress, user, changed);
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

int32_t mbx_dpm_coefficients(uint32_t steps, double strength, int32_t trailing, int64_t i, int64_t restart_at,
                             float coef[5], int32_t* order) {
    return eguard([&] {
        MBX_REQUIRE(coef != nullptr && order != nullptr, "null argument");
        const Ddim d((int)steps, strength, trailing != 0);
        MBX_REQUIRE(i >= 0 && i < (int64_t)d.timesteps.size(), "step index outside the schedule");
        double lambda_prev = 0.0;
        const bool has_prev = i > 0 && i != restart_at;
        if (has_prev) {
            double a, s;
            dpm_abl(d, d.timesteps[size_t(i - 1)], a, s, lambda_prev);
        }
        int o = 0;
        dpm_step_coef(d, size_t(i), has_prev, lambda_prev, coef, &o);
        *order = o;
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
