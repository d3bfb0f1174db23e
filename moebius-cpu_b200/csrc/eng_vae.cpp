// The SDXL VAE (diffusers AutoencoderKL, reference src/vae/{mod,encoder,decoder}.rs)
// on the kernel ABI: block_out (128, 256, 512, 512) (read from the weights),
// 2 resnets per encoder level and 3 per decoder level, one single-head
// attention in each mid block, GroupNorm(32) eps 1e-6. Residuals and shortcut
// outputs are added in the conv epilogues.
#include <cmath>

#include "eng_models.h"

namespace mbx {
namespace eng {

namespace {
constexpr float kVaeEps = 1e-6f;
constexpr float kSoftmaxFlush = -40.0f;  // src/vae/mod.rs:273-275
constexpr int64_t kLatentChannels = 4;
constexpr int64_t kImageChannels = 3;
}  // namespace

VaeResnet VaeResnet::load(const Loader& l, int64_t c_in, int64_t c_out) {
    VaeResnet r;
    r.norm1 = GroupNormP::load(l, "norm1", c_in, kVaeEps);
    r.conv1 = Conv::load3x3(l, "conv1", c_in, c_out);
    r.norm2 = GroupNormP::load(l, "norm2", c_out, kVaeEps);
    r.conv2 = Conv::load3x3(l, "conv2", c_out, c_out);
    if (c_in != c_out) {
        r.has_shortcut = true;
        r.shortcut = Conv::load1x1(l, "conv_shortcut", c_in, c_out, true);
    }
    return r;
}

namespace {
// SiLU(GN(x)) materialised once. The reference applies it inside the 3×3 convs' input
// gather (forward_prologue, src/vae/mod.rs:190-211); on the GPU that gather reads every
// input element nine times (once per tap), so the nine SiLUs cost more MUFU work than the
// tensor cores' MMAs, while one apply pass costs 8 B/elt of HBM traffic. Same values.
Tensor norm_silu(const Tensor& x, const GroupNormP& g) {
    Tensor out(x.ctx(), x.n, x.h, x.w, x.c);
    ck(mbx_group_norm_forward(x.ctx(), x.data(), x.n, x.h, x.w, x.c, g.groups, g.eps, g.gamma.f(), g.beta.f(),
                              nullptr, 1, out.data()));
    return out;
}
}  // namespace

// h = conv1(SiLU(GN1(x))); h = conv2(SiLU(GN2(h))); h + (shortcut(x) | x)  (src/vae/mod.rs:190-211).
Tensor VaeResnet::forward(const Tensor& x) const {
    // norm2's statistics come from conv1's epilogue; only its apply pass reads h.
    Tensor s2, t2;
    Tensor h = conv_gn(norm_silu(x, norm1), conv1, NextNorm{&norm2, nullptr, &s2, &t2});
    Tensor a(h.ctx(), h.n, h.h, h.w, h.c);
    ck(mbx_group_norm_apply(h.ctx(), h.data(), h.n, h.h * h.w, h.c, s2.data(), t2.data(), 1, nullptr, a.data()));
    h = Tensor();
    if (!has_shortcut) return conv3x3(a, conv2, nullptr, nullptr, false, x.data());
    Tensor o = conv3x3(a, conv2);
    a = Tensor();
    return conv1x1(x, shortcut, o.data());
}

VaeAttention VaeAttention::load(const Loader& l, int64_t c) {
    VaeAttention a;
    a.c = c;
    a.norm = GroupNormP::load(l, "group_norm", c, kVaeEps);
    a.to_q = Conv::load1x1(l, "to_q", c, c, true);
    a.to_k = Conv::load1x1(l, "to_k", c, c, true);
    a.to_v = Conv::load1x1(l, "to_v", c, c, true);
    a.to_out = Conv::load1x1(l.sub("to_out"), "0", c, c, true);
    return a;
}

// to_out(softmax(q·kᵀ/√c)·v) + x with q, k, v = 1×1 convs of GN(x) (src/vae/mod.rs:240-270):
// per item one score matrix, the tensor-core GEMM for both products, the flushed row softmax.
Tensor VaeAttention::forward(const Tensor& x) const {
    mbx_ctx* ctx = x.ctx();
    Tensor t(ctx, x.n, x.h, x.w, x.c);
    ck(mbx_group_norm_forward(ctx, x.data(), x.n, x.h, x.w, x.c, norm.groups, norm.eps, norm.gamma.f(),
                              norm.beta.f(), nullptr, 0, t.data()));
    Tensor q = conv1x1(t, to_q), k = conv1x1(t, to_k), v = conv1x1(t, to_v);
    const int64_t hw = x.h * x.w;
    Tensor scores(ctx, 1, 1, hw, hw);
    const float scale = 1.0f / std::sqrt((float)c);
    for (int64_t b = 0; b < x.n; ++b) {
        ck(mbx_gemm(ctx, scores.data(), q.item(b), hw, c, k.item(b), hw, 0, nullptr, nullptr));
        ck(mbx_softmax_rows(ctx, scores.data(), hw, hw, scale, kSoftmaxFlush));
        ck(mbx_gemm(ctx, t.item(b), scores.data(), hw, hw, v.item(b), c, 1, nullptr, nullptr));
    }
    return conv1x1(t, to_out, x.data());
}

Vae::Vae(mbx_ctx* ctx, const StFile& f) : ctx_(ctx) {
    const std::string sf = f.metadata("scaling_factor");
    if (sf.empty() || std::fabs(std::stof(sf) - kScaling) > 1e-7f)
        fail(MBX_ERR_WEIGHTS, "vae scaling_factor metadata \"" + sf + "\", expected \"0.13025\"");
    const Loader root(ctx, &f, "");
    const Loader e = root.sub("encoder"), d = root.sub("decoder");
    // block_out from the encoder's first conv of each level.
    for (int i = 0; i < 4; ++i)
        ch_[i] = e.shape("down_blocks." + std::to_string(i) + ".resnets.0.conv1.weight")[0];

    // Encoder (src/vae/encoder.rs:142-171).
    e_conv_in = Conv::load3x3(e, "conv_in", kImageChannels, ch_[0]);
    int64_t c_prev = ch_[0];
    for (int i = 0; i < 4; ++i) {
        const Loader b = e.sub("down_blocks." + std::to_string(i));
        std::vector<VaeResnet> rs;
        for (int j = 0; j < 2; ++j)
            rs.push_back(VaeResnet::load(b.sub("resnets." + std::to_string(j)), j == 0 ? c_prev : ch_[i], ch_[i]));
        e_res.push_back(std::move(rs));
        if (i < 3) {
            Conv dn = Conv::load3x3(b.sub("downsamplers.0"), "conv", ch_[i], ch_[i]);
            dn.stride = 2;
            dn.pad[0] = dn.pad[1] = 0;  // F.pad(x, (0, 1, 0, 1)) then stride 2 (encoder.rs:105-106)
            e_down.push_back(std::move(dn));
        }
        c_prev = ch_[i];
    }
    const int64_t top = ch_[3];
    e_mid0 = VaeResnet::load(e.sub("mid_block.resnets.0"), top, top);
    e_attn = VaeAttention::load(e.sub("mid_block.attentions.0"), top);
    e_mid1 = VaeResnet::load(e.sub("mid_block.resnets.1"), top, top);
    e_norm_out = GroupNormP::load(e, "conv_norm_out", top, kVaeEps);
    e_conv_out = Conv::load3x3(e, "conv_out", top, 2 * kLatentChannels);
    quant_conv = Conv::load1x1(root, "quant_conv", 2 * kLatentChannels, 2 * kLatentChannels, true);

    // Decoder (src/vae/decoder.rs:41-72).
    post_quant_conv = Conv::load1x1(root, "post_quant_conv", kLatentChannels, kLatentChannels, true);
    d_conv_in = Conv::load3x3(d, "conv_in", kLatentChannels, top);
    d_mid0 = VaeResnet::load(d.sub("mid_block.resnets.0"), top, top);
    d_attn = VaeAttention::load(d.sub("mid_block.attentions.0"), top);
    d_mid1 = VaeResnet::load(d.sub("mid_block.resnets.1"), top, top);
    c_prev = top;
    for (int i = 0; i < 4; ++i) {
        const int64_t c = ch_[3 - i];
        const Loader b = d.sub("up_blocks." + std::to_string(i));
        std::vector<VaeResnet> rs;
        for (int j = 0; j < 3; ++j)
            rs.push_back(VaeResnet::load(b.sub("resnets." + std::to_string(j)), j == 0 ? c_prev : c, c));
        d_res.push_back(std::move(rs));
        if (i < 3) {
            Conv upc = Conv::load3x3(b.sub("upsamplers.0"), "conv", c, c);
            upc.up = true;
            d_up.push_back(std::move(upc));
        }
        c_prev = c;
    }
    d_norm_out = GroupNormP::load(d, "conv_norm_out", ch_[0], kVaeEps);
    d_conv_out = Conv::load3x3(d, "conv_out", ch_[0], kImageChannels);
}

// src/vae/encoder.rs:173-216 (all items at once; the reference runs them one by one).
Tensor Vae::encode(const Tensor& images, const float* noise) const {
    MBX_REQUIRE(images.c == kImageChannels, "VAE encoder expects RGB");
    MBX_REQUIRE(images.h % 8 == 0 && images.w % 8 == 0, "VAE encoder input sides must be multiples of 8");
    Tensor cur = conv3x3(images, e_conv_in);
    for (int i = 0; i < 4; ++i) {
        for (const VaeResnet& r : e_res[size_t(i)]) cur = r.forward(cur);
        if (i < 3) cur = conv3x3(cur, e_down[size_t(i)]);
    }
    cur = e_mid0.forward(cur);
    cur = e_attn.forward(cur);
    cur = e_mid1.forward(cur);
    Tensor mom = conv3x3(norm_silu(cur, e_norm_out), e_conv_out);
    cur = Tensor();
    Tensor moments = conv1x1(mom, quant_conv);
    mom = Tensor();
    Tensor z(ctx_, images.n, images.h / 8, images.w / 8, kLatentChannels);
    ck(mbx_vae_sample(ctx_, moments.data(), noise, z.pixels(), kScaling, z.data()));
    return z;
}

// src/vae/decoder.rs:74-99.
Tensor Vae::decode(const Tensor& latents) const {
    MBX_REQUIRE(latents.c == kLatentChannels, "VAE decoder expects 4 latent channels");
    Tensor z(ctx_, latents.n, latents.h, latents.w, latents.c);
    ck(mbx_scale_add(ctx_, latents.data(), latents.size(), 1.0f / kScaling, 0.0f, z.data()));
    Tensor cur = conv1x1(z, post_quant_conv);
    z = Tensor();
    cur = conv3x3(cur, d_conv_in);
    cur = d_mid0.forward(cur);
    cur = d_attn.forward(cur);
    cur = d_mid1.forward(cur);
    for (int i = 0; i < 4; ++i) {
        for (const VaeResnet& r : d_res[size_t(i)]) cur = r.forward(cur);
        if (i < 3) cur = conv3x3(cur, d_up[size_t(i)]);
    }
    Tensor out = conv3x3(norm_silu(cur, d_norm_out), d_conv_out);
    cur = Tensor();
    ck(mbx_scale_add(ctx_, out.data(), out.size(), 0.5f, 0.5f, out.data()));
    return out;
}

}  // namespace eng
}  // namespace mbx
