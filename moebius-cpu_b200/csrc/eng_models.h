// The reference's networks on the kernel ABI: the Moebius student UNet
// (src/unet/*) and the SDXL VAE (src/vae/*).
#pragma once

#include "eng.h"

namespace mbx {
namespace eng {

// ---------------------------------------------------------------- UNet

// Fixed structure of the shipped network (src/config.rs); the level widths
// and the latent side are read from the weight shapes so that scaled-down
// networks of the same structure (tests) load too.
struct UNetShape {
    int64_t ch[3] = {320, 640, 1280};
    int64_t latent = 64;         // side of the level-0 map (the cross-λ table size)
    int64_t time_proj = 320;     // sinusoid width = ch[0]
    int64_t time_embed = 1280;   // 4·ch[0]
};

constexpr int kUnetIn = 9;
constexpr int kUnetOut = 4;
constexpr int kHeads = 8;
constexpr int kTokens = 10;
constexpr int kEhsDim = 768;
constexpr int kEncoderHid = 3072;
constexpr int kNumEmbeddings = 20;

struct DwConv2d {
    int64_t c_in = 0, c_out = 0;
    DevBuf dw_w, dw_b;
    Conv pw;
    static DwConv2d load(const Loader& l, int64_t c_in, int64_t c_out);
    // gn_scale / gn_shift [n, c_in]: the block's input is SiLU(x*gn_scale + gn_shift), applied on
    // the fly (a GroupNorm + SiLU in front of the block).
    // next: the GroupNorm that consumes the output; its affine comes from the pointwise conv's epilogue.
    Tensor forward(const Tensor& x, const float* gn_scale = nullptr, const float* gn_shift = nullptr,
                   const NextNorm* next = nullptr) const;
};

struct DwResnet {
    int64_t c_in = 0, c_out = 0;
    GroupNormP norm1, norm2;
    DwConv2d conv1, conv2;
    bool has_shortcut = false;
    Conv shortcut;
    int64_t temb_offset = 0;  // column of this resnet's projection in the step's fused time_emb_proj output
    static DwResnet load(const Loader& l, int64_t c_in, int64_t c_out);
    Tensor forward(const Tensor& x, const float* temb_proj) const;  // temb_proj [n, c_out]
};

struct SelfLambdaP {
    int64_t c = 0, k = 0;
    Conv to_q, to_kv;  // to_kv = [to_k | to_v] with bias [0 | b_v]
    Param w_aug;       // [228, k]: 225 taps, the bias column, 2 zero rows
};

struct CrossLambdaP {
    int64_t c = 0, k = 0, hw = 0;
    Conv to_q;
    DevBuf e_table;   // [hw, 10, k]
    DevBuf lambda_c;  // [2][k][k] (uncond, cond)
    DevBuf v_table;   // [2][10][k]
};

struct MixTransformer {
    int64_t c = 0;
    GroupNormP norm;
    Conv proj_in, proj_out;
    DevBuf ln_g[3], ln_b[3];
    SelfLambdaP attn1;
    CrossLambdaP attn2;
    Conv inverted, point;
    DevBuf dw_w, dw_b;
    static MixTransformer load(const Loader& l, int64_t c, int64_t level_hw, const Tensor& ehs);
    // `branch_period`: 2 for CFG batches (uncond, cond, uncond, ...), 1 for cond-only.
    Tensor forward(const Tensor& x, int branch_period) const;
};

class UNet {
public:
    UNet(mbx_ctx* ctx, const StFile& f);
    const UNetShape& shape() const { return shape_; }
    // x [n, L, L, 9] (items already tiled per CFG copy), t_sinusoid [n, time_proj] → ε [n, L, L, 4].
    Tensor forward(const Tensor& x, const float* t_sinusoid, int branch_period) const;
    // The sinusoidal timestep embedding [cos | sin] (src/unet/embed.rs:20-30), host f32.
    void sinusoid(int64_t t, float* out) const;

private:
    mbx_ctx* ctx_;
    UNetShape shape_;
    Conv lin1, lin2, temb_proj;  // temb_proj: every resnet's time_emb_proj, concatenated
    DwConv2d conv_in, conv_out;
    GroupNormP norm_out;
    struct Level {
        std::vector<DwResnet> resnets;
        std::vector<MixTransformer> attns;
        bool has_sample = false;
        Conv sample;
    };
    std::vector<Level> down_, up_;
};

// ---------------------------------------------------------------- VAE

struct VaeResnet {
    GroupNormP norm1, norm2;
    Conv conv1, conv2;
    bool has_shortcut = false;
    Conv shortcut;
    static VaeResnet load(const Loader& l, int64_t c_in, int64_t c_out);
    Tensor forward(const Tensor& x) const;
};

struct VaeAttention {
    int64_t c = 0;
    GroupNormP norm;
    Conv to_q, to_k, to_v, to_out;
    static VaeAttention load(const Loader& l, int64_t c);
    Tensor forward(const Tensor& x) const;
};

class Vae {
public:
    static constexpr float kScaling = 0.13025f;
    Vae(mbx_ctx* ctx, const StFile& f);
    // images [b, H, W, 3] in [-1, 1], noise [b, H/8, W/8, 4] → scaled latents [b, H/8, W/8, 4].
    Tensor encode(const Tensor& images, const float* noise) const;
    // scaled latents [b, h, w, 4] → (dec + 1) / 2, unclamped, [b, 8h, 8w, 3].
    Tensor decode(const Tensor& latents) const;
    const int64_t* block_out() const { return ch_; }

private:
    mbx_ctx* ctx_;
    int64_t ch_[4] = {128, 256, 512, 512};
    // encoder
    Conv e_conv_in, e_conv_out, quant_conv;
    std::vector<std::vector<VaeResnet>> e_res;
    std::vector<Conv> e_down;
    VaeResnet e_mid0, e_mid1;
    VaeAttention e_attn;
    GroupNormP e_norm_out;
    // decoder
    Conv post_quant_conv, d_conv_in, d_conv_out;
    VaeResnet d_mid0, d_mid1;
    VaeAttention d_attn;
    std::vector<std::vector<VaeResnet>> d_res;
    std::vector<Conv> d_up;
    GroupNormP d_norm_out;
};

}  // namespace eng
}  // namespace mbx
