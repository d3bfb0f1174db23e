// The Moebius student UNet (reference src/unet/{mod,blocks,embed,transformer,lambda}.rs)
// on the kernel ABI. Structure (src/unet/mod.rs:59-85):
//
//   conv_in   DWConv2d 9 → ch0
//   down i    2 × (DWResnet, MixTransformer) [+ Downsample2D on levels 0, 1]
//   up i      3 × (concat skip, DWResnet, MixTransformer) [+ Upsample2D on levels 0, 1]
//   out       GroupNorm(32) + SiLU → DWConv2d ch0 → 4
//
// Fusions relative to the reference's op sequence (same arithmetic, fewer
// passes over HBM): the MixTransformer's GroupNorm is applied in proj_in's
// operand gather; a GroupNorm + SiLU in front of a DWConv2d without a skip is
// applied in the depthwise kernel's window; to_k / to_v run as one GEMM; the MixFFN SiLU is the inverted
// conv's epilogue; the λ outputs are added straight into the hidden state; all
// resnets' time_emb_proj run as one GEMM per step.
#include <cmath>
#include <cstring>

#include "eng_models.h"

namespace mbx {
namespace eng {

namespace {
constexpr float kResnetEps = 1e-5f;      // src/config.rs:43-44
constexpr float kTransformerGnEps = 1e-6f;  // src/config.rs:45-46
constexpr float kLayerNormEps = 1e-5f;   // src/config.rs:47-48
constexpr int64_t kWaugRows = 228;       // 225 taps + bias column, padded to a multiple of 4

Tensor layer_norm(const Tensor& x, const DevBuf& g, const DevBuf& b) {
    Tensor out(x.ctx(), x.n, x.h, x.w, x.c);
    ck(mbx_layer_norm(x.ctx(), x.data(), x.pixels(), x.c, g.f(), b.f(), kLayerNormEps, out.data()));
    return out;
}

// gn_scale / gn_shift: the input is read as SiLU(x*gn_scale + gn_shift) (GroupNorm + SiLU prologue).
Tensor depthwise(const Tensor& x, const DevBuf& w, const DevBuf& b, int epilogue, const float* gn_scale = nullptr,
                 const float* gn_shift = nullptr) {
    Tensor out(x.ctx(), x.n, x.h, x.w, epilogue == MBX_EPILOGUE_GLU_SILU ? x.c / 2 : x.c);
    if (gn_scale)
        ck(mbx_depthwise3x3_fused(x.ctx(), x.data(), x.n, x.h, x.w, x.c, gn_scale, gn_shift, 1, w.f(), b.f(),
                                  epilogue, out.data()));
    else
        ck(mbx_depthwise3x3(x.ctx(), x.data(), x.n, x.h, x.w, x.c, w.f(), b.f(), epilogue, out.data()));
    return out;
}

// Depthwise weights [3, 3, c] and bias [c] under `<name>` (src/unet/load.rs:65-69).
void load_depthwise(const Loader& l, const std::string& name, int64_t c, DevBuf& w, DevBuf& b) {
    const Loader s = l.sub(name);
    const std::vector<float> wv = s.f32s("weight", {3, 3, c});
    w = DevBuf(wv.data(), wv.size() * 4);
    b = s.vec("bias", c);
}

// Concatenation of same-width [rows_i, cols] weights in a common precision
// (f16 when every part is f16, else f32).
Param concat_rows(mbx_ctx* ctx, const std::vector<const StTensor*>& parts, int64_t cols) {
    bool all_f16 = true;
    int64_t rows = 0;
    for (const StTensor* t : parts) {
        all_f16 = all_f16 && t->dtype == "F16";
        rows += t->shape[0];
    }
    if (all_f16) {
        std::vector<uint8_t> buf;
        for (const StTensor* t : parts) buf.insert(buf.end(), t->data, t->data + t->bytes);
        return Param(ctx, buf.data(), MBX_DTYPE_F16, rows, 1, cols);
    }
    std::vector<float> buf;
    for (const StTensor* t : parts) {
        const size_t count = t->bytes / (t->dtype == "F32" ? 4 : 2);
        for (size_t i = 0; i < count; ++i) {
            if (t->dtype == "F32") {
                float v;
                std::memcpy(&v, t->data + 4 * i, 4);
                buf.push_back(v);
            } else {
                uint16_t hb;
                std::memcpy(&hb, t->data + 2 * i, 2);
                buf.push_back(f16_to_f32(hb));
            }
        }
    }
    return Param(ctx, buf.data(), MBX_DTYPE_F32, rows, 1, cols);
}

int64_t head_width(int64_t c) {
    if (c % kHeads != 0 || (c / kHeads) % 8 != 0)
        fail(MBX_ERR_WEIGHTS, "lambda layer: " + std::to_string(c) + " channels do not split into 8 heads of 8-aligned width");
    return c / kHeads;
}
}  // namespace

// ---------------------------------------------------------------- blocks (src/unet/blocks.rs)

DwConv2d DwConv2d::load(const Loader& l, int64_t c_in, int64_t c_out) {
    DwConv2d d;
    d.c_in = c_in;
    d.c_out = c_out;
    load_depthwise(l, "conv_dw", c_in, d.dw_w, d.dw_b);
    d.pw = Conv::load1x1(l, "conv_pw", c_in, c_out, true);
    return d;
}

// y = pw1x1(relu(dw3x3(a) + b1)) + b2 (+ a when c_in == c_out), src/unet/blocks.rs:47-53, with a = x
// or a = SiLU(x*gn_scale + gn_shift). Without the skip, a is built inside the depthwise kernel's window
// and never stored; with it, a is stored once for the 1×1 conv's residual read (rebuilding it in the
// conv's epilogue cost that kernel more than the saved pass).
Tensor DwConv2d::forward(const Tensor& x, const float* gn_scale, const float* gn_shift, const NextNorm* next) const {
    const bool skip = c_in == c_out;
    if (gn_scale && skip) {
        Tensor a(x.ctx(), x.n, x.h, x.w, x.c);
        ck(mbx_group_norm_apply(x.ctx(), x.data(), x.n, x.h * x.w, x.c, gn_scale, gn_shift, 1, nullptr, a.data()));
        return forward(a, nullptr, nullptr, next);
    }
    Tensor mid = depthwise(x, dw_w, dw_b, MBX_EPILOGUE_RELU, gn_scale, gn_shift);
    if (next) return conv_gn(mid, pw, *next, skip ? x.data() : nullptr);
    return conv1x1(mid, pw, skip ? x.data() : nullptr);
}

DwResnet DwResnet::load(const Loader& l, int64_t c_in, int64_t c_out) {
    DwResnet r;
    r.c_in = c_in;
    r.c_out = c_out;
    r.norm1 = GroupNormP::load(l, "norm1", c_in, kResnetEps);
    r.conv1 = DwConv2d::load(l.sub("conv1"), c_in, c_out);
    r.norm2 = GroupNormP::load(l, "norm2", c_out, kResnetEps);
    r.conv2 = DwConv2d::load(l.sub("conv2"), c_out, c_out);
    if (c_in != c_out) {
        r.has_shortcut = true;
        r.shortcut = Conv::load1x1(l, "conv_shortcut", c_in, c_out, true);
    }
    return r;
}

// src/unet/blocks.rs:84-112; the time embedding projection arrives precomputed.
Tensor DwResnet::forward(const Tensor& x, const float* temb_proj) const {
    MBX_REQUIRE(x.c == c_in, "DwResnet input channels");
    // Each GroupNorm + SiLU is applied by the DWConv2d that follows it (statistics pass here).
    Tensor scale, shift;
    gn_affine(x, norm1, nullptr, scale, shift);
    // norm2's statistics (of b + temb) come from conv1's pointwise epilogue.
    Tensor scale2, shift2;
    const NextNorm next{&norm2, temb_proj, &scale2, &shift2};
    Tensor b = conv1.forward(x, scale.data(), shift.data(), &next);
    Tensor out = conv2.forward(b, scale2.data(), shift2.data());
    b = Tensor();
    scale = Tensor();
    shift = Tensor();
    if (has_shortcut) return conv1x1(x, shortcut, out.data());
    ck(mbx_add_inplace(x.ctx(), out.data(), x.data(), out.size()));
    return out;
}

// ---------------------------------------------------------------- transformer (src/unet/transformer.rs)

MixTransformer MixTransformer::load(const Loader& l, int64_t c, int64_t level_hw, const Tensor& ehs) {
    MixTransformer m;
    mbx_ctx* ctx = l.ctx();
    m.c = c;
    const int64_t hidden = c * 5 / 2;  // MIX_MLP_RATIO 2.5
    MBX_REQUIRE(c % 2 == 0, "MixTransformer: odd channel count");
    const Loader b = l.sub("transformer_blocks.0");
    const Loader ff = b.sub("ff");
    m.norm = GroupNormP::load(l, "norm", c, kTransformerGnEps);
    m.proj_in = Conv::load1x1(l, "proj_in", c, c, true);
    for (int i = 0; i < 3; ++i) {
        const Loader n = b.sub("norm" + std::to_string(i + 1));
        m.ln_g[i] = n.vec("weight", c);
        m.ln_b[i] = n.vec("bias", c);
    }
    const int64_t k = head_width(c);

    // Self-λ (src/unet/lambda.rs:84-104): q, [k | v] and the folded position filter.
    {
        const Loader a = b.sub("attn1");
        SelfLambdaP& s = m.attn1;
        s.c = c;
        s.k = k;
        s.to_q = Conv::load1x1(a, "to_q", c, c, true);
        const StTensor& wk = a.raw("to_k.weight", {k, c});
        const StTensor& wv = a.raw("to_v.weight", {k, c});
        s.to_kv.w = concat_rows(ctx, {&wk, &wv}, c);
        std::vector<float> bias(size_t(2 * k), 0.0f);
        const std::vector<float> bv = a.f32s("to_v.bias", {k});
        std::copy(bv.begin(), bv.end(), bias.begin() + k);
        s.to_kv.b = DevBuf(bias.data(), bias.size() * 4);
        s.to_kv.c_in = c;
        s.to_kv.c_out = 2 * k;
        const std::vector<float> pw = a.f32s("pos_conv.weight", {k, 225});
        const std::vector<float> pb = a.f32s("pos_conv.bias", {k});
        std::vector<float> waug(size_t(kWaugRows * k), 0.0f);  // [228][k] = [W | b]ᵀ
        for (int64_t d = 0; d < 225; ++d)
            for (int64_t kk = 0; kk < k; ++kk) waug[size_t(d * k + kk)] = pw[size_t(kk * 225 + d)];
        for (int64_t kk = 0; kk < k; ++kk) waug[size_t(225 * k + kk)] = pb[size_t(kk)];
        s.w_aug = Param(ctx, waug.data(), MBX_DTYPE_F32, kWaugRows, 1, k);
    }

    // Cross-λ (src/unet/lambda.rs:203-249): per-branch constants from the fixed conditioning.
    {
        const Loader a = b.sub("attn2");
        CrossLambdaP& x = m.attn2;
        x.c = c;
        x.k = k;
        x.hw = level_hw;
        x.to_q = Conv::load1x1(a, "to_q", c, c, true);
        Conv tk, tv;
        tk.w = a.param("to_k.weight", k, 1, kEhsDim);
        tk.c_in = kEhsDim;
        tk.c_out = k;
        tv.w = a.param("to_v.weight", k, 1, kEhsDim);
        tv.b = a.vec("to_v.bias", k);
        tv.c_in = kEhsDim;
        tv.c_out = k;
        Tensor keys = conv1x1(ehs, tk);  // [2·10, k]: uncond rows, then cond rows
        Tensor vals = conv1x1(ehs, tv);
        x.lambda_c = DevBuf(size_t(2 * k * k) * 4);
        ck(mbx_lambda_content(ctx, keys.data(), k, vals.data(), k, 2, kTokens, k, k, x.lambda_c.f()));
        x.v_table = DevBuf(size_t(2 * kTokens * k) * 4);
        check_cuda(cudaMemcpyAsync(x.v_table.get(), vals.data(), x.v_table.bytes(), cudaMemcpyDeviceToDevice,
                                   ctx->stream),
                   "cross-lambda values");
        const std::vector<int64_t> es = a.shape("rel_pos_emb");
        if (es.size() != 3 || es[0] != level_hw || es[1] != kTokens || es[2] != k)
            fail(MBX_ERR_WEIGHTS, a.key("rel_pos_emb") + ": position table does not match the level's " +
                                      std::to_string(level_hw) + " pixels");
        const std::vector<float> e = a.f32s("rel_pos_emb", {level_hw, kTokens, k});
        x.e_table = DevBuf(e.data(), e.size() * 4);
        check_cuda(cudaStreamSynchronize(ctx->stream), "cross-lambda constants");
    }

    m.inverted = Conv::load1x1(ff.sub("inverted_conv"), "conv", c, 2 * hidden, true);
    load_depthwise(ff.sub("depth_conv"), "conv", 2 * hidden, m.dw_w, m.dw_b);
    m.point = Conv::load1x1(ff.sub("point_conv"), "conv", hidden, c, false);
    m.proj_out = Conv::load1x1(l, "proj_out", c, c, true);
    return m;
}

// src/unet/transformer.rs:319-357 and src/unet/lambda.rs:107-151,252-273.
Tensor MixTransformer::forward(const Tensor& x, int branch_period) const {
    MBX_REQUIRE(x.c == c, "MixTransformer channels");
    mbx_ctx* ctx = x.ctx();
    const int64_t k = attn1.k, hw = x.h * x.w;
    Tensor scale, shift;
    gn_affine(x, norm, nullptr, scale, shift);
    Tensor h = conv1x1(x, proj_in, nullptr, scale.data(), shift.data(), false);
    scale = Tensor();
    shift = Tensor();

    {  // h += selfλ(LN1(h))
        Tensor t = layer_norm(h, ln_g[0], ln_b[0]);
        Tensor q = conv1x1(t, attn1.to_q);
        Tensor kv = conv1x1(t, attn1.to_kv);
        t = Tensor();
        Tensor lam(ctx, x.n, 1, k, k);
        ck(mbx_lambda_content(ctx, kv.data(), 2 * k, kv.data() + k, 2 * k, x.n, hw, k, k, lam.data()));
        Tensor a(ctx, x.pixels() * kHeads, 1, 1, kWaugRows);
        ck(mbx_conv1x1(ctx, q.data(), 1, x.pixels() * kHeads, 1, k, attn1.w_aug.get(), nullptr, nullptr, a.data()));
        ck(mbx_self_lambda_position(ctx, q.data(), lam.data(), a.data(), kWaugRows, kv.data() + k, 2 * k, x.n, x.h,
                                    x.w, k, h.data()));
    }
    {  // h += crossλ(LN2(h))
        MBX_REQUIRE(hw == attn2.hw, "CrossLambda input size does not match the position table");
        Tensor t = layer_norm(h, ln_g[1], ln_b[1]);
        Tensor q = conv1x1(t, attn2.to_q);
        t = Tensor();
        const int64_t first = branch_period == 1 ? 1 : 0;  // cond-only batches use branch 1
        ck(mbx_cross_lambda_position(ctx, q.data(), attn2.e_table.f(), attn2.lambda_c.f() + first * k * k,
                                     attn2.v_table.f() + first * kTokens * k, branch_period, x.n, hw, k, h.data()));
    }
    Tensor u;
    {  // u = h + MixFFN(LN3(h))
        Tensor t = layer_norm(h, ln_g[2], ln_b[2]);
        Tensor a = conv1x1(t, inverted, nullptr, nullptr, nullptr, false, MBX_ACT_SILU);
        t = Tensor();
        Tensor g = depthwise(a, dw_w, dw_b, MBX_EPILOGUE_GLU_SILU);
        a = Tensor();
        u = conv1x1(g, point, h.data());
    }
    h = Tensor();
    return conv1x1(u, proj_out, x.data());
}

// ---------------------------------------------------------------- UNet (src/unet/mod.rs)

UNet::UNet(mbx_ctx* ctx, const StFile& f) : ctx_(ctx) {
    const Loader root(ctx, &f, "");
    const Loader d = root.sub("diff_model");
    // Shape from the weights: ch0 from the time embedding, level widths from the resnets,
    // latent side from the first cross-λ position table.
    const std::vector<int64_t> l1 = d.shape("time_embedding.linear_1.weight");
    MBX_REQUIRE(l1.size() == 2, "time_embedding.linear_1.weight must be 2-D");
    shape_.time_embed = l1[0];
    shape_.time_proj = l1[1];
    for (int i = 0; i < 3; ++i)
        shape_.ch[i] = d.shape("down_blocks." + std::to_string(i) + ".resnets.0.conv1.conv_pw.weight")[0];
    const int64_t hw0 = d.shape("down_blocks.0.attentions.0.transformer_blocks.0.attn2.rel_pos_emb")[0];
    shape_.latent = (int64_t)std::llround(std::sqrt((double)hw0));
    if (shape_.latent * shape_.latent != hw0 || shape_.latent % 4 != 0)
        fail(MBX_ERR_WEIGHTS, "cross-lambda position table is not a square map divisible by 4");
    if (shape_.time_proj != shape_.ch[0] || shape_.time_proj % 2 != 0)
        fail(MBX_ERR_WEIGHTS, "time embedding width does not match the first level");
    const int64_t* ch = shape_.ch;
    auto level_hw = [&](int lvl) { return (shape_.latent >> lvl) * (shape_.latent >> lvl); };

    // Conditioning (src/unet/embed.rs:79-90): rows 10..20 (uncond) then 0..10 (cond) → encoder_hid_proj.
    Tensor ehs;
    {
        const std::vector<float> table = root.f32s("embedding_layer.weight", {kNumEmbeddings, kEncoderHid});
        std::vector<float> rows(table.size());
        const size_t half = size_t(kTokens * kEncoderHid);
        std::copy(table.begin() + half, table.end(), rows.begin());
        std::copy(table.begin(), table.begin() + half, rows.begin() + half);
        Tensor t(ctx, 1, 1, kNumEmbeddings, kEncoderHid);
        check_cuda(cudaMemcpyAsync(t.data(), rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, ctx->stream),
                   "conditioning upload");
        const Conv proj = Conv::load1x1(d, "encoder_hid_proj", kEncoderHid, kEhsDim, true);
        ehs = conv1x1(t, proj);
        check_cuda(cudaStreamSynchronize(ctx->stream), "conditioning");
    }

    const Loader te = d.sub("time_embedding");
    lin1 = Conv::load1x1(te, "linear_1", shape_.time_proj, shape_.time_embed, true);
    lin2 = Conv::load1x1(te, "linear_2", shape_.time_embed, shape_.time_embed, true);
    conv_in = DwConv2d::load(d.sub("conv_in"), kUnetIn, ch[0]);

    std::vector<const StTensor*> tw;  // every resnet's time_emb_proj, in forward order
    std::vector<float> tb;
    auto add_temb = [&](const Loader& l, DwResnet& r) {
        tw.push_back(&l.raw("time_emb_proj.weight", {r.c_out, shape_.time_embed}));
        const std::vector<float> b = l.f32s("time_emb_proj.bias", {r.c_out});
        r.temb_offset = (int64_t)tb.size();
        tb.insert(tb.end(), b.begin(), b.end());
    };

    int64_t c_prev = ch[0];
    std::vector<int64_t> skips{ch[0]};
    for (int i = 0; i < 3; ++i) {
        const Loader l = d.sub("down_blocks." + std::to_string(i));
        Level lv;
        for (int j = 0; j < 2; ++j) {
            const Loader rl = l.sub("resnets." + std::to_string(j));
            lv.resnets.push_back(DwResnet::load(rl, j == 0 ? c_prev : ch[i], ch[i]));
            add_temb(rl, lv.resnets.back());
            lv.attns.push_back(MixTransformer::load(l.sub("attentions." + std::to_string(j)), ch[i], level_hw(i), ehs));
            skips.push_back(ch[i]);
        }
        if (i < 2) {
            lv.has_sample = true;
            lv.sample = Conv::load3x3(l.sub("downsamplers.0"), "conv", ch[i], ch[i]);
            lv.sample.stride = 2;
            skips.push_back(ch[i]);
        }
        down_.push_back(std::move(lv));
        c_prev = ch[i];
    }
    int64_t h_c = ch[2];
    for (int i = 0; i < 3; ++i) {
        const int lvl = 2 - i;
        const int64_t c = ch[lvl];
        const Loader l = d.sub("up_blocks." + std::to_string(i));
        Level lv;
        for (int j = 0; j < 3; ++j) {
            const int64_t skip_c = skips.back();
            skips.pop_back();
            const Loader rl = l.sub("resnets." + std::to_string(j));
            lv.resnets.push_back(DwResnet::load(rl, h_c + skip_c, c));
            add_temb(rl, lv.resnets.back());
            lv.attns.push_back(MixTransformer::load(l.sub("attentions." + std::to_string(j)), c, level_hw(lvl), ehs));
            h_c = c;
        }
        if (i < 2) {
            lv.has_sample = true;
            lv.sample = Conv::load3x3(l.sub("upsamplers.0"), "conv", c, c);
            lv.sample.up = true;
        }
        up_.push_back(std::move(lv));
    }
    MBX_REQUIRE(skips.empty(), "skip stack not consumed");
    norm_out = GroupNormP::load(d, "conv_norm_out", ch[0], kResnetEps);
    conv_out = DwConv2d::load(d.sub("conv_out"), ch[0], kUnetOut);

    temb_proj.w = concat_rows(ctx, tw, shape_.time_embed);
    temb_proj.b = DevBuf(tb.data(), tb.size() * 4);
    temb_proj.c_in = shape_.time_embed;
    temb_proj.c_out = (int64_t)tb.size();
}

// [cos | sin] of t·exp(−ln(10000)·i/half) in f32 (src/unet/embed.rs:20-30).
void UNet::sinusoid(int64_t t, float* out) const {
    const int64_t half = shape_.time_proj / 2;
    const float log_period = -(float)std::log(10000.0);
    for (int64_t i = 0; i < half; ++i) {
        const float freq = std::exp(log_period * (float)i / (float)half);
        const float arg = (float)t * freq;
        out[i] = std::cos(arg);
        out[half + i] = std::sin(arg);
    }
}

Tensor UNet::forward(const Tensor& x, const float* t_sinusoid, int branch_period) const {
    MBX_REQUIRE(x.c == kUnetIn, "UNet input channels");
    MBX_REQUIRE(x.h == shape_.latent && x.w == shape_.latent, "UNet input must be the latent size");
    MBX_REQUIRE(branch_period == 1 || (branch_period == 2 && x.n % 2 == 0), "CFG batches hold (uncond, cond) pairs");
    mbx_ctx* ctx = x.ctx();
    const int64_t n = x.n;

    // Time embedding (src/unet/embed.rs:32-60) and every resnet's projection of SiLU(temb).
    std::vector<Tensor> tps;
    {
        Tensor sin(ctx, n, 1, 1, shape_.time_proj);
        check_cuda(cudaMemcpyAsync(sin.data(), t_sinusoid, size_t(sin.size()) * 4, cudaMemcpyDeviceToDevice,
                                   ctx->stream),
                   "timestep embedding");
        Tensor a = conv1x1(sin, lin1);
        ck(mbx_silu_inplace(ctx, a.data(), a.size()));
        Tensor temb = conv1x1(a, lin2);
        ck(mbx_silu_inplace(ctx, temb.data(), temb.size()));
        Tensor all = conv1x1(temb, temb_proj);
        const int64_t total = temb_proj.c_out;
        for (const std::vector<Level>* levels : {&down_, &up_})
            for (const Level& lv : *levels)
                for (const DwResnet& r : lv.resnets) {
                    Tensor tp(ctx, n, 1, 1, r.c_out);
                    check_cuda(cudaMemcpy2DAsync(tp.data(), size_t(r.c_out) * 4, all.data() + r.temb_offset,
                                                 size_t(total) * 4, size_t(r.c_out) * 4, size_t(n),
                                                 cudaMemcpyDeviceToDevice, ctx->stream),
                               "time projection split");
                    tps.push_back(std::move(tp));
                }
    }

    size_t ri = 0;
    std::vector<Tensor> skips;
    skips.push_back(conv_in.forward(x));
    for (const Level& lv : down_) {
        for (size_t j = 0; j < lv.resnets.size(); ++j) {
            Tensor a = lv.resnets[j].forward(skips.back(), tps[ri++].data());
            skips.push_back(lv.attns[j].forward(a, branch_period));
        }
        if (lv.has_sample) skips.push_back(conv3x3(skips.back(), lv.sample));
    }
    // The last down output is both the hidden state and the first skip (src/unet/mod.rs:261-265).
    Tensor h = std::move(skips.back());
    skips.pop_back();
    bool first = true;
    for (const Level& lv : up_) {
        for (size_t j = 0; j < lv.resnets.size(); ++j) {
            const Tensor& skip = first ? h : skips.back();
            Tensor cat(ctx, h.n, h.h, h.w, h.c + skip.c);
            ck(mbx_concat_channels(ctx, h.data(), h.c, skip.data(), skip.c, h.pixels(), cat.data()));
            if (!first) skips.pop_back();
            first = false;
            h = Tensor();
            Tensor a = lv.resnets[j].forward(cat, tps[ri++].data());
            cat = Tensor();
            h = lv.attns[j].forward(a, branch_period);
        }
        if (lv.has_sample) h = conv3x3(h, lv.sample);
    }
    MBX_REQUIRE(skips.empty(), "skip stack not consumed");
    Tensor scale, shift;
    gn_affine(h, norm_out, nullptr, scale, shift);
    return conv_out.forward(h, scale.data(), shift.data());
}

}  // namespace eng
}  // namespace mbx
