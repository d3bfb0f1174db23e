// TEST INFRASTRUCTURE ONLY — the parity checker and the timed CPU baseline.
//
// A CPU restatement (C++17 + OpenMP) of the moebius-cpu engine kernels
// (the Rust crate's src/engine/*.rs). Only tests/, __graft_entry__.smoke() and
// bench.py (its cpu_baseline leg and `--impl reference` arm) may load this
// library; the product path in moebius-cpu_b200/ never links or calls it.
//
// Every function names the reference lines it restates. The reference's dense
// GEMMs live in the un-vendored crates `gemm` 0.19.0 and `private-gemm-x86`
// 0.1.22 (reference Cargo.lock:457,895); both compute a plain f32
// multiply-accumulate C (+)= A·B with FMA, which `gemm_nt` below restates
// with its own cache blocking (summation order differs inside a dot product,
// exactly as it differs between the reference's two backends).
//
// Built without -ffast-math and with -ffp-contract=off: every fused
// multiply-add below is an explicit fmaf(), matching the reference's mul_add.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <immintrin.h>
#include <omp.h>

namespace {

// ---------------------------------------------------------------- math.rs
// Cephes range reduction + degree-6 polynomial, reference src/engine/math.rs:18-30.
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693359375f;
constexpr float kLn2Lo = -2.12194440e-4f;
constexpr float kMaxX = 88.0f;
constexpr float kMinX = -87.33655f;

inline float ref_exp(float x) {
    x = std::min(std::max(x, kMinX), kMaxX);
    float n = std::round(x * kLog2e);  // Rust f32::round: half away from zero
    float r = fmaf(n, -kLn2Lo, fmaf(n, -kLn2Hi, x));
    float p = 1.9875691e-4f;
    p = fmaf(p, r, 1.3981999e-3f);
    p = fmaf(p, r, 8.3334520e-3f);
    p = fmaf(p, r, 4.1665796e-2f);
    p = fmaf(p, r, 1.6666665e-1f);
    p = fmaf(p, r, 5e-1f);
    float poly = fmaf(p * r, r, r) + 1.0f;
    uint32_t bits = uint32_t(int32_t(n) + 127) << 23;
    float scale;
    std::memcpy(&scale, &bits, 4);
    return poly * scale;
}

// x·σ(x), reference src/engine/math.rs:34-36.
inline float ref_silu(float x) { return x / (1.0f + ref_exp(-x)); }

// ---------------------------------------------------------------- GEMM
// C[m×n] (+)= A[m×k] · Bᵀ where B is stored [n×k] row-major (the reference's
// `MatRef::transposed` weight view, src/engine/gemm.rs:46-49). Restates
// gemm::matmul (src/engine/gemm.rs:63-132) with accumulate = `acc`.
constexpr int MR = 6, NR = 16, KC = 256;

// Packs B rows j0..j0+NR-1, k-range [p0, p0+kc) into bp[kc][NR] (zero padded).
void pack_b(const float* b, int64_t ldb, int64_t n, int64_t j0, int64_t p0, int64_t kc, float* bp) {
    for (int64_t p = 0; p < kc; ++p)
        for (int jj = 0; jj < NR; ++jj) {
            int64_t j = j0 + jj;
            bp[p * NR + jj] = j < n ? b[j * ldb + p0 + p] : 0.0f;
        }
}

void gemm_nt(int64_t m, int64_t n, int64_t k, const float* a, int64_t lda, const float* b, int64_t ldb,
             float* c, int64_t ldc, bool acc) {
    if (m <= 0 || n <= 0) return;
    if (!acc)
        for (int64_t i = 0; i < m; ++i) std::fill(c + i * ldc, c + i * ldc + n, 0.0f);
    if (k <= 0) return;
    const int64_t nb = (n + NR - 1) / NR;
    const int64_t mb = (m + MR - 1) / MR;
    // Row-block major so each thread streams its own A rows; B panels are
    // packed once per (column block, k block) into a shared buffer.
    std::vector<float> bpack((size_t)nb * KC * NR);
    for (int64_t p0 = 0; p0 < k; p0 += KC) {
        const int64_t kc = std::min<int64_t>(KC, k - p0);
#pragma omp parallel for schedule(static)
        for (int64_t jb = 0; jb < nb; ++jb) pack_b(b, ldb, n, jb * NR, p0, kc, &bpack[(size_t)jb * KC * NR]);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
        for (int64_t ib = 0; ib < mb; ++ib)
            for (int64_t jb = 0; jb < nb; ++jb) {
                const int64_t i0 = ib * MR, j0 = jb * NR;
                const int rows = (int)std::min<int64_t>(MR, m - i0);
                const float* bp = &bpack[(size_t)jb * KC * NR];
                __m256 c0[MR], c1[MR];
                for (int r = 0; r < MR; ++r) { c0[r] = _mm256_setzero_ps(); c1[r] = _mm256_setzero_ps(); }
                const float* ar[MR];
                for (int r = 0; r < MR; ++r) ar[r] = a + (i0 + std::min(r, rows - 1)) * lda + p0;
                for (int64_t p = 0; p < kc; ++p) {
                    const __m256 b0 = _mm256_loadu_ps(bp + p * NR);
                    const __m256 b1 = _mm256_loadu_ps(bp + p * NR + 8);
                    for (int r = 0; r < MR; ++r) {
                        const __m256 av = _mm256_broadcast_ss(ar[r] + p);
                        c0[r] = _mm256_fmadd_ps(av, b0, c0[r]);
                        c1[r] = _mm256_fmadd_ps(av, b1, c1[r]);
                    }
                }
                for (int r = 0; r < rows; ++r) {
                    float t[NR];
                    _mm256_storeu_ps(t, c0[r]);
                    _mm256_storeu_ps(t + 8, c1[r]);
                    float* crow = c + (i0 + r) * ldc;
                    const int cols = (int)std::min<int64_t>(NR, n - j0);
                    for (int jj = 0; jj < cols; ++jj) crow[j0 + jj] += t[jj];
                }
            }
    }
}

// init_output, reference src/engine/conv.rs:170-190: prefill with bias,
// residual or residual + bias; returns whether the GEMM accumulates.
bool init_output(float* out, int64_t rows, int64_t cols, const float* bias, const float* residual) {
    if (!bias && !residual) return false;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        float* o = out + r * cols;
        if (bias && !residual)
            std::memcpy(o, bias, cols * 4);
        else if (!bias && residual)
            std::memcpy(o, residual + r * cols, cols * 4);
        else
            for (int64_t j = 0; j < cols; ++j) o[j] = residual[r * cols + j] + bias[j];
    }
    return true;
}

// apply_affine, reference src/engine/norm.rs:134-147.
inline void apply_affine_px(const float* src, const float* scale, const float* shift, bool silu, float* dst,
                            int64_t c) {
    if (silu)
        for (int64_t j = 0; j < c; ++j) dst[j] = ref_silu(fmaf(src[j], scale[j], shift[j]));
    else
        for (int64_t j = 0; j < c; ++j) dst[j] = fmaf(src[j], scale[j], shift[j]);
}

}  // namespace

extern "C" {

void ora_set_threads(int t) { omp_set_num_threads(t > 0 ? t : omp_get_num_procs()); }
int ora_get_threads(void) { return omp_get_max_threads(); }

float ora_exp(float x) { return ref_exp(x); }
float ora_silu(float x) { return ref_silu(x); }

// ops::silu_inplace / add_inplace, reference src/engine/ops.rs:11-19.
void ora_silu_inplace(float* x, int64_t len) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < len; ++i) x[i] = ref_silu(x[i]);
}

void ora_add_inplace(float* a, const float* b, int64_t len) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < len; ++i) a[i] += b[i];
}

// The per-channel bias + per-item [n, c] timestep broadcast add of the
// memory-bound sweep: out = (x + bias[c]) + temb[item, c]. In the reference
// the bias is the conv output prefill (src/engine/conv.rs:170-190) and the
// temb add is the resnet's `h + temb_proj` (src/unet/blocks.rs:98). Either
// operand may be null.
void ora_bias_temb_add(const float* x, int64_t n, int64_t hw, int64_t c, const float* bias, const float* temb,
                       float* out) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t b = 0; b < n; ++b)
        for (int64_t p = 0; p < hw; ++p) {
            const float* xs = x + (b * hw + p) * c;
            float* o = out + (b * hw + p) * c;
            for (int64_t j = 0; j < c; ++j) {
                float v = xs[j];
                if (bias) v = v + bias[j];
                if (temb) v = v + temb[b * c + j];
                o[j] = v;
            }
        }
}

// Tensor::concat_channels_into, reference src/engine/tensor.rs:59-73.
void ora_concat_channels(const float* a, int64_t ca, const float* b, int64_t cb, int64_t pixels, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < pixels; ++p) {
        std::memcpy(out + p * (ca + cb), a + p * ca, ca * 4);
        std::memcpy(out + p * (ca + cb) + ca, b + p * cb, cb * 4);
    }
}

// GroupNorm::affine, reference src/engine/norm.rs:57-105 with gn_stats
// :110-129: per-channel f32 Σy, Σy² over 256-pixel chunks, folded to f64 per
// group, chunks summed in f64, var = E[y²] − mean² clamped at 0.
void ora_group_norm_affine(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t groups, float eps,
                           const float* gamma, const float* beta, const float* add, float* scale, float* shift) {
    const int64_t hw = h * w, cg = c / groups;
    const int64_t chunk = 256;
    const int64_t nchunks = (hw + chunk - 1) / chunk;
    const double count = double(hw * cg);
    std::vector<double> part((size_t)nchunks * groups * 2);
    for (int64_t b = 0; b < n; ++b) {
        const float* src = x + b * hw * c;
        const float* add_b = add ? add + b * c : nullptr;
#pragma omp parallel
        {
            std::vector<float> s(c), q(c);
#pragma omp for schedule(static)
            for (int64_t ch = 0; ch < nchunks; ++ch) {
                std::fill(s.begin(), s.end(), 0.0f);
                std::fill(q.begin(), q.end(), 0.0f);
                const int64_t p1 = std::min(hw, (ch + 1) * chunk);
                for (int64_t p = ch * chunk; p < p1; ++p) {
                    const float* px = src + p * c;
                    for (int64_t j = 0; j < c; ++j) {
                        float y = add_b ? px[j] + add_b[j] : px[j];
                        s[j] += y;
                        q[j] = fmaf(y, y, q[j]);
                    }
                }
                for (int64_t g = 0; g < groups; ++g) {
                    double ss = 0.0, qq = 0.0;
                    for (int64_t j = g * cg; j < (g + 1) * cg; ++j) {
                        ss += double(s[j]);
                        qq += double(q[j]);
                    }
                    part[(ch * groups + g) * 2] = ss;
                    part[(ch * groups + g) * 2 + 1] = qq;
                }
            }
        }
        for (int64_t g = 0; g < groups; ++g) {
            double sum = 0.0, sumsq = 0.0;
            for (int64_t ch = 0; ch < nchunks; ++ch) {
                sum += part[(ch * groups + g) * 2];
                sumsq += part[(ch * groups + g) * 2 + 1];
            }
            const double mean = sum / count;
            const double var = std::max(sumsq / count - mean * mean, 0.0);
            const double rstd = 1.0 / std::sqrt(var + double(eps));
            for (int64_t j = g * cg; j < (g + 1) * cg; ++j) {
                const double sc = rstd * double(gamma[j]);
                const double pre = add_b ? double(add_b[j]) : 0.0;
                scale[b * c + j] = float(sc);
                shift[b * c + j] = float(double(beta[j]) + (pre - mean) * sc);
            }
        }
    }
}

// GroupNorm::forward's apply pass (src/engine/norm.rs:41-53, apply_affine
// :134-147): out = [SiLU](x·scale[item,c] + shift[item,c]).
void ora_group_norm_apply(const float* x, int64_t n, int64_t hw, int64_t c, const float* scale, const float* shift,
                          int silu, float* out) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t b = 0; b < n; ++b)
        for (int64_t p = 0; p < hw; ++p)
            apply_affine_px(x + (b * hw + p) * c, scale + b * c, shift + b * c, silu != 0, out + (b * hw + p) * c, c);
}

// GroupNorm::forward, reference src/engine/norm.rs:41-53.
void ora_group_norm_forward(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, int64_t groups, float eps,
                            const float* gamma, const float* beta, const float* add, int silu, float* out) {
    std::vector<float> scale(n * c), shift(n * c);
    ora_group_norm_affine(x, n, h, w, c, groups, eps, gamma, beta, add, scale.data(), shift.data());
    ora_group_norm_apply(x, n, h * w, c, scale.data(), shift.data(), silu, out);
}

// layer_norm / ln_rows, reference src/engine/norm.rs:151-172.
void ora_layer_norm(const float* x, int64_t tokens, int64_t c, const float* gamma, const float* beta, float eps,
                    float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
        const float* s = x + t * c;
        float* d = out + t * c;
        float sum = 0.0f;
        for (int64_t j = 0; j < c; ++j) sum += s[j];
        const float mean = sum / float(c);
        float vs = 0.0f;
        for (int64_t j = 0; j < c; ++j) vs += (s[j] - mean) * (s[j] - mean);
        const float var = vs / float(c);
        const float rstd = 1.0f / std::sqrt(var + eps);
        for (int64_t j = 0; j < c; ++j) d[j] = fmaf((s[j] - mean) * rstd, gamma[j], beta[j]);
    }
}

// depthwise3x3, reference src/engine/depthwise.rs:31-59 (acc_block :112-143,
// tail_pixel :148-185): acc = bias, then taps in (ky, kx) order with
// fma(tap, x, acc); padding taps are skipped. epilogue 0 None, 1 ReLU,
// 2 GLU·SiLU (output c/2 channels: y[:c/2]·SiLU(y[c/2:])).
void ora_depthwise3x3(const float* x, int64_t n, int64_t h, int64_t w, int64_t c, const float* weight,
                      const float* bias, int epilogue, float* out) {
    const int64_t c_out = epilogue == 2 ? c / 2 : c;
#pragma omp parallel
    {
        std::vector<float> acc(c);
#pragma omp for schedule(static) collapse(2)
        for (int64_t b = 0; b < n; ++b)
            for (int64_t oy = 0; oy < h; ++oy)
                for (int64_t ox = 0; ox < w; ++ox) {
                    std::memcpy(acc.data(), bias, c * 4);
                    for (int64_t ky = 0; ky < 3; ++ky) {
                        const int64_t iy = oy + ky - 1;
                        if (iy < 0 || iy >= h) continue;
                        for (int64_t kx = 0; kx < 3; ++kx) {
                            const int64_t ix = ox + kx - 1;
                            if (ix < 0 || ix >= w) continue;
                            const float* src = x + ((b * h + iy) * w + ix) * c;
                            const float* tap = weight + (ky * 3 + kx) * c;
                            for (int64_t j = 0; j < c; ++j) acc[j] = fmaf(tap[j], src[j], acc[j]);
                        }
                    }
                    float* d = out + ((b * h + oy) * w + ox) * c_out;
                    if (epilogue == 0)
                        std::memcpy(d, acc.data(), c * 4);
                    else if (epilogue == 1)
                        for (int64_t j = 0; j < c; ++j) d[j] = std::max(acc[j], 0.0f);
                    else
                        for (int64_t j = 0; j < c_out; ++j) d[j] = acc[j] * ref_silu(acc[c_out + j]);
                }
    }
}

// Conv1x1::forward, reference src/engine/conv.rs:38-55: out = x·Wᵀ + bias
// (+ residual) via init_output prefill + accumulating GEMM. weight [c_out, c_in].
void ora_conv1x1(const float* x, int64_t pixels, int64_t c_in, const float* weight, int64_t c_out, const float* bias,
                 const float* residual, float* out) {
    bool acc = init_output(out, pixels, c_out, bias, residual);
    gemm_nt(pixels, c_out, c_in, x, c_in, weight, c_in, out, c_out, acc);
}

// Conv3x3::output_hw, reference src/engine/conv.rs:77-81.
void ora_conv3x3_output_hw(int64_t h, int64_t w, int64_t stride, const int64_t* pad, int upsample2x, int64_t* ho,
                           int64_t* wo) {
    const int64_t up = upsample2x ? 2 : 1;
    *ho = (h * up + pad[0] + pad[2] - 3) / stride + 1;
    *wo = (w * up + pad[1] + pad[3] - 3) / stride + 1;
}

// Conv3x3::forward_im2col, reference src/engine/conv.rs:106-130 with
// Geometry::gather :145-165: banded patch rows [band × 9·c_in] (K order
// ky, kx, c_in) times the [c_out, 9·c_in] weight, bias prefilled.
// Optional GN prologue (scale/shift [n, c_in], silu) applied to in-image taps
// only; the reference restricts its prologue to the Winograd path, and the
// values are identical either way.
void ora_conv3x3_im2col(const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in, const float* weight,
                        int64_t c_out, const float* bias, int64_t stride, const int64_t* pad, int upsample2x,
                        const float* pro_scale, const float* pro_shift, int pro_silu, float* out) {
    int64_t ho, wo;
    ora_conv3x3_output_hw(h, w, stride, pad, upsample2x, &ho, &wo);
    const int64_t k = 9 * c_in;
    const int64_t total = n * ho * wo;
    const int64_t band = std::min<int64_t>(std::max<int64_t>(std::min<int64_t>((8 << 20) / k, 4096), 64), total);
    const int shift = upsample2x ? 1 : 0;
    const int64_t hi = h << shift, wi = w << shift;
    std::vector<float> cols((size_t)band * k);
    for (int64_t start = 0; start < total; start += band) {
        const int64_t m = std::min(band, total - start);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < m; ++i) {
            const int64_t p = start + i;
            const int64_t b = p / (ho * wo), rem = p % (ho * wo);
            const int64_t oy = rem / wo, ox = rem % wo;
            float* row = &cols[(size_t)i * k];
            for (int64_t ky = 0; ky < 3; ++ky) {
                const int64_t iy = oy * stride + ky - pad[0];
                for (int64_t kx = 0; kx < 3; ++kx) {
                    const int64_t ix = ox * stride + kx - pad[1];
                    float* dst = row + (ky * 3 + kx) * c_in;
                    if (iy >= 0 && iy < hi && ix >= 0 && ix < wi) {
                        const float* src = x + ((b * h + (iy >> shift)) * w + (ix >> shift)) * c_in;
                        if (pro_scale)
                            apply_affine_px(src, pro_scale + b * c_in, pro_shift + b * c_in, pro_silu != 0, dst, c_in);
                        else
                            std::memcpy(dst, src, c_in * 4);
                    } else {
                        std::memset(dst, 0, c_in * 4);
                    }
                }
            }
        }
        float* dst = out + start * c_out;
        bool acc = init_output(dst, m, c_out, bias, nullptr);
        gemm_nt(m, c_out, k, cols.data(), k, weight, k, dst, c_out, acc);
    }
}

// Winograd F(2×2,3×3) for stride 1 / pad 1, reference src/engine/winograd.rs:48-120
// (kernel_transform :272-296, input_transform :302-326, output_transform
// :332-351, fill_strip's prologue :210-251). Banded over whole tile rows to
// bound memory; each tile is independent so banding does not change values.
void ora_conv3x3_winograd(const float* x, int64_t n, int64_t h, int64_t w, int64_t ci, const float* weight,
                          int64_t co, const float* bias_in, int upsample2x, const float* pro_scale,
                          const float* pro_shift, int pro_silu, float* out) {
    const int shift = upsample2x ? 1 : 0;
    const int64_t hi = h << shift, wi = w << shift;
    const int64_t th = (hi + 1) / 2, tw = (wi + 1) / 2;
    const int64_t tiles = n * th * tw;
    std::vector<float> bias0(co, 0.0f);
    const float* bias = bias_in ? bias_in : bias0.data();
    // U = G g Gᵀ, stored [16][co][ci] so each plane is a [co × ci] NT operand.
    std::vector<float> u((size_t)16 * co * ci);
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < co; ++o) {
        const float* g = weight + o * 9 * ci;
        for (int64_t i = 0; i < ci; ++i) {
            float t[4][3];
            for (int kx = 0; kx < 3; ++kx) {
                const float g0 = g[kx * ci + i], g1 = g[(3 + kx) * ci + i], g2 = g[(6 + kx) * ci + i];
                t[0][kx] = g0;
                t[1][kx] = 0.5f * (g0 + g1 + g2);
                t[2][kx] = 0.5f * (g0 - g1 + g2);
                t[3][kx] = g2;
            }
            for (int a = 0; a < 4; ++a) {
                u[((size_t)(a * 4) * co + o) * ci + i] = t[a][0];
                u[((size_t)(a * 4 + 1) * co + o) * ci + i] = 0.5f * (t[a][0] + t[a][1] + t[a][2]);
                u[((size_t)(a * 4 + 2) * co + o) * ci + i] = 0.5f * (t[a][0] - t[a][1] + t[a][2]);
                u[((size_t)(a * 4 + 3) * co + o) * ci + i] = t[a][2];
            }
        }
    }
    const int64_t band = std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>((4 << 20) / (16 * ci), 256), 4096) / tw) * tw;
    std::vector<float> v((size_t)16 * std::min(band, tiles) * ci);
    std::vector<float> mm((size_t)16 * std::min(band, tiles) * co);
    for (int64_t t0 = 0; t0 < tiles; t0 += band) {
        const int64_t mb = std::min(band, tiles - t0);
        // V planes [16][mb][ci].
#pragma omp parallel
        {
            std::vector<float> d(16 * ci);
#pragma omp for schedule(static)
            for (int64_t i = 0; i < mb; ++i) {
                const int64_t t = t0 + i;
                const int64_t b = t / (th * tw), rem = t % (th * tw);
                const int64_t ty = rem / tw, tx = rem % tw;
                for (int kk = 0; kk < 16; ++kk) {
                    const int64_t iy = 2 * ty + kk / 4 - 1, ix = 2 * tx + kk % 4 - 1;
                    float* dst = &d[kk * ci];
                    if (iy >= 0 && iy < hi && ix >= 0 && ix < wi) {
                        const float* src = x + ((b * h + (iy >> shift)) * w + (ix >> shift)) * ci;
                        if (pro_scale)
                            apply_affine_px(src, pro_scale + b * ci, pro_shift + b * ci, pro_silu != 0, dst, ci);
                        else
                            std::memcpy(dst, src, ci * 4);
                    } else {
                        std::memset(dst, 0, ci * 4);
                    }
                }
                for (int64_t c = 0; c < ci; ++c) {
                    float tt[16];
                    for (int col = 0; col < 4; ++col) {
                        const float d0 = d[col * ci + c], d1 = d[(4 + col) * ci + c], d2 = d[(8 + col) * ci + c],
                                    d3 = d[(12 + col) * ci + c];
                        tt[col] = d0 - d2;
                        tt[4 + col] = d1 + d2;
                        tt[8 + col] = d2 - d1;
                        tt[12 + col] = d1 - d3;
                    }
                    for (int r = 0; r < 4; ++r) {
                        const float* q = &tt[r * 4];
                        v[((size_t)(r * 4) * mb + i) * ci + c] = q[0] - q[2];
                        v[((size_t)(r * 4 + 1) * mb + i) * ci + c] = q[1] + q[2];
                        v[((size_t)(r * 4 + 2) * mb + i) * ci + c] = q[2] - q[1];
                        v[((size_t)(r * 4 + 3) * mb + i) * ci + c] = q[1] - q[3];
                    }
                }
            }
        }
        for (int xi = 0; xi < 16; ++xi)
            gemm_nt(mb, co, ci, &v[(size_t)xi * mb * ci], ci, &u[(size_t)xi * co * ci], ci, &mm[(size_t)xi * mb * co],
                    co, false);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < mb; ++i) {
            const int64_t t = t0 + i;
            const int64_t b = t / (th * tw), rem = t % (th * tw);
            const int64_t ty = rem / tw, tx = rem % tw;
            for (int64_t o = 0; o < co; ++o) {
                float m[16];
                for (int xi = 0; xi < 16; ++xi) m[xi] = mm[((size_t)xi * mb + i) * co + o];
                float u0[4], u1[4];
                for (int r = 0; r < 4; ++r) {
                    const float a = m[r * 4], bb = m[r * 4 + 1], cc = m[r * 4 + 2], dd = m[r * 4 + 3];
                    u0[r] = a + bb + cc;
                    u1[r] = bb - cc - dd;
                }
                const float y[4] = {u0[0] + u0[1] + u0[2] + bias[o], u1[0] + u1[1] + u1[2] + bias[o],
                                    u0[1] - u0[2] - u0[3] + bias[o], u1[1] - u1[2] - u1[3] + bias[o]};
                for (int kk = 0; kk < 4; ++kk) {
                    const int64_t oy = 2 * ty + kk / 2, ox = 2 * tx + kk % 2;
                    if (oy < hi && ox < wi) out[((b * hi + oy) * wi + ox) * co + o] = y[kk];
                }
            }
        }
    }
}

// Conv3x3::forward_prologue dispatch, reference src/engine/conv.rs:92-102:
// stride 1 / pad 1 → Winograd, anything else → im2col.
void ora_conv3x3(const float* x, int64_t n, int64_t h, int64_t w, int64_t c_in, const float* weight, int64_t c_out,
                 const float* bias, int64_t stride, const int64_t* pad, int upsample2x, const float* pro_scale,
                 const float* pro_shift, int pro_silu, float* out) {
    if (stride == 1 && pad[0] == 1 && pad[1] == 1 && pad[2] == 1 && pad[3] == 1)
        ora_conv3x3_winograd(x, n, h, w, c_in, weight, c_out, bias, upsample2x, pro_scale, pro_shift, pro_silu, out);
    else
        ora_conv3x3_im2col(x, n, h, w, c_in, weight, c_out, bias, stride, pad, upsample2x, pro_scale, pro_shift,
                           pro_silu, out);
}

// C[m×n] (+)= A[m×k]·Bᵀ with B stored [n×k] (the blocked GEMM above, exposed
// for the attention contractions of src/vae/mod.rs:259-262).
void ora_gemm_nt(int64_t m, int64_t n, int64_t k, const float* a, const float* b, float* c, int accumulate) {
    gemm_nt(m, n, k, a, k, b, k, c, n, accumulate != 0);
}

// softmax_rows, reference src/vae/mod.rs:273-293: in place per n-long row,
// a = (v − max)·scale, e = a < −40 ? 0 : exp(a), then v = e · (1 / Σe).
void ora_softmax_rows(float* x, int64_t rows, int64_t n, float scale) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        float* row = x + r * n;
        float mx = -INFINITY;
        for (int64_t i = 0; i < n; ++i) mx = std::max(mx, row[i]);
        float sum = 0.0f;
        for (int64_t i = 0; i < n; ++i) {
            const float a = (row[i] - mx) * scale;
            row[i] = a < -40.0f ? 0.0f : ref_exp(a);
            sum += row[i];
        }
        const float inv = 1.0f / sum;
        for (int64_t i = 0; i < n; ++i) row[i] *= inv;
    }
}

// gemm::matmul with arbitrary strides, reference src/engine/gemm.rs:63-132
// (MatRef :25-53). c is dense row-major [m × n]. Small cases only.
void ora_matmul(float* c, const float* a, int64_t m, int64_t k, int64_t a_rs, int64_t a_cs, const float* b, int64_t n,
                int64_t b_rs, int64_t b_cs, int accumulate) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (int64_t p = 0; p < k; ++p) s = fmaf(a[i * a_rs + p * a_cs], b[p * b_rs + j * b_cs], s);
            c[i * n + j] = accumulate ? c[i * n + j] + s : s;
        }
}

// ---------------------------------------------------------------- lambda.rs
// softmax_lambda, reference src/unet/lambda.rs:318-359 (column_max :361-369,
// exp_and_sum :371-380): keys [rows × k] is overwritten with exp(key − colmax);
// per-column sums in f32 over 256-row chunks folded in f64; λ = keysᵀ·v with
// f32 FMA accumulation, each row scaled by (float)(1 / sum).
void ora_softmax_lambda(float* keys, const float* v, int64_t rows, int64_t k, int64_t vd, float* lam) {
    std::vector<float> mx(size_t(k), -INFINITY);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t kk = 0; kk < k; ++kk) mx[size_t(kk)] = std::max(mx[size_t(kk)], keys[r * k + kk]);
    std::vector<double> sum(size_t(k), 0.0);
    for (int64_t r0 = 0; r0 < rows; r0 += 256) {
        std::vector<float> s(size_t(k), 0.0f);
        for (int64_t r = r0; r < std::min<int64_t>(rows, r0 + 256); ++r)
            for (int64_t kk = 0; kk < k; ++kk) {
                float& e = keys[r * k + kk];
                e = ref_exp(e - mx[size_t(kk)]);
                s[size_t(kk)] += e;
            }
        for (int64_t kk = 0; kk < k; ++kk) sum[size_t(kk)] += (double)s[size_t(kk)];
    }
#pragma omp parallel for schedule(static)
    for (int64_t kk = 0; kk < k; ++kk) {
        const float inv = (float)(1.0 / sum[size_t(kk)]);
        for (int64_t j = 0; j < vd; ++j) {
            float acc = 0.0f;
            for (int64_t r = 0; r < rows; ++r) acc = fmaf(keys[r * k + kk], v[r * vd + j], acc);
            lam[kk * vd + j] = acc * inv;
        }
    }
}

// tap_filter, reference src/unet/lambda.rs:154-184: for every pixel of one item and
// head, o[h] += A[p,h,225], then o[h] = fma(A[p,h,d], V[p+d], o[h]) over the in-map
// taps d = ky·15 + kx of the 15×15 window. a: [hw × 8 × 226]; v: [hw × vd];
// o: [hw × 8·vd].
void ora_tap_filter(const float* a, const float* v, float* o, int64_t hh, int64_t ww, int64_t vd) {
    const int64_t c = 8 * vd, hw = hh * ww;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < hw; ++p) {
        const int64_t y = p / ww, x = p % ww;
        const float* ap = a + p * 8 * 226;
        float* op = o + p * c;
        for (int h = 0; h < 8; ++h) {
            const float bias = ap[h * 226 + 225];
            for (int64_t t = 0; t < vd; ++t) op[h * vd + t] += bias;
        }
        const int64_t kx0 = std::max<int64_t>(0, 7 - x), kx1 = std::min<int64_t>(15, ww + 7 - x);
        for (int64_t ky = 0; ky < 15; ++ky) {
            const int64_t iy = y + ky - 7;
            if (iy < 0 || iy >= hh) continue;
            for (int64_t kx = kx0; kx < kx1; ++kx) {
                const float* vr = v + (iy * ww + x + kx - 7) * vd;
                const int64_t d = ky * 15 + kx;
                for (int h = 0; h < 8; ++h) {
                    const float coef = ap[h * 226 + d];
                    for (int64_t t = 0; t < vd; ++t) op[h * vd + t] = fmaf(coef, vr[t], op[h * vd + t]);
                }
            }
        }
    }
}

// dot with 8 independent lanes, then the lane sum and the tail (reference
// src/unet/lambda.rs:297-309).
static float lambda_dot(const float* a, const float* b, int64_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int64_t body = n / 8 * 8;
    float tail = 0.0f;
    for (int64_t i = body; i < n; ++i) tail += a[i] * b[i];
    for (int64_t i = 0; i < body; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = 0.0f;
    for (int l = 0; l < 8; ++l) s += acc[l];
    return s + tail;
}

// position_term, reference src/unet/lambda.rs:276-295: per pixel and head,
// B[m] = Q_h · E[p, m], then o[h] = fma(B[m], V[m], o[h]) for the 10 tokens.
// q, o: [hw × 8k]; e: [hw × 10 × k]; v: [10 × k].
void ora_position_term(const float* q, const float* e, const float* v, float* o, int64_t hw, int64_t k) {
    const int64_t c = 8 * k;
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < hw; ++p) {
        const float* ep = e + p * 10 * k;
        for (int h = 0; h < 8; ++h) {
            const float* qh = q + p * c + h * k;
            float* oh = o + p * c + h * k;
            for (int m = 0; m < 10; ++m) {
                const float b = lambda_dot(qh, ep + m * k, k);
                for (int64_t t = 0; t < k; ++t) oh[t] = fmaf(b, v[m * k + t], oh[t]);
            }
        }
    }
}

// timestep_sinusoid, reference src/unet/embed.rs:20-30: [cos | sin] of
// t · exp(log_period · i / half) with log_period = −ln(10000) as f32.
void ora_timestep_sinusoid(int64_t t, int64_t dim, float* out) {
    const int64_t half = dim / 2;
    const float log_period = -(float)std::log(10000.0);
    for (int64_t i = 0; i < half; ++i) {
        const float freq = std::exp(log_period * (float)i / (float)half);
        const float arg = (float)t * freq;
        out[i] = std::cos(arg);
        out[half + i] = std::sin(arg);
    }
}

// sample, reference src/vae/encoder.rs:219-230:
// z = fma(exp(0.5·clamp(logvar, −30, 20)), noise, mean) · 0.13025 per pixel;
// moments [pixels × 8] = mean(4) ‖ logvar(4).
void ora_vae_sample(const float* moments, const float* noise, int64_t pixels, float* z) {
    for (int64_t p = 0; p < pixels; ++p)
        for (int c = 0; c < 4; ++c) {
            const float lv = std::min(std::max(moments[p * 8 + 4 + c], -30.0f), 20.0f);
            z[p * 4 + c] = fmaf(ref_exp(0.5f * lv), noise[p * 4 + c], moments[p * 8 + c]) * 0.13025f;
        }
}

}  // extern "C"
