// Internal declarations shared by the moebius-cuda translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "../../include/moebius_cuda.h"

namespace mbx {

// Error raised inside the library; converted to a status code at the C ABI.
struct Error : std::runtime_error {
    int32_t code;
    Error(int32_t c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int32_t code, const std::string& msg) { throw Error(code, msg); }

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        int32_t code = e == cudaErrorMemoryAllocation ? MBX_ERR_OUT_OF_MEMORY : MBX_ERR_CUDA;
        fail(code, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

#define MBX_REQUIRE(cond, msg)                                     \
    do {                                                           \
        if (!(cond)) ::mbx::fail(MBX_ERR_INVALID_ARGUMENT, (msg)); \
    } while (0)

// Device-side error record written by kernels whose bounded waits gave up:
// [0] = code (0 = none), [1] = kernel id, [2] = detail (barrier / stage).
enum DeviceErr : int { kErrNone = 0, kErrWaitTimeout = 1 };
enum KernelId : int { kKConvTc = 1, kKGnSlab = 2, kKDepthwise = 3, kKWaitProbe = 4 };

// Stream-ordered best-fit caching allocator (device analogue of the
// reference's Scratch pool). All blocks are used on the context stream, so a
// block freed by one call can be handed to the next call without a sync.
class Pool {
public:
    explicit Pool(int device) : device_(device) {}
    ~Pool();
    void* alloc(size_t bytes);
    void free(void* p);
    void release_below(size_t min_bytes);
    size_t cached_bytes() const { return cached_; }
    size_t in_use_bytes() const { return in_use_; }

private:
    int device_;
    std::multimap<size_t, void*> free_;        // size -> block
    std::unordered_map<void*, size_t> used_;   // block -> size
    size_t cached_ = 0, in_use_ = 0;
    mutable std::mutex mu_;
};

}  // namespace mbx

struct mbx_ctx {
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int sm_count = 0;
    int* dev_err = nullptr;       // 4 ints, device memory, zeroed at create
    mbx::Pool* pool = nullptr;
    uint64_t launches = 0;
};

struct mbx_param {
    int32_t dtype = MBX_DTYPE_F32;
    int64_t c_out = 0, taps = 0, c_in = 0;
    int cin_pad = 0;   // c_in rounded up to the 32-channel K chunk
    int bn = 0;        // N tile (output channels per CTA tile)
    int cout_pad = 0;  // c_out rounded up to bn
    float* hi = nullptr;  // [cout_pad][taps][cin_pad] TF32-rounded high part (or the f16 values)
    float* lo = nullptr;  // same layout, TF32-rounded (w - hi); null for f16 weights (exact in TF32)
    CUtensorMap tmap_hi;
    CUtensorMap tmap_lo;
};

namespace mbx {

// Sets the calling thread's mbx_last_error() message (for entry points that
// catch their own exceptions).
void record_error(int32_t code, const char* msg);

// Raises `kernel`'s dynamic shared-memory limit to at least `bytes` on the
// calling thread's current device. The attribute belongs to the device that is
// current when it is set, so a process driving several GPUs needs it once per
// device: it is set on the first request per (device, kernel) and again only
// for a larger request. Safe to call from several host threads.
void ensure_smem_limit(const void* kernel, int bytes, const char* what);

// Kernel launchers (each returns after enqueueing on ctx->stream).
void launch_silu_inplace(mbx_ctx* ctx, float* x, int64_t len);
void launch_add(mbx_ctx* ctx, const float* a, const float* b, float* out, int64_t len);
void launch_bias_temb_add(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* bias,
                          const float* temb, float* out);
void launch_concat(mbx_ctx* ctx, const float* a, int64_t ca, const float* b, int64_t cb, int64_t pixels,
                   float* out);

// GroupNorm: partial sums per (item, pixel chunk, group) into `part`
// (f64 [n][chunks][groups][2]), then the fold into scale/shift.
int64_t gn_chunks(int64_t hw);
void launch_gn_partials(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, int64_t groups,
                        const float* add, double* part);
void launch_gn_finalize(mbx_ctx* ctx, const double* part, int64_t n, int64_t hw, int64_t c, int64_t groups,
                        float eps, const float* gamma, const float* beta, const float* add, float* scale,
                        float* shift);
void launch_gn_apply(mbx_ctx* ctx, const float* x, int64_t n, int64_t hw, int64_t c, const float* scale,
                     const float* shift, bool silu, const float* residual, float* out);
void launch_layer_norm(mbx_ctx* ctx, const float* x, int64_t tokens, int64_t c, const float* gamma,
                       const float* beta, float eps, float* out);

void launch_depthwise3x3(mbx_ctx* ctx, const float* x, int64_t n, int64_t h, int64_t w, int64_t c,
                         const float* weight, const float* bias, int epilogue, float* out,
                         const float* pro_scale = nullptr, const float* pro_shift = nullptr, bool pro_silu = false);

struct ConvShape {
    int64_t n, h, w, c_in;
    int64_t ho, wo;
    int stride, pad_t, pad_l, up;
};
// One thread waits, with the given limit in clock cycles, on a barrier nothing arrives at
// (the bounded-wait self-test behind mbx_selftest_wait_timeout).
void launch_wait_probe(mbx_ctx* ctx, int64_t cycles);
void launch_conv_tc(mbx_ctx* ctx, const float* x, const ConvShape& s, const mbx_param* p, const float* bias,
                    const float* pro_scale, const float* pro_shift, bool pro_silu, const float* residual,
                    float* out, int act = 0, float* gn_part = nullptr, const float* gn_add = nullptr);
// GroupNorm statistics gathered in the conv epilogue (gn_part of launch_conv_tc): possible when the
// output has c_out % 4 == 0 channels and maps of a multiple of 256 pixels (a 256-pixel statistics
// chunk is then two whole 128-row M tiles of one item); the scratch holds conv_gn_part_floats floats.
bool conv_gn_fusable(const ConvShape& s, int64_t c_out);
int64_t conv_gn_part_floats(const ConvShape& s, int64_t c_out);
// Folds the epilogue's per-(M tile, drain warp) sums into the per-(item, chunk, group) f64 partials
// that launch_gn_finalize takes (f32 per channel and chunk, then f64 over the group's channels).
void launch_gn_fold_tiles(mbx_ctx* ctx, const float* tile_part, int64_t n, int64_t hw, int64_t c, int64_t groups,
                          double* part);
// A tiled TMA map over f32 data: dims innermost first, strides in bytes for dims 1.., box in
// elements; reads outside the map fill with zeros.
void encode_tensor_map_f32(CUtensorMap* map, const float* base, int rank, const uint64_t* dims,
                           const uint64_t* strides, const uint32_t* box, bool swizzle128);
// Tensor maps for a param's hi / lo arrays (TMA, 128-byte swizzle).
void encode_param_tmaps(mbx_param* p);
// N tile for c_out output channels: 160 at most with f16 weights, 128 with f32 (3×TF32 keeps
// a lo weight tile too, so wider tiles would leave too few pipeline stages).
int choose_bn(int64_t c_out, bool f32_weights);

void launch_softmax_rows(mbx_ctx* ctx, float* x, int64_t rows, int64_t n, float scale, float flush);
void launch_split_to_param(mbx_ctx* ctx, const float* b, int64_t n, int64_t k, bool b_is_kn, mbx_param* p);
void launch_scale_add(mbx_ctx* ctx, const float* x, int64_t len, float mul, float add, float* out);

// λ layers (k_lambda.cu). lambda_content needs scratch: pmax and psum
// [items][chunks][k], plam [items][chunks][k][vd] with chunks = lambda_chunks(rows).
int64_t lambda_chunks(int64_t rows);
void launch_lambda_content(mbx_ctx* ctx, const float* keys, int64_t ks, const float* vals, int64_t vs,
                           int64_t items, int64_t rows, int64_t k, int64_t vd, float* pmax, float* plam,
                           float* psum, float* lam);
void launch_self_position(mbx_ctx* ctx, const float* q, const float* lam, const float* a, int64_t a_stride,
                          const float* v, int64_t v_stride, int64_t n, int64_t h, int64_t w, int64_t k, float* out);
void launch_cross_position(mbx_ctx* ctx, const float* q, const float* e_table, const float* lam, const float* vtab,
                           int64_t period, int64_t n, int64_t hw, int64_t k, float* out);

// Pipeline element work (k_pipeline.cu).
void launch_inpaint_prepare(mbx_ctx* ctx, const uint8_t* img, const uint8_t* mask, int64_t n, int64_t h, int64_t w,
                            int ch, float* images, uint8_t* bin, float* mask_lat, int32_t* nonempty);
void launch_vae_sample(mbx_ctx* ctx, const float* moments, const float* noise, int64_t pixels, float scale,
                       float* z);
void launch_latents_init(mbx_ctx* ctx, const float* z_pairs, const float* noise_init, const float* noise_offset,
                         int64_t n, int64_t hw, float offset_scale, float sa, float sb, bool pure, float* x);
void launch_unet_input(mbx_ctx* ctx, const float* x, const float* mask_lat, const float* z_pairs, int64_t n,
                       int64_t hw, int copies, float* out);
void launch_cfg_ddim(mbx_ctx* ctx, const float* eps, int64_t n, int64_t per, int copies, float guidance,
                     const float coef[4], float* x);
void launch_blur_lines(mbx_ctx* ctx, const uint8_t* in, uint8_t* out, int64_t lines, int64_t lines_per_item,
                       int64_t item_stride, int64_t line_stride, int64_t elem_stride, int len, int radius,
                       uint32_t ww, uint32_t fw, int passes);
// The square crop window around a mask bbox (reference CropPlan::new, src/imaging/crop.rs:30-62):
// the mask's long side plus half of it on each side, at least min(model side, image long
// side), at most the image long side; centred on the mask and shifted inside the image when
// it fits, else centred on the image (negative origin = padding).
struct CropWindow {
    int64_t x, y, side;
};

inline int64_t place_window(int64_t start, int64_t len, int64_t side, int64_t extent) {
    if (side <= extent) {
        const int64_t centred = (2 * start + len) / 2 - side / 2;
        return centred < 0 ? 0 : (centred > extent - side ? extent - side : centred);
    }
    return -((side - extent) / 2);
}

inline CropWindow crop_window(int64_t bx, int64_t by, int64_t bw, int64_t bh, int64_t width, int64_t height,
                              int64_t model_side) {
    const int64_t lng = bw > bh ? bw : bh;
    const int64_t img_long = width > height ? width : height;
    int64_t side = lng + 2 * (lng / 2);
    const int64_t floor_side = model_side < img_long ? model_side : img_long;
    if (side < floor_side) side = floor_side;
    if (side > img_long) side = img_long;
    return CropWindow{place_window(bx, bw, side, width), place_window(by, bh, side, height), side};
}

// The part of the window inside the image (CropPlan::source_rect, crop.rs:44-51).
inline mbx_rect source_rect(const CropWindow& c, int64_t width, int64_t height) {
    const int64_t x0 = c.x < 0 ? 0 : c.x, y0 = c.y < 0 ? 0 : c.y;
    const int64_t x1 = c.x + c.side < width ? c.x + c.side : width;
    const int64_t y1 = c.y + c.side < height ? c.y + c.side : height;
    return mbx_rect{(uint32_t)x0, (uint32_t)y0, (uint32_t)(x1 - x0), (uint32_t)(y1 - y0)};
}

// Imaging around the model window (k_imaging.cu).
void lanczos_table(int64_t in, int64_t out, int32_t* bounds, int32_t* coeffs, int64_t* ksize);
void launch_mask_dilate(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t stride, int64_t k,
                        uint8_t* scratch, uint8_t* out);
void launch_mask_bbox(mbx_ctx* ctx, const uint8_t* mask, int64_t n, int64_t h, int64_t w, int64_t stride,
                      int32_t* box);
void launch_window_to_model(mbx_ctx* ctx, const uint8_t* image, int64_t stride, int64_t channels,
                            const uint8_t* mask, int64_t mask_stride, int64_t origin_x, int64_t origin_y,
                            int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, int64_t model,
                            uint8_t* rgb, uint8_t* bin);
void launch_model_to_window(mbx_ctx* ctx, const float* rgb, int64_t n, int64_t model, int64_t side, uint8_t* out);
void launch_paste(mbx_ctx* ctx, uint8_t* image, int64_t n, int64_t stride, int64_t channels, const uint8_t* mask,
                  int64_t mask_stride, int64_t origin_x, int64_t origin_y, int64_t region_w, int64_t region_h,
                  int64_t width, int64_t height, int64_t win_x, int64_t win_y, int64_t side, const uint8_t* result,
                  uint32_t mode, const int32_t* active);
// Pillow's GaussianBlur(radius) of n single-channel h × w planes (3 box passes per axis).
void gaussian_blur(mbx_ctx* ctx, const uint8_t* in, int64_t n, int64_t h, int64_t w, float radius, uint8_t* scratch,
                   uint8_t* out);
void launch_broadcast_rows(mbx_ctx* ctx, const float* row, int64_t len, int64_t copies, float* out);
void launch_cfg_dpm(mbx_ctx* ctx, const float* eps, int64_t n, int64_t per, int copies, float guidance,
                    const float coef[5], int order, float* x, float* x0_prev);
void launch_feather_paste(mbx_ctx* ctx, const float* result, const uint8_t* blurred, uint8_t* image, int64_t pixels,
                          int64_t item_pixels, int ch, const int32_t* nonempty);

void launch_matmul_simt(mbx_ctx* ctx, float* c, const float* a, int64_t m, int64_t k, int64_t a_rs, int64_t a_cs,
                        const float* b, int64_t n, int64_t b_rs, int64_t b_cs, bool accumulate);

// Scoped pool allocation for per-call scratch (stream-ordered reuse).
struct PoolBuf {
    mbx_ctx* ctx = nullptr;
    void* p = nullptr;
    PoolBuf() = default;
    PoolBuf(mbx_ctx* c, size_t bytes) : ctx(c), p(c->pool->alloc(bytes)) {}
    PoolBuf(const PoolBuf&) = delete;
    PoolBuf& operator=(const PoolBuf&) = delete;
    PoolBuf(PoolBuf&& o) noexcept : ctx(o.ctx), p(o.p) { o.p = nullptr; }
    PoolBuf& operator=(PoolBuf&& o) noexcept {
        if (this != &o) {
            release();
            ctx = o.ctx;
            p = o.p;
            o.p = nullptr;
        }
        return *this;
    }
    ~PoolBuf() { release(); }
    void release() {
        if (p && ctx) {
            try {
                ctx->pool->free(p);
            } catch (...) {
            }
        }
        p = nullptr;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

// Launch-configuration helpers.
inline int grid_for(mbx_ctx* ctx, int64_t work_items, int per_block, int max_waves = 8) {
    int64_t blocks = (work_items + per_block - 1) / per_block;
    int64_t cap = (int64_t)ctx->sm_count * max_waves;
    if (blocks > cap) blocks = cap;
    return (int)(blocks < 1 ? 1 : blocks);
}

inline void after_launch(mbx_ctx* ctx, const char* what) {
    check_cuda(cudaGetLastError(), what);
    ctx->launches++;
}

}  // namespace mbx
