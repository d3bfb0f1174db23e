// Dense 1×1 and 3×3 convolutions as implicit GEMMs on the sm_100a tensor
// cores (tcgen05.mma, TMEM accumulator, TMA-fed weights).
//
// GEMM view: M = output pixels (n·ho·wo, raster order), N = c_out,
// K = taps·c_in walked in 32-channel chunks per tap (K chunk kc → tap
// kc / cin_chunks, channels 32·(kc % cin_chunks)…). This is the reference's
// im2col K order [ky, kx, c_in] (src/engine/conv.rs:145-165) without ever
// materialising the patch matrix, and replaces its Winograd path
// (src/engine/winograd.rs) for stride 1 / pad 1.
//
// CTA = one 128 × bn output tile at a time (bn ≤ 160); persistent: one CTA per
// SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... (N tile fastest) with
// every ring carried across tiles, so one tile's epilogue overlaps the next
// tile's loads and MMAs. 14 warps:
//   warps 0-3   loaders: gather the A tile (128 output pixels × 32 channels of
//               one tap) from NHWC global memory with 16-byte cp.async into a
//               raw staging ring (as many 16 KB slots as shared memory holds);
//               zero padding (src-size 0), stride and the nearest-2× upsample
//               are all address arithmetic here.
//   warps 10-13 converters: split each value v into hi = v (the tensor core
//               reads it truncated to TF32) and lo = v − trunc_TF32(v) (exact),
//               and tcgen05.st both into TMEM. An optional GroupNorm prologue
//               runs as its own pass before the kernel (launch_conv_tc).
//   warp 4      MMA issuer (one thread) + TMEM allocation; K chunks go out in
//               pairs, one barrier wait and one fence per 16 or 24 MMAs.
//   warp 5      TMA issuer (one thread) for the pre-split weight tiles.
//   warps 6-9   accumulator drain + epilogue (TMEM lane quadrant = warp % 4).
// One ring of K-chunk stages: stage s holds the weight tile (shared memory, by
// TMA) and the A tile (TMEM, by the converters) behind one full barrier (128
// converter arrivals + the TMA's expect-tx) and one empty barrier (the MMA's commit).
// Loading and converting are separate warps because the converters' waits on
// their staging slot would otherwise serialise with every global load in flight.
// Precision: f32 weights → 3×TF32 (a_lo·w_hi + a_hi·w_lo + a_hi·w_hi, weights
// split round-to-nearest at load), f16 weights (exact in TF32) → 2×TF32
// (a_lo·w + a_hi·w). The truncation split leaves at most the lo part's own
// truncation (≤ 2^-21 of |a|) per product. The tensor core
// adds each MMA's products into its f32 accumulator with truncation, which
// biases long sums toward zero (about 1e-4 relative at K = 11520; the error
// grows with the length of each unbroken sum). So K is cut into equal segments
// of at most 512 K-elements for f16 weights, 256 for f32 weights (a shorter K
// is one segment, so short-K tiles skip the fold and hold one accumulator): the MMA warp
// alternates between two TMEM accumulators, and the drain warps fold each
// finished segment into a running sum in shared memory with round-to-nearest
// f32 adds while the next segment accumulates (error then ≈ an f32 FMA loop).
// TMEM (512 columns) holds the two accumulators (2·bn) and the A stages
// (64 columns each: high parts, then low parts; lane = tile row) that the
// MMA reads directly (A from tensor memory), so the converted activations never
// pass through shared memory.
// The last segment is folded straight into the epilogue: + bias (+ residual)
// → global. Every mbarrier wait is bounded; on timeout the CTA records the
// error in the context's device error word, skips its stores, waits (bounded)
// until the bulk copies it issued have landed, and exits.
#include <cudaTypedefs.h>

#include <algorithm>

#include "mbx_device.cuh"
#include "mbx_internal.h"

namespace mbx {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;                  // f32 elements per 128-byte swizzle row
constexpr uint32_t A_BYTES = BM * BK * 4;  // 16 KB
constexpr int kThreads = 448;  // 14 warps; see the role map above
constexpr int kMinStgSlots = 3;  // raw A staging slots (16 KB each): at least, and at most
constexpr int kMaxStgSlots = 6;
// At most this many K chunks (of 32) per accumulator segment: f16 weights add two truncating MMAs
// per K step, f32 weights three, so their segments are shorter.
constexpr int kSegMaxChunksF16 = 16;
constexpr int kSegMaxChunksF32 = 8;

// Chunks per segment: K split into the fewest segments of at most the cap, as equal as possible.
template <bool F32W>
__device__ __forceinline__ int seg_chunks(int k_chunks) {
    constexpr int cap = F32W ? kSegMaxChunksF32 : kSegMaxChunksF16;
    const int n = (k_chunks + cap - 1) / cap;
    return (k_chunks + n - 1) / n;
}
constexpr int kMaxBn = 160;  // 2 · bn accumulator columns + A stages of 64 columns ≤ 512 (3 stages at 160)
constexpr int kMaxAStages = 4;
constexpr long long kWaitLimit = 4ll << 30;  // clock cycles (about 2 s)
constexpr int kMaxSmem = 232448;             // 227 KB opt-in limit per CTA

struct ConvArgs {
    const float* x;
    int64_t m_total;
    int h, w, c_in, ho, wo, stride, pad_t, pad_l, up;
    int cin_chunks, k_chunks;
    int flat;  // 1×1 conv: input pixel = output pixel (no padding, stride or upsample)
    int c_out, bn, n_tiles, stages, a_stages, tmem_cols;
    int stg_slots;  // raw A staging slots: as many as shared memory holds (more chunks in flight)
    // A-operand loads: 0 = cp.async gather by the loader warps; 1 = one TMA box per chunk from a
    // 2-D map [m_total][c_in] (1×1 convs); 2 = one TMA box {32 channels, a_bw, a_bh, 1} per chunk
    // and tap from a 4-D map [n][h][w][c_in] (3×3, stride 1, no upsample; the box's zero fill
    // outside the map is the padding).
    int a_tma, a_bw;
    // Epilogue by bulk tensor stores (single-segment tiles, float4 outputs): the drain adds bias
    // and residual (then the activation) while copying the accumulator into 32 × 32
    // swizzled blocks in shared memory, and one lane per warp stores them with TMA; the residual
    // blocks arrive by TMA beforehand (has_res).
    int tma_out, has_res;
    int64_t tiles;  // m tiles × n tiles
    const float* bias;
    const float* residual;
    float* out;
    int act;  // epilogue activation after bias and residual: 0 none, 1 SiLU
    // GroupNorm statistics of the output (null = off): per M tile and drain warp, the f32 sums of
    // y and y² over the warp's 32 rows per channel, y = out + gn_add[item] ([n][c_out] or null);
    // layout [m_tiles][4][2][c_out].
    float* gn_part;
    const float* gn_add;
    int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void record_timeout(int* err, int kernel, int site) {
    if (atomicCAS(err, 0, kErrWaitTimeout) == 0) {
        err[1] = kernel;
        err[2] = site;
    }
}

// Bounded wait for phase `parity` of `bar`. Returns false when the CTA is
// aborting (another role gave up) or after `limit` cycles, in which case
// the error is recorded and the abort flag raised.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int site, volatile int* abort_flag,
                                       bool honour_abort, long long limit = kWaitLimit, int kernel = kKConvTc) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (honour_abort && *abort_flag) return false;
        if (clock64() - t0 > limit) {
            record_timeout(err, kernel, site);
            *abort_flag = 1;
            return false;
        }
    }
}

// Abort path: waits, until the clock64 value `deadline`, for phase `parity` of `bar`, a phase
// armed by a bulk copy of this CTA; it completes once the copy has landed (and every other
// arrival the phase counts has been made).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, long long deadline, int* err, int site) {
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() > deadline) {
            record_timeout(err, kKConvTc, site);
            return;
        }
    }
}


__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Bulk tensor store of a shared-memory box (global coordinates {x, y}); out-of-range elements are
// not written. Completion is tracked per thread with the bulk-group counters.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// All this thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// All this thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_slot), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle,
// 8-row groups 1024 bytes apart (SBO), LBO unused (1), sm_100 version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_tf32(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// D (+)= A · Bᵀ with A (128 rows × 8 TF32, lane = row, one column per element) in TMEM.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
        "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The A-operand split: the tensor core reads an f32 operand as TF32 by dropping
// its 13 low mantissa bits, so the raw value serves as the high part and
// v − trunc_tf32(v) (exact in f32) as the low part. The two truncated parts
// carry v to within 2^-21 relative, one-signed per element; summed over
// products of either sign the error of a K-long dot product stays near 2^-22
// of Σ|a·w| (a CPU simulation at K up to 11520 gives ≤ 1e-8), far below the
// f32 accumulation error, and costs two integer/FP ops instead of two cvt.
__device__ __forceinline__ float tf32_split_lo(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xffffe000u); }

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// One arrival on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// GN: the epilogue also gathers GroupNorm statistics (args.gn_part); a separate instantiation, so the
// other convs' epilogue code is unchanged.
template <bool F32W, bool VEC4, bool FLAT, bool GN>
__global__ void __maxnreg__(128)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_hi, const __grid_constant__ CUtensorMap tmap_lo,
                   const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_out,
                   const __grid_constant__ CUtensorMap tmap_res, const ConvArgs args) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const int bn = args.bn;
    // One ring of K-chunk stages: stage s holds the weight tile (shared memory, by TMA) and the A
    // tile (TMEM, by the converters); a single full barrier (128 converter arrivals + the TMA's
    // expect-tx arrival) and a single empty barrier (the MMA commit) per stage, so the MMA thread
    // does one barrier wait per chunk.
    const int bstages = args.stages;
    const int astages = args.stages;
    const uint32_t b_bytes = (uint32_t)bn * 128u;
    const uint32_t bstage_bytes = (F32W ? 2 : 1) * b_bytes;
    const uint32_t stg_base = base + (uint32_t)bstages * bstage_bytes;  // raw A staging ring
    // Barriers: b_full/b_empty per weight stage, sfull/sempty per staging slot, a_full/a_empty per
    // TMEM A stage, acc_full/acc_empty per accumulator, final (abort path).
    // Running sums of the finished K segments: 128 rows × (bn + 4) floats (the 4-float pad
    // staggers rows across banks for the row-per-thread float4 accesses of the drain warps).
    const uint32_t sum_stride = (uint32_t)(bn + 4) * 4u;
    const int nstg = args.stg_slots;
    const uint32_t sum_base = stg_base + (uint32_t)nstg * A_BYTES;
    const uint32_t bars = sum_base + 128u * sum_stride;
    auto b_full_bar = [&](int s) { return bars + 8u * s; };
    auto b_empty_bar = [&](int s) { return bars + 8u * (bstages + s); };
    const uint32_t sbars = bars + 16u * bstages;
    auto sfull_bar = [&](int q) { return sbars + 8u * q; };
    auto sempty_bar = [&](int q) { return sbars + 8u * (kMaxStgSlots + q); };
    const uint32_t tbars = sbars + 16u * kMaxStgSlots;
    auto a_full_bar = [&](int a) { return b_full_bar(a); };
    auto a_empty_bar = [&](int a) { return b_empty_bar(a); };
    const uint32_t abars = tbars + 16u * kMaxAStages;
    auto acc_full_bar = [&](int b) { return abars + 8u * b; };
    auto acc_empty_bar = [&](int b) { return abars + 16u + 8u * b; };
    const uint32_t final_bar = abars + 32u;  // abort path: all issued MMAs retired
    const uint32_t misc = final_bar + 8u;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (misc - base));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (misc + 4 - base));
    volatile int* s_wfills = reinterpret_cast<volatile int*>(gbase + (misc + 8 - base));
    // Residual-block barriers of the bulk-store epilogue, one per drain warp.
    auto res_bar = [&](int qd) { return misc + 16u + 8u * qd; };
    // Fill counts for the abort path: arrivals this converter thread made on the stage full
    // barriers, weight tiles and A boxes the TMA issuers armed (a CTA's chunk count stays below
    // 2^31, checked at launch). Each role derives its count from its loop position when it leaves
    // the loop, so no counter stays live in the hot loops.
    int conv_fills = 0, w_fills = 0, a_fills = 0;
    // Bulk-store epilogue, drain lane 0: a residual load in flight and the phase it completes.
    int res_pending = 0;
    uint32_t res_phase = 0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Converters: warps 10-13, plus warps 0-3 for 1×1 convs with TMA-fed A rows (the loader warps are
    // free then; short-K 1×1 tiles gain from the faster hand-off, long 3×3 ones do not); with
    // eight, each thread converts half of its row's 32 channels.
    const bool split = args.a_tma == 1;
    const int conv_threads = split ? 256 : 128;
    const bool is_converter = warp >= 10 || (split && warp < 4);
    const int K = args.k_chunks;
    const int seg_len = seg_chunks<F32W>(K);
    const int nseg = (K + seg_len - 1) / seg_len;
    // Persistent CTA: tiles blockIdx.x, blockIdx.x + gridDim.x, ... (N tile fastest, so the CTAs
    // in flight share A rows through L2). Every ring keeps its position and phase across tiles,
    // so the next tile's loads and MMAs overlap this tile's epilogue.
    const int64_t tiles = args.tiles;
    // Fill counts of a role that walked all of this CTA's tiles, or stopped at chunk kc of tile t.
    auto all_fills = [&]() { return (int)((tiles - blockIdx.x + gridDim.x - 1) / gridDim.x) * K; };
    auto fills_at = [&](int64_t t, int kc) { return (int)((t - blockIdx.x) / gridDim.x) * K + kc; };
    auto tile_m0 = [&](int64_t t) { return (t / args.n_tiles) * (int64_t)BM; };
    auto tile_n0 = [&](int64_t t) { return (int)(t % args.n_tiles) * bn; };
    // TMEM columns: accumulators [0, 2·bn), A stage a at 2·bn + 64·a (32 columns of TF32
    // high parts, then 32 of low parts; lane = tile row).
    auto a_col = [&](int a) { return (uint32_t)(2 * bn + 64 * a); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < bstages; ++s) {
            mbar_init(b_full_bar(s), (uint32_t)conv_threads + 1u);
            mbar_init(b_empty_bar(s), 1);
        }
        for (int q = 0; q < nstg; ++q) {
            mbar_init(sfull_bar(q), args.a_tma ? 1 : 128);
            mbar_init(sempty_bar(q), (uint32_t)conv_threads);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full_bar(b), 1);
            mbar_init(acc_empty_bar(b), 128);
        }
        mbar_init(final_bar, 1);
        for (int qd = 0; qd < 4; ++qd) mbar_init(res_bar(qd), 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 4) {
        tmem_alloc(smem_u32(tmem_slot), 512u);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int hi_img = args.h << args.up, wi_img = args.w << args.up;
    const int64_t hw_out = (int64_t)args.ho * args.wo;
    // Row geometry: item index and the top-left input tap packed as (iy0 << 16) | (ix0 & 0xffff);
    // rows past the end get an iy0 far outside the image, so every tap reads as padding.
    auto row_geo = [&](int64_t m0, int r, int& pb, int& geo) {
        const int64_t m = m0 + r;
        const bool valid = m < args.m_total;
        const int64_t mm = valid ? m : 0;
        const int64_t b = mm / hw_out;
        const int64_t rem = mm - b * hw_out;
        const int oy = (int)(rem / args.wo);
        const int ox = (int)(rem - (int64_t)oy * args.wo);
        pb = (int)b;
        const int iy0 = valid ? oy * args.stride - args.pad_t : -30000;
        const int ix0 = ox * args.stride - args.pad_l;
        geo = (int)(((uint32_t)iy0 << 16) | ((uint32_t)ix0 & 0xffffu));
    };
    // Spatial validity and input pixel index of row r's tap (ky, kx).
    auto tap_pixel = [&](int64_t m0, int r, int pb, int geo, int ky, int kx, bool& ok) -> int64_t {
        if constexpr (FLAT) {
            const int64_t pix = m0 + r;
            ok = pix < args.m_total;
            return pix;
        } else {
            const int iy = (geo >> 16) + ky, ix = (int)(int16_t)(geo & 0xffff) + kx;
            ok = iy >= 0 && iy < hi_img && ix >= 0 && ix < wi_img;
            return ((int64_t)pb * args.h + (iy >> args.up)) * args.w + (ix >> args.up);
        }
    };

    if (warp < 4 && !args.a_tma) {
        // ------------------------------------------------------------ loaders
        // cp.async 16-byte copies (zero-filled at padding) into the raw staging ring;
        // completion is signalled per thread with cp.async.mbarrier.arrive, so a loader
        // never waits on its data and keeps up to nstg chunks in flight.
        const int tid = threadIdx.x;
        const int j = tid & 7;       // 16-byte chunk (4 channels) of the 128-byte row
        const int rbase = tid >> 3;  // rows rbase + 16·i
        int q = 0, qphase = 0;
        bool live = true;
        for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
            const int64_t m0 = tile_m0(t);
            int pb[8], geo[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                pb[i] = 0;
                geo[i] = 0;
                if constexpr (!FLAT) row_geo(m0, rbase + 16 * i, pb[i], geo[i]);
            }
            int tap = 0, cchunk = 0;
            for (int kc = 0; kc < K; ++kc) {
                if (!mbar_wait(sempty_bar(q), (uint32_t)(qphase ^ 1), args.err, 8, abort_flag, true)) {
                    live = false;
                    break;
                }
                const int c0 = cchunk * BK + 4 * j;
                const int ky = tap / 3, kx = tap - 3 * (tap / 3);
                const uint32_t stg = stg_base + (uint32_t)q * A_BYTES;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = rbase + 16 * i;
                    const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(j ^ (r & 7)) << 4);
                    bool ok;
                    const int64_t pix = tap_pixel(m0, r, pb[i], geo[i], ky, kx, ok);
                    if constexpr (VEC4) {
                        const bool in = ok && c0 < args.c_in;
                        cp_async_16(stg + off,
                                    in ? (const void*)(args.x + pix * args.c_in + c0) : (const void*)args.x,
                                    in ? 16u : 0u);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const bool in = ok && c0 + e < args.c_in;
                            cp_async_4(stg + off + 4u * e,
                                       in ? (const void*)(args.x + pix * args.c_in + c0 + e) : (const void*)args.x,
                                       in ? 4u : 0u);
                        }
                    }
                }
                cp_async_mbar_arrive(sfull_bar(q));
                if (++q == nstg) {
                    q = 0;
                    qphase ^= 1;
                }
                if (++cchunk == args.cin_chunks) {
                    cchunk = 0;
                    ++tap;
                }
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight at exit (abort path)
    } else if (is_converter) {
        // ------------------------------------------------------------ converters
        // One tile row per thread (its TMEM lane): staging row (zeros at padding taps; channel
        // padding beyond c_in meets zero weights) → TF32 high and low parts written to the A stage
        // in TMEM. With eight converter warps, warps 10-13 take channels 0-15 and warps 0-3 16-31.
        const int qd = warp & 3;
        const int half = warp < 4 ? 1 : 0;
        const int r = qd * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
        int q = 0, qphase = 0, a = 0, aphase = 0;
        bool live = true;
        for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
            for (int kc = 0; kc < K; ++kc) {
                if (!mbar_wait(sfull_bar(q), (uint32_t)qphase, args.err, 9, abort_flag, true) ||
                    !mbar_wait(a_empty_bar(a), (uint32_t)(aphase ^ 1), args.err, 1, abort_flag, true)) {
                    live = false;
                    conv_fills = fills_at(t, kc);
                    break;
                }
                const uint32_t stg = stg_base + (uint32_t)q * A_BYTES + (uint32_t)r * 128u;
                // Loads 4·NV channels (16-byte units j0 …) of the row, stores the high parts, releases
                // the staging slot and stores the low parts at column c0.
                auto convert = [&](auto nv_tag, int j0, uint32_t c0) {
                    constexpr int NV = decltype(nv_tag)::value;
                    float v[4 * NV];
#pragma unroll
                    for (int jj = 0; jj < NV; ++jj) {
                        const float4 f = ld_shared_v4(stg + ((uint32_t)((j0 + jj) ^ (r & 7)) << 4));
                        v[4 * jj] = f.x;
                        v[4 * jj + 1] = f.y;
                        v[4 * jj + 2] = f.z;
                        v[4 * jj + 3] = f.w;
                    }
                    if (!args.a_tma) mbar_arrive(sempty_bar(q));  // the staging row is in registers
                    // High part: the value itself (the tensor core reads its TF32 truncation); low
                    // part: v − trunc_tf32(v), exact in f32 (again read truncated).
                    if constexpr (NV == 8) tmem_st32(lane_base + a_col(a) + c0, v);
                    else tmem_st16(lane_base + a_col(a) + c0, v);  // v stays untouched until the wait
                    float lo[4 * NV];
#pragma unroll
                    for (int e = 0; e < 4 * NV; ++e) lo[e] = tf32_split_lo(v[e]);
                    if (args.a_tma) {
                        // The next TMA write into this slot is an async-proxy access: the row's
                        // generic loads (complete here, their values are in use) are ordered before it.
                        fence_proxy_async_smem();
                        mbar_arrive(sempty_bar(q));
                    }
                    if constexpr (NV == 8) tmem_st32(lane_base + a_col(a) + 32u + c0, lo);
                    else tmem_st16(lane_base + a_col(a) + 32u + c0, lo);
                };
                if (split)
                    convert(std::integral_constant<int, 4>{}, 4 * half, 16u * (uint32_t)half);
                else
                    convert(std::integral_constant<int, 8>{}, 0, 0u);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(a_full_bar(a));
                if (++q == nstg) {
                    q = 0;
                    qphase ^= 1;
                }
                if (++a == astages) {
                    a = 0;
                    aphase ^= 1;
                }
            }
        }
        if (live) conv_fills = all_fills();
    } else if (warp == 4) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            // The tensor pipe queues almost nothing ahead, so every cycle this thread spends
            // between MMAs is a pipe bubble: ring positions and phases advance incrementally
            // (no division), descriptors step by their 16-byte address units.
            const uint32_t idesc = idesc_tf32(bn);
            // Issues one K chunk (4 K-steps of 8) from stage st into accumulator d.
            auto issue = [&](int st, uint32_t d, bool first) {
                const uint32_t ah = tmem + a_col(st), al = ah + 32u;
                const uint32_t b_hi = base + (uint32_t)st * bstage_bytes;
                const uint64_t bdh0 = sw128_desc(b_hi);
                const uint64_t bdl0 = sw128_desc(b_hi + b_bytes);
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint64_t bdh = bdh0 + (uint64_t)(2 * kk);  // + kk·32 bytes
                    const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
                    const uint32_t ko = (uint32_t)kk * 8u;
                    if constexpr (F32W) {
                        const uint64_t bdl = bdl0 + (uint64_t)(2 * kk);
                        mma_tf32_ts(d, al + ko, bdh, idesc, acc);
                        mma_tf32_ts(d, ah + ko, bdl, idesc, 1u);
                        mma_tf32_ts(d, ah + ko, bdh, idesc, 1u);
                    } else {
                        mma_tf32_ts(d, al + ko, bdh, idesc, acc);
                        mma_tf32_ts(d, ah + ko, bdh, idesc, 1u);
                    }
                }
            };
            // Chunks go out in pairs (one synchronisation per 16 or 24 MMAs); a segment's odd
            // last chunk goes alone. With only three stages (160-wide tiles, f32 weights) one chunk
            // at a time: a pair would leave the converters a single stage of head room (1×1 convs
            // at 160 wide 3-6 % faster, f32-weight 3×3 4.5 %).
            int s = 0, sphase = 0, seg = 0;
            bool live = true;
            for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
                int kin = 0;
                for (int kc = 0; kc < K;) {
                    const int b = seg & 1;
                    const bool seg_first = kin == 0;
                    const int left = min(seg_len - kin, K - kc);
                    const int g = (left >= 2 && bstages >= 4) ? 2 : 1;
                    const int s1 = s + 1 == bstages ? 0 : s + 1;
                    const int ph1 = s + 1 == bstages ? sphase ^ 1 : sphase;
                    if (seg_first &&
                        !mbar_wait(acc_empty_bar(b), ((seg >> 1) & 1) ^ 1, args.err, 5, abort_flag, true)) {
                        live = false;
                        break;
                    }
                    if (!mbar_wait(b_full_bar(s), (uint32_t)sphase, args.err, 3, abort_flag, true) ||
                        (g == 2 && !mbar_wait(b_full_bar(s1), (uint32_t)ph1, args.err, 3, abort_flag, true))) {
                        live = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(b * bn);
                    issue(s, d, seg_first);
                    if (g == 2) issue(s1, d, false);
                    mma_commit(b_empty_bar(s));  // frees the stage's weight tile and A tile
                    if (g == 2) mma_commit(b_empty_bar(s1));
                    kc += g;
                    kin += g;
                    if (kin == seg_len || kc == K) {
                        mma_commit(acc_full_bar(b));
                        kin = 0;
                        ++seg;
                    }
                    if (g == 2) {
                        s = s1 + 1 == bstages ? 0 : s1 + 1;
                        sphase = s1 + 1 == bstages ? ph1 ^ 1 : ph1;
                    } else {
                        s = s1;
                        sphase = ph1;
                    }
                }
            }
            if (*abort_flag) {
                // Do not let TMEM be freed under MMAs that are still running.
                mma_commit(final_bar);
                mbar_wait(final_bar, 0, args.err, 7, abort_flag, false);
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ------------------------------------------------------------ TMA issuers
        // Lane 1: the A boxes (one 16 KB box per K chunk into the staging ring; the 128-byte
        // swizzle gives the same layout the cp.async gather writes). Lane 0: the weight tiles.
        if (lane == 1 && args.a_tma) {
            int q = 0, qphase = 0;
            bool live = true;
            for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
                const int64_t m0 = tile_m0(t);
                int item = 0, y0 = 0, x0 = 0;
                if (args.a_tma == 2) {
                    item = (int)(m0 / hw_out);
                    const int64_t rem = m0 - (int64_t)item * hw_out;
                    y0 = (int)(rem / args.wo);
                    x0 = (int)(rem - (int64_t)y0 * args.wo);
                }
                int tap = 0, cchunk = 0;
                for (int kc = 0; kc < K; ++kc) {
                    if (!mbar_wait(sempty_bar(q), (uint32_t)(qphase ^ 1), args.err, 8, abort_flag, true)) {
                        live = false;
                        a_fills = fills_at(t, kc);
                        break;
                    }
                    const uint32_t stg = stg_base + (uint32_t)q * A_BYTES;
                    mbar_arrive_expect_tx(sfull_bar(q), A_BYTES);
                    if (args.a_tma == 1) {
                        tma_load_2d(stg, &tmap_a, cchunk * BK, (int)m0, sfull_bar(q));
                    } else {
                        const int ky = tap / 3, kx = tap - 3 * (tap / 3);
                        tma_load_4d(stg, &tmap_a, cchunk * BK, x0 + kx - args.pad_l, y0 + ky - args.pad_t, item,
                                    sfull_bar(q));
                    }
                    if (++q == nstg) {
                        q = 0;
                        qphase ^= 1;
                    }
                    if (++cchunk == args.cin_chunks) {
                        cchunk = 0;
                        ++tap;
                    }
                }
            }
            if (live) a_fills = all_fills();
        }
        if (lane == 0) {
            int s = 0, sphase = 0;
            bool live = true;
            for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
                const int n0 = tile_n0(t);
                for (int kc = 0; kc < K; ++kc) {
                    if (!mbar_wait(b_empty_bar(s), (uint32_t)(sphase ^ 1), args.err, 4, abort_flag, true)) {
                        live = false;
                        w_fills = fills_at(t, kc);
                        break;
                    }
                    const uint32_t b_hi = base + (uint32_t)s * bstage_bytes;
                    mbar_arrive_expect_tx(b_full_bar(s), bstage_bytes);
                    tma_load_2d(b_hi, &tmap_hi, kc * BK, n0, b_full_bar(s));
                    if constexpr (F32W) tma_load_2d(b_hi + b_bytes, &tmap_lo, kc * BK, n0, b_full_bar(s));
                    if (++s == bstages) {
                        s = 0;
                        sphase ^= 1;
                    }
                }
            }
            if (live) w_fills = all_fills();
            *s_wfills = w_fills;
        }
        __syncwarp();
    } else if (warp >= 6 && warp < 10) {
        // ------------------------------------------------------------ drain + epilogue
        const int qd = warp & 3;  // TMEM lane quadrant this warp may access
        const int row = qd * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(qd * 32) << 16);
        const uint32_t srow = sum_base + (uint32_t)row * sum_stride;
        if (args.tma_out) {
            // Bulk-store epilogue. This warp's bn/32 blocks of 32 rows × 32 columns sit in the sum
            // buffer (4 KB each, 128-byte swizzle: float4 v of row r at r·128 + ((v ^ (r & 7))·16),
            // the layout of a {32, 32} TMA box). A tile's residual blocks are loaded into them by TMA
            // while the tile accumulates; the drain adds bias and residual (then the activation)
            // while copying its row out of TMEM, releases the accumulator, and lane 0 stores the
            // blocks with TMA (rows and columns outside the output are clipped by the tensor map).
            const int nblk = bn / 32;
            const uint32_t wreg = sum_base + (uint32_t)(qd * nblk) * 4096u;
            const uint32_t rbar = res_bar(qd);
            const uint32_t rrow = (uint32_t)lane * 128u;
            const int x7 = lane & 7;
            auto issue_res = [&](int64_t t) {  // lane 0
                const int64_t m0 = tile_m0(t);
                const int n0 = tile_n0(t);
                int live_blocks = 0;
                for (int cb = 0; cb < nblk; ++cb) live_blocks += n0 + 32 * cb < args.c_out ? 1 : 0;
                mbar_arrive_expect_tx(rbar, (uint32_t)live_blocks * 4096u);
                for (int cb = 0; cb < nblk; ++cb)
                    if (n0 + 32 * cb < args.c_out)
                        tma_load_2d(wreg + (uint32_t)cb * 4096u, &tmap_res, n0 + 32 * cb, (int)(m0 + 32 * qd), rbar);
                res_pending = 1;
            };
            bool live = true;
            int gseg = 0;  // accumulator segments drained so far (the MMA warp's count)
            if (args.has_res && lane == 0 && (int64_t)blockIdx.x < tiles) issue_res(blockIdx.x);
            for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
                const int64_t m0 = tile_m0(t);
                const int n0 = tile_n0(t);
                // The tile's bias, loaded before the accumulator wait: lane l holds float4 groups l and
                // l + 32 of the tile's columns (bn ≤ 256); the drain shuffles each out when it is needed.
                float4 bias_q[2], gadd_q[2];
#pragma unroll
                for (int sq = 0; sq < 2; ++sq) {
                    const int c = n0 + 4 * (lane + 32 * sq);
                    const bool ok = 4 * (lane + 32 * sq) < bn && c < args.c_out;
                    bias_q[sq] = args.bias && ok ? __ldg(reinterpret_cast<const float4*>(args.bias + c))
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
                    // GroupNorm add of the tile's item (its rows all belong to one item).
                    gadd_q[sq] = GN && args.gn_add && ok
                                     ? __ldg(reinterpret_cast<const float4*>(args.gn_add + (m0 / hw_out) * args.c_out + c))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                bool seg_live = true;
                for (int seg = 0; seg < nseg; ++seg, ++gseg) {
                    const int b = gseg & 1;
                    const bool first = seg == 0, last = seg + 1 == nseg;
                    if (!mbar_wait(acc_full_bar(b), (uint32_t)((gseg >> 1) & 1), args.err, 6, abort_flag, true)) {
                        seg_live = false;
                        break;
                    }
                    tc_fence_after();
                    if (first) {
                        if (args.has_res) {
                            // The previous tile's stores finished reading the blocks before this load
                            // was issued.
                            if (!mbar_wait(rbar, res_phase, args.err, 13, abort_flag, true)) {
                                seg_live = false;
                                break;
                            }
                            res_phase ^= 1u;
                            res_pending = 0;
                        } else {
                            if (lane == 0) bulk_wait_read_all();  // the previous tile's stores have read the blocks
                            __syncwarp();
                        }
                    }
                    // One 32-column block of this thread's row into the block: the first segment adds
                    // bias (+ residual) to its sum, later ones fold theirs into the running value, the
                    // last one then applies the activation. Both choices are template arguments: a
                    // runtime test inside the loop would be predicated into every block.
                    auto drain_block = [&](auto first_tag, auto act_tag, int cb) {
                        constexpr bool FIRST = decltype(first_tag)::value;
                        constexpr bool ACT = decltype(act_tag)::value;
                        float acc[32];
                        tmem_ld32(lane_base + (uint32_t)(b * bn + 32 * cb), acc);
                        const uint32_t blk = wreg + (uint32_t)cb * 4096u + rrow;
                        const float4 bsel = cb < 4 ? bias_q[0] : bias_q[1];  // groups 8·cb … 8·cb + 7
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            const uint32_t addr = blk + ((uint32_t)(v ^ x7) << 4);
                            float4 pre;
                            if constexpr (FIRST) {
                                const int src = (8 * cb + v) & 31;
                                pre = make_float4(__shfl_sync(0xffffffffu, bsel.x, src),
                                                  __shfl_sync(0xffffffffu, bsel.y, src),
                                                  __shfl_sync(0xffffffffu, bsel.z, src),
                                                  __shfl_sync(0xffffffffu, bsel.w, src));
                                if (args.has_res) {
                                    const float4 r4 = ld_shared_v4(addr);
                                    pre = make_float4(r4.x + pre.x, r4.y + pre.y, r4.z + pre.z, r4.w + pre.w);
                                }
                            } else {
                                pre = ld_shared_v4(addr);  // the running value
                            }
                            float4 o = make_float4(pre.x + acc[4 * v], pre.y + acc[4 * v + 1], pre.z + acc[4 * v + 2],
                                                   pre.w + acc[4 * v + 3]);
                            if constexpr (ACT)
                                o = make_float4(dev_silu(o.x), dev_silu(o.y), dev_silu(o.z), dev_silu(o.w));
                            st_shared_v4(addr, o.x, o.y, o.z, o.w);
                        }
                    };
                    const bool act_now = last && args.act;
                    for (int cb = 0; cb < nblk; ++cb) {
                        if (first) {
                            if (act_now)
                                drain_block(std::true_type{}, std::true_type{}, cb);
                            else
                                drain_block(std::true_type{}, std::false_type{}, cb);
                        } else {
                            if (act_now)
                                drain_block(std::false_type{}, std::true_type{}, cb);
                            else
                                drain_block(std::false_type{}, std::false_type{}, cb);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(acc_empty_bar(b));
                }
                if (!seg_live) {
                    live = false;
                    break;
                }
                fence_proxy_async_smem();  // the blocks' writes, before the bulk stores read them
                __syncwarp();
                if (lane == 0) {
                    for (int cb = 0; cb < nblk; ++cb)
                        if (n0 + 32 * cb < args.c_out)
                            tma_store_2d(&tmap_out, n0 + 32 * cb, (int)(m0 + 32 * qd), wreg + (uint32_t)cb * 4096u);
                    bulk_commit();
                }
                if constexpr (GN) {
                    // GroupNorm statistics of y = out + add over this warp's 32 rows, read back from the
                    // blocks while the stores run: lane l takes float4 group l % 8 of rows 4i + l / 8,
                    // two shuffles fold the lanes sharing those columns (a fixed order), and lanes 0-7
                    // write the warp's sums: [M tile][warp][2][c_out]. Fusable shapes have whole M tiles.
                    const int j = lane & 7;
                    for (int cb = 0; cb < nblk; ++cb) {
                        const int col = n0 + 32 * cb + 4 * j;
                        const float4 gsel = cb < 4 ? gadd_q[0] : gadd_q[1];
                        const int src = (8 * cb + j) & 31;
                        const float4 g = make_float4(__shfl_sync(0xffffffffu, gsel.x, src),
                                                     __shfl_sync(0xffffffffu, gsel.y, src),
                                                     __shfl_sync(0xffffffffu, gsel.z, src),
                                                     __shfl_sync(0xffffffffu, gsel.w, src));
                        float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), gq = gs;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = 4 * i + (lane >> 3);
                            const float4 o = ld_shared_v4(wreg + (uint32_t)cb * 4096u + (uint32_t)r * 128u +
                                                          ((uint32_t)(j ^ (r & 7)) << 4));
                            const float4 y = make_float4(o.x + g.x, o.y + g.y, o.z + g.z, o.w + g.w);
                            gs = make_float4(gs.x + y.x, gs.y + y.y, gs.z + y.z, gs.w + y.w);
                            gq = make_float4(fmaf(y.x, y.x, gq.x), fmaf(y.y, y.y, gq.y), fmaf(y.z, y.z, gq.z),
                                             fmaf(y.w, y.w, gq.w));
                        }
#pragma unroll
                        for (int o = 8; o <= 16; o <<= 1) {
                            gs.x += __shfl_xor_sync(0xffffffffu, gs.x, o);
                            gs.y += __shfl_xor_sync(0xffffffffu, gs.y, o);
                            gs.z += __shfl_xor_sync(0xffffffffu, gs.z, o);
                            gs.w += __shfl_xor_sync(0xffffffffu, gs.w, o);
                            gq.x += __shfl_xor_sync(0xffffffffu, gq.x, o);
                            gq.y += __shfl_xor_sync(0xffffffffu, gq.y, o);
                            gq.z += __shfl_xor_sync(0xffffffffu, gq.z, o);
                            gq.w += __shfl_xor_sync(0xffffffffu, gq.w, o);
                        }
                        if (lane < 8 && col < args.c_out) {
                            float* dst = args.gn_part + ((m0 / BM) * 4 + qd) * 2 * (int64_t)args.c_out + col;
                            *reinterpret_cast<float4*>(dst) = gs;
                            *reinterpret_cast<float4*>(dst + args.c_out) = gq;
                        }
                    }
                }
                if (lane == 0) {
                    const int64_t tn = t + gridDim.x;
                    if (args.has_res && tn < tiles) {
                        bulk_wait_read_all();
                        issue_res(tn);
                    }
                }
                __syncwarp();
            }
            if (lane == 0) bulk_wait_all();
        } else {
            const bool vec_out = (args.c_out & 3) == 0;
            // Transposed (coalesced) stores for float4 outputs; a SiLU epilogue keeps one row per thread
            // (inside the UNet its transposed form ran 22 % slower) unless statistics are gathered.
            const bool transpose = vec_out && (!args.act || GN);
            int gseg = 0;
            bool live = true;
            // Transposed epilogue: lane l owns the float4 column group l % 8 of rows 4i + l / 8 of each
            // 32 × 32 block. Its bias and GroupNorm-add operands for a block are loaded one block ahead
            // (the first block's before the accumulator wait), so no block waits out their latency
            // (loaded per block, that wait cost the short-K 1×1 convs up to 16 %).
            const int tj = lane & 7;
            struct BlockIn {
                float4 bias, gadd;
            };
            auto load_block = [&](int64_t t, int n0, int cc, BlockIn& in) {
                const int col = n0 + cc + 4 * tj;
                const bool ok = n0 + cc < args.c_out && col < args.c_out;  // c_out % 4 == 0: whole float4s
                const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                in.bias = args.bias && ok ? __ldg(reinterpret_cast<const float4*>(args.bias + col)) : z;
                in.gadd = GN && args.gn_add && ok
                              ? __ldg(reinterpret_cast<const float4*>(args.gn_add + (tile_m0(t) / hw_out) * args.c_out + col))
                              : z;
            };
            for (int64_t t = blockIdx.x; live && t < tiles; t += gridDim.x) {
                const int64_t m = tile_m0(t) + row;
                const int n0 = tile_n0(t);
                BlockIn cur;
                for (int seg = 0; seg < nseg; ++seg, ++gseg) {
                    const int b = gseg & 1;
                    const bool last = seg + 1 == nseg;
                    if (last && transpose) load_block(t, n0, 0, cur);
                    if (!mbar_wait(acc_full_bar(b), (gseg >> 1) & 1, args.err, 6, abort_flag, true)) {
                        live = false;
                        break;
                    }
                    tc_fence_after();
                    for (int cc = 0; cc < bn; cc += 32) {
                        float acc[32];
                        tmem_ld32(lane_base + (uint32_t)(b * bn + cc), acc);
                        if (seg > 0) {
#pragma unroll
                            for (int v = 0; v < 8; ++v) {
                                const float4 r4 = ld_shared_v4(srow + (uint32_t)(cc + 4 * v) * 4u);
                                acc[4 * v] = r4.x + acc[4 * v];
                                acc[4 * v + 1] = r4.y + acc[4 * v + 1];
                                acc[4 * v + 2] = r4.z + acc[4 * v + 2];
                                acc[4 * v + 3] = r4.w + acc[4 * v + 3];
                            }
                        }
                        if (!last || transpose) {
#pragma unroll
                            for (int v = 0; v < 8; ++v)
                                st_shared_v4(srow + (uint32_t)(cc + 4 * v) * 4u, acc[4 * v], acc[4 * v + 1],
                                             acc[4 * v + 2], acc[4 * v + 3]);
                            continue;
                        }
                        if (m >= args.m_total) continue;
                        const int nb = n0 + cc;
                        if (nb >= args.c_out) continue;
                        // One row per thread: float4 stores (SiLU epilogues), or scalar stores for output
                        // widths that are not a multiple of 4 (the VAE's 3-channel conv_out).
                        float* dst = args.out + m * args.c_out + nb;
                        const float* res = args.residual ? args.residual + m * args.c_out + nb : nullptr;
                        if (vec_out && nb + 32 <= args.c_out) {
#pragma unroll
                            for (int v = 0; v < 8; ++v) {
                                float4 pre = args.bias ? __ldg(reinterpret_cast<const float4*>(args.bias + nb) + v)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                                if (res) {
                                    const float4 r4 = __ldg(reinterpret_cast<const float4*>(res) + v);
                                    pre = make_float4(r4.x + pre.x, r4.y + pre.y, r4.z + pre.z, r4.w + pre.w);
                                }
                                float4 o4 = make_float4(pre.x + acc[4 * v], pre.y + acc[4 * v + 1],
                                                        pre.z + acc[4 * v + 2], pre.w + acc[4 * v + 3]);
                                if (args.act)
                                    o4 = make_float4(dev_silu(o4.x), dev_silu(o4.y), dev_silu(o4.z), dev_silu(o4.w));
                                reinterpret_cast<float4*>(dst)[v] = o4;
                            }
                        } else {
                            const int lim = min(32, args.c_out - nb);
#pragma unroll
                            for (int i = 0; i < 32; ++i) {
                                if (i < lim) {
                                    float pre = args.bias ? __ldg(args.bias + nb + i) : 0.0f;
                                    if (res) pre = __ldg(res + i) + pre;
                                    const float o = pre + acc[i];
                                    dst[i] = args.act ? dev_silu(o) : o;
                                }
                            }
                        }
                    }
                    // The accumulator has been read (into registers, or into the sum buffer for folds
                    // and transposed epilogues): the MMA warp may start the segment after next in it
                    // while the stores below run.
                    tc_fence_before();
                    mbar_arrive(acc_empty_bar(b));
                    if (!last || !transpose) continue;
                    __syncwarp();  // the rows written above are read by other lanes below
                    for (int cc = 0; cc < bn; cc += 32) {
                        // Transposed stores: the warp's 32 × 32 block goes through this row's slot
                        // of the (segment) sum buffer, so each store instruction writes four
                        // whole 128-byte row pieces instead of 32 scattered 16-byte ones. The row stride
                        // (bn + 4 words, ≡ 4 mod 32) keeps both passes free of bank conflicts.
                        BlockIn nxt;
                        if (cc + 32 < bn) load_block(t, n0, cc + 32, nxt);
                        const int nb = n0 + cc;
                        if (nb < args.c_out) {
                            const int col = nb + 4 * tj;
                            const bool col_ok = col < args.c_out;
                            const int64_t m_base = tile_m0(t) + qd * 32 + (lane >> 3);
                            float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), gq = gs;
                            // All eight shared loads, then all eight residual loads, then the stores: a
                            // residual load placed after a store would wait out its whole latency.
                            float4 a4[8], r4[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                a4[i] = ld_shared_v4(sum_base + (uint32_t)(qd * 32 + 4 * i + (lane >> 3)) * sum_stride +
                                                     (uint32_t)(cc + 4 * tj) * 4u);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const int64_t mr = m_base + 4 * i;
                                r4[i] = args.residual && col_ok && mr < args.m_total
                                            ? __ldg(reinterpret_cast<const float4*>(args.residual + mr * args.c_out + col))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
                            }
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const int64_t mr = m_base + 4 * i;
                                if (mr >= args.m_total || !col_ok) continue;
                                const float4 a = a4[i];
                                const float4 pre = make_float4(r4[i].x + cur.bias.x, r4[i].y + cur.bias.y,
                                                               r4[i].z + cur.bias.z, r4[i].w + cur.bias.w);
                                float4 o4 = make_float4(pre.x + a.x, pre.y + a.y, pre.z + a.z, pre.w + a.w);
                                // Only statistics-gathering convs reach this path with an activation (see
                                // `transpose`). A runtime-only test let the compiler predicate the SiLU
                                // instead of branching: 32 exp/divide pairs per block on every conv.
                                if (GN && args.act)
                                    o4 = make_float4(dev_silu(o4.x), dev_silu(o4.y), dev_silu(o4.z), dev_silu(o4.w));
                                *reinterpret_cast<float4*>(args.out + mr * args.c_out + col) = o4;
                                if constexpr (GN) {
                                    const float4 g = cur.gadd;
                                    const float4 y = make_float4(o4.x + g.x, o4.y + g.y, o4.z + g.z, o4.w + g.w);
                                    gs = make_float4(gs.x + y.x, gs.y + y.y, gs.z + y.z, gs.w + y.w);
                                    gq = make_float4(fmaf(y.x, y.x, gq.x), fmaf(y.y, y.y, gq.y), fmaf(y.z, y.z, gq.z),
                                                     fmaf(y.w, y.w, gq.w));
                                }
                            }
                            if constexpr (GN) {
                                // Lanes j, j + 8, j + 16, j + 24 hold the same columns: fold them (a fixed
                                // order, so results do not depend on timing), then lanes 0-7 write the
                                // warp's sums for their four channels.
#pragma unroll
                                for (int o = 8; o <= 16; o <<= 1) {
                                    gs.x += __shfl_xor_sync(0xffffffffu, gs.x, o);
                                    gs.y += __shfl_xor_sync(0xffffffffu, gs.y, o);
                                    gs.z += __shfl_xor_sync(0xffffffffu, gs.z, o);
                                    gs.w += __shfl_xor_sync(0xffffffffu, gs.w, o);
                                    gq.x += __shfl_xor_sync(0xffffffffu, gq.x, o);
                                    gq.y += __shfl_xor_sync(0xffffffffu, gq.y, o);
                                    gq.z += __shfl_xor_sync(0xffffffffu, gq.z, o);
                                    gq.w += __shfl_xor_sync(0xffffffffu, gq.w, o);
                                }
                                if (lane < 8 && col_ok) {
                                    float* dst = args.gn_part + ((tile_m0(t) / BM) * 4 + qd) * 2 * (int64_t)args.c_out + col;
                                    *reinterpret_cast<float4*>(dst) = gs;
                                    *reinterpret_cast<float4*>(dst + args.c_out) = gq;
                                }
                            }
                        }
                        if (cc + 32 < bn) cur = nxt;
                    }
                    __syncwarp();  // the slots are read before any lane overwrites them
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {  // uniform: nothing raises the flag after the barrier above
        // Abort path: no bulk copy may still be writing this CTA's shared memory when it exits,
        // so the TMA issuers wait for the last phase of every slot they armed. A weight stage's
        // phase also counts one arrival per converter thread: converters that stopped early make
        // theirs for the fills the weight issuer armed. The weight issuer arms fill i only after
        // fill i - stages was consumed, so it is at most `stages` fills ahead of any converter,
        // and each such arrival lands in the phase of its own fill.
        const long long deadline = clock64() + kWaitLimit;
        if (is_converter) {
            const int armed = *s_wfills;
            for (int i = conv_fills; i < armed; ++i) mbar_arrive(b_full_bar(i % bstages));
        }
        if (warp == 5 && lane == 0)
            for (int i = max(0, w_fills - bstages); i < w_fills; ++i)
                drain_wait(b_full_bar(i % bstages), (uint32_t)((i / bstages) & 1), deadline, args.err, 10);
        if (warp == 5 && lane == 1 && args.a_tma)
            for (int i = max(0, a_fills - nstg); i < a_fills; ++i)
                drain_wait(sfull_bar(i % nstg), (uint32_t)((i / nstg) & 1), deadline, args.err, 11);
        // A residual load of the bulk-store epilogue still in flight completes its barrier phase.
        if (warp >= 6 && warp < 10 && lane == 0 && res_pending)
            drain_wait(res_bar(warp & 3), res_phase, deadline, args.err, 14);
        __syncthreads();
    }
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)args.tmem_cols);
    }
}

// Self-test of the bounded-wait error path: one thread initialises a barrier that nothing will
// ever arrive at and waits on it as the conv roles wait, with the caller's limit; no copy is
// issued. The wait gives up, records the timeout in the context's error word, and the kernel
// returns.
__global__ void wait_probe_kernel(int* err, long long limit) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    abort_flag = 0;
    fence_mbarrier_init();
    (void)mbar_wait(b, 0, err, 12, &abort_flag, false, limit, kKWaitProbe);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
        if (q != cudaDriverEntryPointSuccess || !p) fail(MBX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

void encode_one(CUtensorMap* map, const float* data, int64_t kdim, int64_t rows, int bn) {
    cuuint64_t dims[2] = {(cuuint64_t)kdim, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kdim * 4};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(data), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(MBX_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

// Tensor map over the activations x (f32, channels innermost) for the A-operand boxes; reads
// outside the map fill with zeros.
void encode_a_map(CUtensorMap* map, const float* x, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                  const cuuint32_t* box) {
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<float*>(x), dims,
                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(MBX_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (" + std::to_string((int)r) + ")");
}

int sum_bytes(int bn) { return 128 * (bn + 4) * 4; }

int stage_count(bool f32w, int bn) {
    const int stage = (f32w ? 2 : 1) * bn * 128;
    return std::min(8, (kMaxSmem - 2048 - kMinStgSlots * (int)A_BYTES - sum_bytes(bn)) / stage);
}

template <bool F32W, bool VEC4, bool FLAT, bool GN>
void run_conv(mbx_ctx* ctx, const mbx_param* p, const ConvArgs& a, const CUtensorMap& tmap_a,
              const CUtensorMap& tmap_out, const CUtensorMap& tmap_res, int64_t m_tiles) {
    auto kernel = conv_tc_kernel<F32W, VEC4, FLAT, GN>;
    const int stage = (F32W ? 2 : 1) * a.bn * 128;
    const int smem = a.stages * stage + a.stg_slots * (int)A_BYTES + sum_bytes(a.bn) + 1024 + 512;
    // The register check depends on the build only, so once per process suffices; the
    // shared-memory limit is a per-device attribute.
    static std::once_flag checked;
    std::call_once(checked, [&] {
        cudaFuncAttributes fa;
        check_cuda(cudaFuncGetAttributes(&fa, kernel), "conv attributes");
        if (fa.maxThreadsPerBlock < kThreads)
            fail(MBX_ERR_INTERNAL, "conv kernel built with " + std::to_string(fa.numRegs) +
                                       " registers per thread cannot launch " + std::to_string(kThreads) +
                                       " threads");
    });
    ensure_smem_limit(reinterpret_cast<const void*>(kernel), kMaxSmem, "conv smem attribute");
    (void)m_tiles;
    // Persistent: one CTA per SM (the shared-memory footprint allows one), tiles strided over them.
    const int64_t blocks = std::min<int64_t>(a.tiles, (int64_t)ctx->sm_count);
    kernel<<<(unsigned)blocks, kThreads, smem, ctx->stream>>>(p->tmap_hi, F32W ? p->tmap_lo : p->tmap_hi, tmap_a,
                                                              tmap_out, tmap_res, a);
}

}  // namespace

bool conv_gn_fusable(const ConvShape& s, int64_t c_out) { return c_out % 4 == 0 && (s.ho * s.wo) % 256 == 0; }

int64_t conv_gn_part_floats(const ConvShape& s, int64_t c_out) {
    return (s.n * s.ho * s.wo + BM - 1) / BM * 4 * 2 * c_out;
}

void launch_wait_probe(mbx_ctx* ctx, int64_t cycles) {
    wait_probe_kernel<<<1, 1, 0, ctx->stream>>>(ctx->dev_err, (long long)cycles);
    after_launch(ctx, "wait probe");
}

void encode_tensor_map_f32(CUtensorMap* map, const float* base, int rank, const uint64_t* dims,
                           const uint64_t* strides, const uint32_t* box, bool swizzle128) {
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], estr[5] = {1, 1, 1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        if (i + 1 < rank) st[i] = strides[i];
    }
    CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<float*>(base), d, st,
                             b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(MBX_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

int choose_bn(int64_t c_out, bool f32_weights) {
    // Fewest padded columns, with a per-tile cost for tiles that re-read the same A rows.
    int best = 32;
    int64_t best_cost = INT64_MAX;
    for (int bn = 128; bn >= 32; bn -= 32) {
        const int64_t tiles = (c_out + bn - 1) / bn;
        const int64_t cost = tiles * bn + 32 * tiles;
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    // 160-wide tiles (three pipeline stages instead of four) only where they pad less
    // than the 128-wide ones: 320, 800, 1600 ... output channels.
    if (!f32_weights && best == 128 && (c_out + 159) / 160 * 160 < (c_out + 127) / 128 * 128) best = kMaxBn;
    return best;
}

void encode_param_tmaps(mbx_param* p) {
    const int64_t kdim = p->taps * p->cin_pad;
    encode_one(&p->tmap_hi, p->hi, kdim, p->cout_pad, p->bn);
    if (p->lo)
        encode_one(&p->tmap_lo, p->lo, kdim, p->cout_pad, p->bn);
    else
        p->tmap_lo = p->tmap_hi;
}

void launch_conv_tc(mbx_ctx* ctx, const float* x, const ConvShape& s, const mbx_param* p, const float* bias,
                    const float* pro_scale, const float* pro_shift, bool pro_silu, const float* residual,
                    float* out, int act, float* gn_part, const float* gn_add) {
    if (pro_scale) {
        // The GroupNorm prologue as its own memory-bound pass into a pooled buffer. Applied per
        // K chunk in the converters it is redone for every tap and every N tile that reads the
        // pixel (36 times for a 3×3 conv to 512 channels), and its per-chunk scale / shift loads sit
        // on the converters' critical path: 3×3 convs with it ran 3.3× slower, 1×1 convs 1.9×.
        // Padding stays zero either way (the conv reads zeros outside the map).
        PoolBuf normed(ctx, size_t(s.n * s.h * s.w * s.c_in) * sizeof(float));
        launch_gn_apply(ctx, x, s.n, s.h * s.w, s.c_in, pro_scale, pro_shift, pro_silu, nullptr,
                        normed.as<float>());
        launch_conv_tc(ctx, normed.as<float>(), s, p, bias, nullptr, nullptr, false, residual, out, act, gn_part,
                       gn_add);
        return;
    }
    ConvArgs a{};
    a.x = x;
    a.m_total = s.n * s.ho * s.wo;
    a.h = (int)s.h;
    a.w = (int)s.w;
    a.c_in = (int)s.c_in;
    a.ho = (int)s.ho;
    a.wo = (int)s.wo;
    a.stride = s.stride;
    a.pad_t = s.pad_t;
    a.pad_l = s.pad_l;
    a.up = s.up;
    a.cin_chunks = p->cin_pad / BK;
    a.k_chunks = (int)p->taps * a.cin_chunks;
    a.flat = p->taps == 1 ? 1 : 0;
    a.c_out = (int)p->c_out;
    a.bn = p->bn;
    a.n_tiles = p->cout_pad / p->bn;
    const bool f32w = p->lo != nullptr;
    a.stages = std::min(stage_count(f32w, p->bn), std::min(kMaxAStages, (512 - 2 * p->bn) / 64));
    // The MMA thread waits for two consecutive stages at once: the ring needs at least two.
    if (a.stages < 2) fail(MBX_ERR_INTERNAL, "conv: fewer than two pipeline stages fit");
    {
        const int stage = (f32w ? 2 : 1) * p->bn * 128;
        a.stg_slots = std::min(kMaxStgSlots, (kMaxSmem - 2048 - a.stages * stage - sum_bytes(p->bn)) / (int)A_BYTES);
        if (a.stg_slots < kMinStgSlots) fail(MBX_ERR_INTERNAL, "conv: fewer than three staging slots fit");
    }
    a.tmem_cols = 512;
    a.a_stages = a.stages;
    a.bias = bias;
    a.residual = residual;
    a.out = out;
    a.act = act;
    a.gn_part = gn_part;
    a.gn_add = gn_add;
    MBX_REQUIRE(!gn_part || conv_gn_fusable(s, p->c_out),
                "conv: GroupNorm statistics in the epilogue need c_out % 4 == 0 and output maps of 256k pixels");
    a.err = ctx->dev_err;
    MBX_REQUIRE(a.m_total < (int64_t(1) << 40), "conv: too many output pixels");
    const int64_t m_tiles = (a.m_total + BM - 1) / BM;
    MBX_REQUIRE(m_tiles * a.n_tiles < (int64_t(1) << 40), "conv: too many tiles");
    a.tiles = m_tiles * a.n_tiles;
    // The abort path counts a CTA's K chunks in 32-bit integers.
    MBX_REQUIRE((a.tiles + ctx->sm_count - 1) / ctx->sm_count * a.k_chunks < (int64_t(1) << 31),
                "conv: too many K chunks per CTA");
    const bool vec4 = (s.c_in & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const bool aligned_out = (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                             (!residual || (reinterpret_cast<uintptr_t>(residual) & 15) == 0) &&
                             (!bias || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
    MBX_REQUIRE(aligned_out || (p->c_out & 3) != 0,
                "conv: out, residual and bias must be 16-byte aligned when c_out is a multiple of 4");
    // A by TMA where one box per chunk covers the tile's 128 rows: 1×1 convs (a 2-D view of x), and
    // 3×3 stride-1 convs whose tiles are whole image rows or 128-pixel pieces of one row.
    CUtensorMap tmap_a = p->tmap_hi;  // unused when a_tma == 0
    a.a_tma = 0;
    a.a_bw = 0;
    if (vec4 && s.c_in >= BK && a.m_total < (int64_t(1) << 31)) {  // boxes no wider than the map
        const int64_t hw = s.h * s.w;
        if (a.flat) {
            a.a_tma = 1;
            cuuint64_t dims[2] = {(cuuint64_t)s.c_in, (cuuint64_t)a.m_total};
            cuuint64_t strides[1] = {(cuuint64_t)s.c_in * 4};
            cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BM};
            encode_a_map(&tmap_a, x, 2, dims, strides, box);
        } else if (s.stride == 1 && s.up == 0 && s.ho == s.h && s.wo == s.w && hw % BM == 0 &&
                   (s.w % BM == 0 || BM % s.w == 0) && s.h < (1 << 30) && s.w < (1 << 30) && s.n < (1 << 30)) {
            a.a_tma = 2;
            a.a_bw = (int)std::min<int64_t>(s.w, BM);
            cuuint64_t dims[4] = {(cuuint64_t)s.c_in, (cuuint64_t)s.w, (cuuint64_t)s.h, (cuuint64_t)s.n};
            cuuint64_t strides[3] = {(cuuint64_t)s.c_in * 4, (cuuint64_t)(s.w * s.c_in) * 4,
                                     (cuuint64_t)(hw * s.c_in) * 4};
            cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)a.a_bw, (cuuint32_t)(BM / a.a_bw), 1};
            encode_a_map(&tmap_a, x, 4, dims, strides, box);
        }
    }
    // Bulk-store epilogue: float4 outputs.
    CUtensorMap tmap_out = p->tmap_hi, tmap_res = p->tmap_hi;  // unused unless tma_out
    a.tma_out = 0;
    a.has_res = 0;
    if ((p->c_out & 3) == 0 && a.m_total < (int64_t(1) << 31)) {
        a.tma_out = 1;
        cuuint64_t dims[2] = {(cuuint64_t)p->c_out, (cuuint64_t)a.m_total};
        cuuint64_t strides[1] = {(cuuint64_t)p->c_out * 4};
        cuuint32_t box[2] = {32, 32};
        encode_a_map(&tmap_out, out, 2, dims, strides, box);
        if (residual) {
            a.has_res = 1;
            encode_a_map(&tmap_res, residual, 2, dims, strides, box);
        }
    }
    auto dispatch = [&](auto gn) {
        constexpr bool G = decltype(gn)::value;
        if (a.flat) {
            if (f32w)
                vec4 ? run_conv<true, true, true, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles)
                     : run_conv<true, false, true, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles);
            else
                vec4 ? run_conv<false, true, true, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles)
                     : run_conv<false, false, true, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles);
        } else {
            if (f32w)
                vec4 ? run_conv<true, true, false, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles)
                     : run_conv<true, false, false, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles);
            else
                vec4 ? run_conv<false, true, false, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles)
                     : run_conv<false, false, false, G>(ctx, p, a, tmap_a, tmap_out, tmap_res, m_tiles);
        }
    };
    if (gn_part)
        dispatch(std::true_type{});
    else
        dispatch(std::false_type{});
    after_launch(ctx, "conv (tcgen05)");
}

}  // namespace mbx
