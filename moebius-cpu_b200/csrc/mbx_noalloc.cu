// mbx_group_norm_forward_noalloc: GroupNorm(+SiLU) forward for callers that
// must not allocate device memory.
//
// Who needs it: hosts that plan every byte of device memory themselves (a
// serving runtime with a fixed budget, a plugin handed a stream and buffers
// by its host application) and code running on a stream owned by another
// framework. Such callers cannot let a kernel library call cudaMalloc or
// cudaFree behind their back: those calls can synchronise the whole device,
// stalling the host's other streams, and they draw from memory the host has
// already promised elsewhere. They also often have no mbx_ctx (whose creation
// allocates its pool and error word), so this entry point takes a plain stream.
//
// The statistics scratch (f64 chunk partials, then per-item scale/shift) lives
// in one file-scope __device__ array of kScratchBytes (8 MiB). Every GPU that
// loads this library holds that array until the process exits.
#include <mutex>

#include "mbx_internal.h"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

// The shared scratch. Host code only ever sees the host-side stand-in for this
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_gn_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

// Once per device, with that device current: resolve the array's device address.
void device_setup(int dev, void** ptr, int* sms) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        int major = 0, minor = 0, count = 0;
        mbx::check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "device query");
        mbx::check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev), "device query");
        if (major != 10 || minor != 0) mbx::fail(MBX_ERR_UNSUPPORTED_DEVICE, "needs an sm_100 GPU (B200)");
        mbx::check_cuda(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev), "device query");
        void* p = nullptr;
        mbx::check_cuda(cudaGetSymbolAddress(&p, g_gn_scratch), "cudaGetSymbolAddress(GroupNorm scratch)");
        g_sm_count[dev] = count;
        g_scratch_ptr[dev] = p;
    }
    *ptr = g_scratch_ptr[dev];
    *sms = g_sm_count[dev];
}

}  // namespace

extern "C" int32_t mbx_group_norm_forward_noalloc(void* stream, const float* x, int64_t n, int64_t h, int64_t w,
                                                  int64_t c, int64_t groups, float eps, const float* gamma,
                                                  const float* beta, const float* add, int32_t silu, float* out) {
    try {
        MBX_REQUIRE(n >= 0 && h >= 0 && w >= 0 && c > 0, "bad shape");
        MBX_REQUIRE(groups > 0 && c % groups == 0, "channels not divisible by groups");
        MBX_REQUIRE(c <= 8192 && groups <= 1024, "GroupNorm supports at most 8192 channels and 1024 groups");
        if (n == 0) return MBX_OK;
        MBX_REQUIRE(h * w > 0, "GroupNorm over an empty image");
        MBX_REQUIRE(x && gamma && beta && out, "null pointer");
        const int64_t hw = h * w;
        const size_t part_bytes = size_t(n) * mbx::gn_chunks(hw) * groups * 2 * sizeof(double);
        const size_t ss_off = (part_bytes + 255) & ~size_t(255);
        const size_t need = ss_off + size_t(n) * c * 2 * sizeof(float);
        if (need > kScratchBytes)
            mbx::fail(MBX_ERR_INVALID_ARGUMENT,
                      "mbx_group_norm_forward_noalloc: needs " + std::to_string(need) +
                          " bytes of scratch (n * ceil(h*w/256) * groups * 16 + n * c * 8), above its fixed " +
                          std::to_string(kScratchBytes) + "-byte maximum; use mbx_group_norm_forward");
        int dev = 0;
        mbx::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        MBX_REQUIRE(dev >= 0 && dev < kMaxDevices, "device index out of range");
        void* scratch = nullptr;
        int sms = 0;
        device_setup(dev, &scratch, &sms);

        mbx_ctx view;  // a stack view over the caller's stream: no pool, no allocation
        view.device = dev;
        view.stream = static_cast<cudaStream_t>(stream);
        view.own_stream = view.stream;
        view.sm_count = sms;
        double* part = static_cast<double*>(scratch);
        float* scale = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + ss_off);
        float* shift = scale + n * c;
        // Every partial and every scale/shift entry is written before it is read, so
        // nothing in the shared array has to start at zero.
        mbx::launch_gn_partials(&view, x, n, hw, c, groups, add, part);
        mbx::launch_gn_finalize(&view, part, n, hw, c, groups, eps, gamma, beta, add, scale, shift);
        mbx::launch_gn_apply(&view, x, n, hw, c, scale, shift, silu != 0, nullptr, out);
        return MBX_OK;
    } catch (const mbx::Error& e) {
        mbx::record_error(e.code, e.what());
        return e.code;
    } catch (...) {
        mbx::record_error(MBX_ERR_INTERNAL, "internal error");
        return MBX_ERR_INTERNAL;
    }
}
