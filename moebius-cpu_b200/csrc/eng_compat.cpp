// The reference's outer C ABI (moebius_* in include/moebius_cpu.h) over this
// library's engine ABI (mbx_* in include/moebius_cuda_engine.h), so a host
// built against moebius-cpu links this library unchanged. Reference
// implementation of the same calls: src/ffi.rs:105-233.
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "../../include/moebius_cpu.h"
#include "../../include/moebius_cuda_engine.h"
#include "mbx_internal.h"

// One engine per handle. The reference shares an Engine across threads
// (`&self`, src/pipeline.rs:119-136); the GPU engine keeps per-call state on one
// stream, so concurrent calls on a handle take turns.
struct MoebiusEngine {
    mbx_engine* eng = nullptr;
    std::mutex mu;
};

static_assert(sizeof(MoebiusParams) == sizeof(mbx_inpaint_params), "params layouts differ");
static_assert(offsetof(MoebiusParams, seed) == offsetof(mbx_inpaint_params, seed), "params layouts differ");
static_assert(offsetof(MoebiusParams, mask_dilate) == offsetof(mbx_inpaint_params, mask_dilate),
              "params layouts differ");
static_assert(sizeof(MoebiusRect) == sizeof(mbx_rect), "rect layouts differ");

namespace {

// The reference has codes 0-6; the GPU-only failures (7 out of memory, 8 CUDA error,
// 9 device wait timed out) are internal errors to its hosts. The message is kept.
int32_t to_moebius(int32_t status) { return status <= MBX_ERR_INTERNAL ? status : MOEBIUS_ERR_INTERNAL; }

// MOEBIUS_CUDA_DEVICE selects the GPU (default 0).
int32_t device_from_env(int32_t* device) {
    const char* v = std::getenv("MOEBIUS_CUDA_DEVICE");
    *device = 0;
    if (!v || !*v) return MBX_OK;
    char* end = nullptr;
    const long d = std::strtol(v, &end, 10);
    if (*end != '\0' || d < 0 || d > 1024) {
        mbx::record_error(MBX_ERR_INVALID_ARGUMENT, "MOEBIUS_CUDA_DEVICE must be a device index");
        return MBX_ERR_INVALID_ARGUMENT;
    }
    *device = (int32_t)d;
    return MBX_OK;
}

}  // namespace

extern "C" {

uint32_t moebius_abi_version(void) { return MOEBIUS_ABI_VERSION; }

const char* moebius_last_error(void) { return mbx_last_error(); }

int32_t moebius_engine_create(const char* weights_dir, uint32_t threads, MoebiusEngine** out) {
    (void)threads;  // a CPU thread-pool size; the work runs on the GPU
    if (!weights_dir || !out) {
        mbx::record_error(MBX_ERR_INVALID_ARGUMENT, "null argument");
        return MOEBIUS_ERR_INVALID_ARGUMENT;
    }
    // As in the reference, *out is written only on success.
    int32_t device = 0;
    int32_t st = device_from_env(&device);
    if (st != MBX_OK) return to_moebius(st);
    auto* h = new (std::nothrow) MoebiusEngine();
    if (!h) {
        mbx::record_error(MBX_ERR_INTERNAL, "host allocation failed");
        return MOEBIUS_ERR_INTERNAL;
    }
    st = mbx_engine_create(weights_dir, device, &h->eng);
    if (st != MBX_OK) {
        delete h;
        return to_moebius(st);
    }
    *out = h;
    return MOEBIUS_OK;
}

void moebius_engine_destroy(MoebiusEngine* engine) {
    if (!engine) return;
    mbx_engine_destroy(engine->eng);
    delete engine;
}

int32_t moebius_inpaint(const MoebiusEngine* engine, uint8_t* pixels, uint32_t width, uint32_t height,
                        uint32_t stride, uint32_t channels, const uint8_t* mask, uint32_t mask_stride,
                        const MoebiusParams* params, MoebiusProgressFn progress, void* user, MoebiusRect* changed) {
    if (!engine) {
        mbx::record_error(MBX_ERR_INVALID_ARGUMENT, "null engine");
        return MOEBIUS_ERR_INVALID_ARGUMENT;
    }
    auto* h = const_cast<MoebiusEngine*>(engine);
    std::lock_guard<std::mutex> lock(h->mu);
    const int32_t st =
        mbx_inpaint(h->eng, pixels, width, height, stride, channels, mask, mask_stride,
                    reinterpret_cast<const mbx_inpaint_params*>(params), reinterpret_cast<mbx_progress_fn>(progress),
                    user, reinterpret_cast<mbx_rect*>(changed));
    return to_moebius(st);
}

}  // extern "C"
