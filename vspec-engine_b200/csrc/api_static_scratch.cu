// api_static_scratch.cu -- the low-bit GEMV with a scratch buffer that the
// library never allocates: a file-scope __device__ array.
//
// Who needs it: callers that must not see a device allocation inside a call.
//   * Runtimes whose device memory belongs to their own arena or pool
//     allocator (Vspec's IR scheduler plans every buffer up front): an
//     allocation behind the allocator's back can fail once the pool has
//     reserved the device, or fragment it.
//   * Decode loops that must not stall: the library-managed workspace of
//     vspec_b200_lowbit_linear grows on the first use of a larger shape with a
//     device synchronisation, cudaFree and cudaMalloc.
//   Callers that can pass their own zeroed workspace use
//   vspec_b200_lowbit_linear instead and have no size limit.
//
// Contract:
//   * scratch: kStaticGemvScratchBytes (16 MiB) per device.  Shapes whose
//     workspace (vspec_b200_lowbit_linear_workspace_bytes) exceeds it are
//     rejected with VSPEC_B200_ERR_ARG before anything is launched.
//   * what must start at zero: the first 64 KiB (split-K tile counters).
//     Every call clears them with a cudaMemsetAsync on its own stream before
//     the launch (a memset, not an allocation).  A completed launch leaves
//     them zero anyway, but one whose bounded wait gave up (the flag read by
//     vspec_b200_gemv_timeout_flag) can leave a tile's count part-way, and the
//     caller has no other way to reach this array; the clear keeps such a
//     launch from corrupting every later call on the device.  The fp32
//     partials after the counters need no initialisation.
//   * set-up: the first call on a device (with that device current) looks up
//     the array's device address with cudaGetSymbolAddress and keeps it.
//     Under CUDA's default lazy module loading that lookup is also what loads
//     this file's module and reserves the 16 MiB on the device (at process
//     start with CUDA_MODULE_LOADING=EAGER).  So make that first call before
//     the caller's arena or pool allocator reserves the device's memory, and
//     before any stream capture; later calls allocate nothing.
//   * one buffer per device: calls on the same device that overlap (different
//     streams, host threads, or graphs replayed concurrently) race on the
//     counters and partials.  Calls must be ordered on one stream.
#include "common.cuh"

#include <mutex>

#include "vspec_b200.h"

namespace {

constexpr size_t kStaticGemvScratchBytes = 16u << 20;
// The split-K tile counters at the start of any GEMV workspace (the fixed
// 16384-int region the merge kernels count in).
constexpr size_t kStaticGemvCounterBytes = 64u << 10;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_gemv_scratch[kStaticGemvScratchBytes];

void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the static scratch on the current device (set-up on the
// first call per device).  Returns VSPEC_B200_OK or an error code.
int static_scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return vb200::cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        vb200::set_error("device %d out of range for the static GEMV scratch", dev);
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_static_gemv_scratch);
        if (e != cudaSuccess) return vb200::cuda_status(e, "cudaGetSymbolAddress(static GEMV scratch)");
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return VSPEC_B200_OK;
}

}  // namespace

extern "C" int vspec_b200_lowbit_linear_static(const VspecB200LinearArgs* a, void* stream) {
    if (!a) { vb200::set_error("args is NULL"); return VSPEC_B200_ERR_ARG; }
    if (a->d_workspace || a->workspace_bytes) {
        vb200::set_error("vspec_b200_lowbit_linear_static uses its own static scratch: d_workspace must be NULL "
                         "and workspace_bytes 0");
        return VSPEC_B200_ERR_ARG;
    }
    if (a->m == 0 || a->n == 0 || a->k == 0) { vb200::set_error("zero dimension"); return VSPEC_B200_ERR_ARG; }
    const size_t need = vspec_b200_lowbit_linear_workspace_bytes(a->m, a->n, a->k, a->flags);
    if (need > kStaticGemvScratchBytes) {
        vb200::set_error("shape m=%zu n=%zu k=%zu needs %zu bytes of GEMV scratch; the static scratch holds %zu "
                         "(use vspec_b200_lowbit_linear with a caller workspace)",
                         a->m, a->n, a->k, need, kStaticGemvScratchBytes);
        return VSPEC_B200_ERR_ARG;
    }
    void* ptr = nullptr;
    const int rc = static_scratch_for_current_device(&ptr);
    if (rc != VSPEC_B200_OK) return rc;
    // The split-K counters must start at zero; a launch that aborted on a
    // bounded wait may have left some set.
    cudaError_t e = cudaMemsetAsync(ptr, 0, kStaticGemvCounterBytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return vb200::cuda_status(e, "cudaMemsetAsync(static GEMV counters)");
    VspecB200LinearArgs b = *a;
    b.d_workspace = ptr;
    b.workspace_bytes = kStaticGemvScratchBytes;
    return vspec_b200_lowbit_linear(&b, stream);
}

// Test hook: the counter region of the current device's static scratch filled
// with `byte`, the state a launch whose bounded wait gave up can leave behind.
extern "C" int vspec_b200_debug_poison_static_scratch(int byte) {
    void* ptr = nullptr;
    const int rc = static_scratch_for_current_device(&ptr);
    if (rc != VSPEC_B200_OK) return rc;
    const cudaError_t e = cudaMemset(ptr, byte & 0xFF, kStaticGemvCounterBytes);
    return e == cudaSuccess ? VSPEC_B200_OK : vb200::cuda_status(e, "poison static scratch");
}
