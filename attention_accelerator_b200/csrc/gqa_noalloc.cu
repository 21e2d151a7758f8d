// gqa_noalloc.cu -- gqa_decode_noalloc: the single-sequence decode with its
// scratch memory (split table and FP32 split partials) in a fixed, library-owned
// device array instead of a caller-allocated workspace.
//
// Who needs it: callers that may not allocate device memory themselves, e.g. a
// plug-in running inside a host program that owns every device allocation (a
// fixed memory budget or an allocator that must account for all memory), or a
// latency-critical serving loop that cannot afford cudaMalloc's implicit device
// synchronisation.  Such a caller passes only its inputs and outputs.
//
// The array is GQA_NOALLOC_SCRATCH_BYTES large and, like any file-scope device
// variable, exists on every GPU that loads this library until the process exits.
// In host code `g_noalloc_scratch` names a host-side stand-in, not the device
// array, so its device address is looked up with cudaGetSymbolAddress, once per
// device, with that device current, on the first call made on that device.
#include "gqa_b200.h"

#include <cuda_runtime.h>

#include <mutex>

namespace {

constexpr size_t kScratchBytes = GQA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up on first use).
int scratch_for_current_device(void** ptr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GQA_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return GQA_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *ptr = g_scratch_ptr[dev];
    return GQA_OK;
}

}  // namespace

extern "C" int gqa_decode_noalloc(const void* q, const void* k, const void* v, void* out, const gqa_params* p,
                                  void* stream) {
    const int st = gqa_validate(p);
    if (st != GQA_OK) return st;
    // Scratch this call needs (host-side planning; nothing is allocated).
    const size_t need = gqa_workspace_bytes(p, nullptr, 1);
    if (need == 0) return GQA_ERR_CUDA;
    if (need > kScratchBytes) return GQA_ERR_WORKSPACE;  // beyond the fixed scratch: use gqa_decode
    void* scratch = nullptr;
    const int sst = scratch_for_current_device(&scratch);
    if (sst != GQA_OK) return sst;
    // The split table and partials are written before they are read within a
    // call.  The only state that must start at zero, the per-KV-head split
    // arrival counters, is zero when the library loads (device variables are
    // zero-initialised) and the last split of each head sets its counter back
    // to zero before the kernel ends, so nothing needs clearing between calls.
    return gqa_decode(q, k, v, out, p, scratch, kScratchBytes, stream);
}
