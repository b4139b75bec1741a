// noalloc.cu -- fp4attn_forward_noalloc: the forward pass for callers that
// cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc (or any allocator) at
// the point where they need attention: code that runs while a stream is being
// captured into a CUDA graph, runtimes that own every byte of device memory
// and forbid allocation after start-up, and latency-critical loops where an
// allocation could block on the driver.  fp4attn_forward needs a workspace
// for the quantised Q and K; this entry point uses a fixed scratch array that
// the library holds instead, so the caller passes only inputs and outputs.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (64 MiB).  It lives in this file's own module, so it is reserved on a device
// when the module is first loaded there (at the first call of this entry
// point, or when the context is created under CUDA_MODULE_LOADING=EAGER) and
// stays reserved until the process exits.  Problems whose workspace
// (fp4attn_workspace_size) exceeds it are rejected with FP4ATTN_EWORKSPACE.
//
// Every call on a device uses the same scratch.  Calls that can overlap on the
// GPU (different streams, no ordering between them) race on it; serialise them
// (one stream, or events).  The scratch keeps whatever the previous call left
// in it.  The only words that must start at zero -- the arrival counters of
// the key partitions small problems are split into -- are cleared by each
// call's quantiser launch; every other byte the attention kernel reads is
// written by that same call first (codes of every real row, scale tiles of
// every row including padding rows, the FP16 copy of V for FP32 input, and
// the partitions' partial results).
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/fp4attn.h"

namespace fp4attn {
void set_error_detail(const char* msg);          // fp4attn.cu
unsigned long long current_context_id();         // fp4attn.cu
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per device: the scratch's device address and the context it belongs to.
struct ScratchAddr {
    unsigned long long ctx = 0;
    void* addr = nullptr;
};
std::mutex g_setup_mutex;
ScratchAddr g_scratch_addr[kMaxDevices];

// Device address of the scratch array on `dev` (the current device), looked
// up once per device with that device current: the host-side name of a
// __device__ array is not a device address.  The lookup is repeated when the
// device's context has changed since (a device reset destroys the context,
// and the module, with the array, is loaded again at another address).
int scratch_address(int dev, void** out)
{
    if (dev < 0 || dev >= kMaxDevices) {
        fp4attn::set_error_detail("fp4attn_forward_noalloc: device ordinal out of range");
        return FP4ATTN_EUNSUPPORTED;
    }
    const unsigned long long ctx = fp4attn::current_context_id();
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    ScratchAddr& s = g_scratch_addr[dev];
    if (!s.addr || ctx == 0 || s.ctx != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            char buf[160];
            snprintf(buf, sizeof buf, "fp4attn_forward_noalloc: cudaGetSymbolAddress failed: %s",
                     cudaGetErrorString(e));
            fp4attn::set_error_detail(buf);
            return FP4ATTN_ECUDA;
        }
        s.addr = p;
        // The lookup itself makes the primary context current when none was.
        s.ctx = ctx != 0 ? ctx : fp4attn::current_context_id();
    }
    *out = s.addr;
    return FP4ATTN_OK;
}

}  // namespace

extern "C" int fp4attn_forward_noalloc(const void* Q, const void* K, const void* V, void* Out, int in_dtype,
                                       int out_dtype, int batch, int heads, int seq_q, int seq_k, int head_dim,
                                       float softmax_scale, int scale_mode, void* stream)
{
    const size_t need = fp4attn_workspace_size(batch, heads, seq_q, seq_k, head_dim, in_dtype);
    if (need > kNoAllocScratchBytes) {
        char buf[200];
        snprintf(buf, sizeof buf,
                 "fp4attn_forward_noalloc: this problem needs %zu bytes of scratch, more than the %zu bytes "
                 "the no-allocation entry point holds; use fp4attn_forward with a caller workspace",
                 need, kNoAllocScratchBytes);
        fp4attn::set_error_detail(buf);
        return FP4ATTN_EWORKSPACE;
    }
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        fp4attn::set_error_detail("fp4attn_forward_noalloc: cudaGetDevice failed");
        return FP4ATTN_ECUDA;
    }
    void* scratch = nullptr;
    const int rc = scratch_address(dev, &scratch);
    if (rc != FP4ATTN_OK) return rc;
    // Invalid shapes (need == 0) are reported in detail by fp4attn_forward.
    return fp4attn_forward(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale,
                           scale_mode, scratch, kNoAllocScratchBytes, stream);
}
