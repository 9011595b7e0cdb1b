// attention_noalloc.cu -- grouped attention for callers that cannot allocate device memory.
//
// satori_grouped_attention_device needs scratch space for its split-K partial records and gets it
// from a context that calls cudaMalloc.  Some callers cannot do that: a host application that has
// already handed all of the GPU's memory to its own pool, or a code path that cannot accept the
// device-wide synchronisation cudaMalloc implies.  satori_grouped_attention_noalloc runs the same two
// kernels with their scratch in a fixed array that lives in this library's device image, so the call
// itself allocates nothing: the caller passes device pointers for the inputs and the output and a
// stream, and that is all.
//
// The array is kNoAllocScratchFloats floats (4 MiB) per device; every GPU that loads the library
// holds it until the process exits.  A request whose partial records would not fit is rejected.
#include <mutex>

#include "attention.cuh"
#include "capi_internal.h"

namespace {

constexpr size_t kNoAllocScratchFloats = 1u << 20;  // 4 MiB of partial records per device
constexpr int kMaxDevices = 64;

// The scratch lives here.  Host code must not pass this name to a kernel: on the host it is only a
// stand-in for the symbol, and its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

struct DeviceSetup {
    bool ready = false;
    float *scratch = nullptr;  // device address of g_noalloc_scratch on that device
    int sm_count = 0;
};

std::mutex g_setup_lock;
DeviceSetup g_setup[kMaxDevices];

// Once per device, with that device current: resolve the array's device address and the SM count.
int setup_current_device(DeviceSetup **out)
{
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return satori::cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return satori::set_error(SATORI_ERR_NOT_SUPPORTED, "device %d", dev);
    std::lock_guard<std::mutex> lock(g_setup_lock);
    DeviceSetup &s = g_setup[dev];
    if (!s.ready) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return satori::cuda_fail(e, "cudaGetSymbolAddress(scratch)");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return satori::cuda_fail(e, "cudaDeviceGetAttribute");
        s.scratch = static_cast<float *>(ptr);
        s.sm_count = sms;
        s.ready = true;
    }
    *out = &s;
    return SATORI_OK;
}

}  // namespace

extern "C" int satori_grouped_attention_noalloc(const float *q, const float *keys, const float *values, int q_heads,
                                                int kv_heads, int head_dim, int tokens, float *out, void *stream)
{
    if (!q || !keys || !values || !out) return satori::set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (head_dim <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || tokens <= 0)
        return satori::set_error(SATORI_ERR_ARGUMENT, "Invalid grouped-attention dimensions.");
    if (head_dim > 256) return satori::set_error(SATORI_ERR_NOT_SUPPORTED, "head_dim > 256 is not supported");
    DeviceSetup *dev = nullptr;
    int rc = setup_current_device(&dev);
    if (rc) return rc;
    const size_t need = satori::attn_scratch_floats(q_heads, kv_heads, head_dim, tokens, dev->sm_count);
    if (need > kNoAllocScratchFloats)
        return satori::set_error(SATORI_ERR_ARGUMENT,
                                 "attention needs %zu scratch floats; the allocation-free entry point holds %zu "
                                 "(use satori_grouped_attention_device)",
                                 need, kNoAllocScratchFloats);
    // Every record the merge kernel reads is written by the partial kernel of the same call, so the
    // array's previous contents never matter and nothing has to be cleared.
    satori::AttnArgs a = {};
    a.q = q;
    a.keys = keys;
    a.values = values;
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.tokens = tokens;
    a.max_tokens = tokens;
    a.out = out;
    a.scratch = dev->scratch;
    cudaError_t e = satori::launch_attention(a, dev->sm_count, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? SATORI_OK : satori::cuda_fail(e, "launch attention");
}
