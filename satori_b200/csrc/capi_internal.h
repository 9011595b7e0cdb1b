// capi_internal.h -- shared host-side state of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include <string>

#include "../../include/satori_cuda.h"
#include "xchg.cuh"

struct satori_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;     // current stream (own or caller's)
    cudaStream_t own_stream = nullptr;
    int sm_count = 0;
    size_t smem_optin = 0;
    unsigned *d_err = nullptr;         // device error word (bounded waits)
    int *d_status = nullptr;           // validation status scratch
    float *attn_scratch = nullptr;     // grow-only partial records for one-shot attention calls
    size_t attn_scratch_floats = 0;
    // Weights the next MatVec of a captured sequence will stream: the current launch prefetches their
    // head into L2 during its tail.  Set by the caller just before run_gemv, consumed (cleared) by it.
    const uint8_t *next_payload = nullptr;
    size_t next_bytes = 0;
    uint8_t *tc_scratch = nullptr;     // grow-only split activations + split-K tiles of tensor-order calls
    size_t tc_scratch_bytes = 0;
};

struct satori_matrix {
    satori_ctx *ctx = nullptr;
    uint8_t *d_payload = nullptr;
    size_t bytes = 0;
    int rows = 0, cols = 0, format = 0;
    float *d_x = nullptr, *d_y = nullptr;     // device work vectors for host-pointer calls
    float *h_x = nullptr, *h_y = nullptr;     // pinned staging
    size_t cap_positions = 0;
};

namespace satori {

int set_error(int status, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);

// Makes a handle's device current for one entry point and gives the caller's device back at the end:
// a process may hold contexts on several GPUs and call the library from any thread, and allocations,
// copies and launches must land on the handle's device.  When that device is already current (one GPU
// per process) nothing changes.  The device-pointer entry points do not take one: they work on the
// caller's current device, which a caller capturing them into a CUDA graph has already chosen.
struct DeviceScope {
    int prev = -1, dev;
    cudaError_t status = cudaSuccess;
    explicit DeviceScope(int device) : dev(device)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) status = cudaSetDevice(dev);
    }
    ~DeviceScope()
    {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
    DeviceScope(const DeviceScope &) = delete;
    DeviceScope &operator=(const DeviceScope &) = delete;
};

// Clears the context's device error word on its stream.
cudaError_t clear_dev_error(satori_ctx *ctx);
// Reads the device error word (synchronises the stream) and maps it to a status.
int check_dev_error(satori_ctx *ctx);
bool is_valid_format(int format);
size_t payload_bytes(int rows, int cols, int format);
int validate_shape(int rows, int cols, int format);
// Uploads and validates a payload; on success *out owns a device copy padded for bulk copies.
int upload_payload(satori_ctx *ctx, const uint8_t *src, bool src_is_device, size_t bytes, int rows, int cols,
                   int format, uint8_t **out);
// Grows the context's tensor-order scratch to at least `bytes`.
int ensure_tc_scratch(satori_ctx *ctx, size_t bytes);
// Runs the MatVec on device pointers with the library's plan for this shape.
int run_gemv(satori_ctx *ctx, const uint8_t *d_payload, int rows, int cols, int format, int order,
             const float *dx, float *dy, int positions, int epilogue, const float *bias, float *residual,
             cudaStream_t stream, int use_pdl, const float *norm_w = nullptr, float norm_eps = 0.0f,
             const XPush *xp = nullptr, const XWait *xw = nullptr);

}  // namespace satori
