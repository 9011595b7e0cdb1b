// capi.cu -- C ABI: contexts, resident matrices, quantizers and attention entry points.
//
// Every entry point validates its arguments the way the reference's public API does (and
// returns the status the matching C# exception maps to), never writes a caller output unless the
// whole call succeeded, and routes all device work through the context's stream.
#include "attention.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "gemv.cuh"

#include <math.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#define SATORI_VERSION "0.1.0"

namespace {
thread_local std::string g_last_error;
}

namespace satori {

int set_error(int status, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what)
{
    cudaGetLastError();  // clear a non-sticky error so it does not surface in a later, unrelated call
    if (e == cudaErrorMemoryAllocation)
        return set_error(SATORI_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return set_error(SATORI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

cudaError_t opt_in_smem(const void *kernel, size_t bytes)
{
    if (bytes <= 48 * 1024) return cudaSuccess;   // the default limit needs no opt-in
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex lock;
    static std::map<std::pair<const void *, int>, size_t> granted;
    std::lock_guard<std::mutex> guard(lock);
    size_t &have = granted[std::make_pair(kernel, dev)];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

cudaError_t clear_dev_error(satori_ctx *ctx) { return cudaMemsetAsync(ctx->d_err, 0, sizeof(unsigned), ctx->stream); }

int check_dev_error(satori_ctx *ctx)
{
    unsigned err = 0;
    cudaError_t e = cudaMemcpyAsync(&err, ctx->d_err, sizeof err, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "synchronize");
    if (err & kDevErrTimeout) return set_error(SATORI_ERR_TIMEOUT, "a bounded device wait expired");
    return SATORI_OK;
}

bool is_valid_format(int f)
{
    return f == SATORI_Q8_0 || f == SATORI_Q4_0 || f == SATORI_Q4_K || f == SATORI_Q6_K || f == 64 || f == 128 ||
           f == 256 || is_bitplane(f);
}

size_t payload_bytes(int rows, int cols, int format)
{
    const int be = gemv_block_elems(format), bb = gemv_block_bytes(format);
    return (size_t)rows * (size_t)((cols + be - 1) / be) * (size_t)bb;
}

// QuantizedMatrixShape (src/Satori.Core/QuantizedMatrixShape.cs:5-22) and Ternary2Shape
// (src/Satori.Core/Ternary2Shape.cs:5-15): positive dimensions, complete 32-weight GGUF rows,
// supported block size, byte length within Int32.
int validate_shape(int rows, int cols, int format)
{
    if (!is_valid_format(format)) return set_error(SATORI_ERR_ARGUMENT, "unsupported format %d", format);
    if (rows <= 0 || cols <= 0) return set_error(SATORI_ERR_ARGUMENT, "dimensions must be positive");
    if (format <= 1 && cols % 32 != 0)
        return set_error(SATORI_ERR_ARGUMENT, "complete 32-weight rows required (cols=%d)", cols);
    if (is_kquant(format) && cols % 256 != 0)
        return set_error(SATORI_ERR_ARGUMENT, "Columns must be a positive multiple of 256 (cols=%d)", cols);
    if (payload_bytes(rows, cols, format) > 0x7fffffffull)
        return set_error(SATORI_ERR_ARGUMENT, "payload exceeds Int32 limits");
    return SATORI_OK;
}

int upload_payload(satori_ctx *ctx, const uint8_t *src, bool src_is_device, size_t bytes, int rows, int cols,
                   int format, uint8_t **out)
{
    int rc = validate_shape(rows, cols, format);
    if (rc) return rc;
    if (!src) return set_error(SATORI_ERR_ARGUMENT, "payload is null");
    if (bytes != payload_bytes(rows, cols, format))
        return set_error(SATORI_ERR_ARGUMENT, "payload length %zu does not match the %dx%d shape (%zu)", bytes, rows,
                         cols, payload_bytes(rows, cols, format));
    uint8_t *d = nullptr;
    // Padding: the MatVec reads whole 16-byte granules around each row segment.
    cudaError_t e = cudaMalloc(&d, bytes + 256);
    if (e != cudaSuccess) return cuda_fail(e, "allocate payload");
    e = cudaMemsetAsync(d + bytes, 0, 256, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d, src, bytes, src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_status, 0, sizeof(int), ctx->stream);
    if (e == cudaSuccess) e = launch_validate(d, rows, cols, format, ctx->d_status, ctx->stream);
    int status = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "upload payload");
    }
    if (status != 0) {
        cudaFree(d);
        // Quantized: InvalidDataException (QuantizedMatVec.cs:40).  Ternary2 import from a packed
        // buffer: ArgumentException (Ternary2Matrix.cs:92,98); the mapped STQ2 path rethrows it as
        // InvalidDataException (MappedTernary2Matrix.cs:25-28), which the Python mirror does.
        const bool gguf = format <= 1 || is_kquant(format);
        return set_error(gguf ? SATORI_ERR_INVALID_DATA : SATORI_ERR_ARGUMENT,
                         gguf ? "non-finite block scale" : "invalid block scale, weight code or padding");
    }
    *out = d;
    return SATORI_OK;
}

// SATORI_GEMV_STREAM=0 routes every decode MatVec to gemv_rows (both kernels give the same bits).
bool stream_kernel_enabled()
{
    static const bool on = [] {
        const char *v = getenv("SATORI_GEMV_STREAM");
        return !(v && strcmp(v, "0") == 0);
    }();
    return on;
}

bool gemv_fused_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit)
{
    return (stream_kernel_enabled() && gemv_stream_takes(rows, cols, format, epilogue, sm_count, smem_limit)) ||
           gemv_rows_takes(rows, cols, format, epilogue, sm_count, smem_limit);
}

int run_gemv(satori_ctx *ctx, const uint8_t *d_payload, int rows, int cols, int format, int order, const float *dx,
             float *dy, int positions, int epilogue, const float *bias, float *residual, cudaStream_t stream,
             int use_pdl, const float *norm_w, float norm_eps, const XPush *xp, const XWait *xw)
{
    // The caller's hint about the next MatVec of its sequence applies to this call only.
    const uint8_t *hint = ctx->next_payload;
    const size_t hint_bytes = hint ? ctx->next_bytes : 0;
    ctx->next_payload = nullptr;
    ctx->next_bytes = 0;
    if (order == SATORI_ORDER_TENSOR) {
        if (norm_w || xp || xw)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "the tensor order takes no fused RmsNorm or exchange");
        if (!tc_gemm_takes(rows, cols, format, 1, epilogue))
            return set_error(SATORI_ERR_NOT_SUPPORTED,
                             "the tensor order takes Q8_0 / Q4_0 with a multiple of 64 columns");
        for (int p0 = 0; p0 < positions; p0 += 128) {
            const int np = std::min(128, positions - p0);
            const size_t need = tc_scratch_bytes(rows, cols, np, ctx->sm_count);
            int rc = ensure_tc_scratch(ctx, need);
            if (rc) return rc;
            TcGemm g = {};
            g.payload = d_payload;
            g.rows = rows;
            g.cols = cols;
            g.format = format;
            g.x = dx + (size_t)p0 * cols;
            g.positions = np;
            g.epilogue = epilogue;
            const int ldy = epilogue == kEpiSwiGlu ? rows / 2 : rows;
            g.y = dy ? dy + (size_t)p0 * ldy : nullptr;
            g.bias = bias;
            g.residual = residual ? residual + (size_t)p0 * rows : nullptr;
            g.scratch = ctx->tc_scratch;
            g.scratch_bytes = ctx->tc_scratch_bytes;
            g.err = ctx->d_err;
            cudaError_t e = launch_tc_gemm(g, ctx->sm_count, stream);
            if (e != cudaSuccess) return cuda_fail(e, "launch tensor-core projection");
        }
        return SATORI_OK;
    }
    if (is_kquant(format)) {
        if (norm_w || xp || xw || epilogue == kEpiSwiGlu)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "fused RmsNorm / SwiGLU / exchange are not available for K-quants");
        if (order != SATORI_ORDER_BATCH && epilogue != kEpiNone)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "K-quant epilogues need the batch order");
        if (cols > 32768) return set_error(SATORI_ERR_NOT_SUPPORTED, "K-quant rows wider than 32768 columns");
        // Positions are independent in every order (one accumulator per position), so one launch each.
        for (int p = 0; p < positions; ++p) {
            GemvArgs a = {};
            a.payload = d_payload;
            a.rows = rows;
            a.cols = cols;
            a.format = format;
            a.order = order;
            a.x = dx + (size_t)p * cols;
            a.y = dy + (size_t)p * rows;
            a.positions = 1;
            a.epilogue = epilogue;
            a.bias = bias;
            a.residual = residual;
            a.err = ctx->d_err;
            a.use_pdl = use_pdl;
            cudaError_t e = launch_kq_gemv(a, stream);
            if (e != cudaSuccess) return cuda_fail(e, "launch K-quant MatVec");
        }
        return SATORI_OK;
    }
    if (format >= 64) {
        // Ternary2 / bitplane: the row-streaming kernel takes the AVX2 order on whole blocks; bitplane
        // matrices otherwise use the row-per-thread kernel, Ternary2 the general kernel below.
        if (order == SATORI_ORDER_BATCH)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "ExecuteBatch is defined for the GGUF formats only");
        if (epilogue != kEpiNone || norm_w || xp || xw || positions != 1)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "ternary MatVec takes one position and no epilogue");
        GemvArgs a = {};
        a.payload = d_payload;
        a.rows = rows;
        a.cols = cols;
        a.format = format;
        a.order = order;
        a.x = dx;
        a.y = dy;
        a.positions = 1;
        a.epilogue = kEpiNone;
        a.err = ctx->d_err;
        a.use_pdl = use_pdl;
        bool taken = false;
        cudaError_t e = launch_ternary_stream(a, ctx->sm_count, ctx->smem_optin, stream, &taken);
        if (e != cudaSuccess) return cuda_fail(e, "launch ternary MatVec");
        if (taken) return SATORI_OK;
        if (is_bitplane(format)) {
            e = launch_bitplane_rowwise(a, stream);
            return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "launch bitplane MatVec");
        }
    }
    const int per_launch = order == SATORI_ORDER_BATCH ? 8 : 1;
    for (int p0 = 0; p0 < positions; p0 += per_launch) {
        const int np = std::min(per_launch, positions - p0);
        if (order == SATORI_ORDER_BATCH && np == 1) {
            // One decode position: the dedicated kernel when the shape qualifies.
            GemvArgs a = {};
            a.payload = d_payload;
            a.rows = rows;
            a.cols = cols;
            a.format = format;
            a.order = order;
            a.x = dx + (size_t)p0 * cols;
            a.y = dy + (size_t)p0 * rows;
            a.positions = 1;
            a.epilogue = epilogue;
            a.bias = bias;
            a.residual = residual;
            a.err = ctx->d_err;
            a.use_pdl = use_pdl;
            a.norm_w = norm_w;
            a.norm_eps = norm_eps;
            if (xp) a.xp = *xp;
            if (xw) a.xw = *xw;
            a.next_payload = hint;
            a.next_bytes = hint_bytes;
            DecodePlan dp = {};
            if (stream_kernel_enabled()) {
                dp = plan_gemv_stream(a, ctx->sm_count, ctx->smem_optin);
                if (dp.ok) {
                    cudaError_t e = launch_gemv_stream(a, dp, stream);
                    if (e != cudaSuccess) return cuda_fail(e, "launch decode MatVec");
                    continue;
                }
            }
            dp = plan_gemv_rows(a, ctx->sm_count, ctx->smem_optin);
            if (dp.ok) {
                cudaError_t e = launch_gemv_rows(a, dp, stream);
                if (e != cudaSuccess) return cuda_fail(e, "launch decode MatVec");
                continue;
            }
            if (norm_w || xp || xw)
                return set_error(SATORI_ERR_NOT_SUPPORTED, "fused RmsNorm / peer exchange need the decode rows kernel");
            dp = plan_gemv_decode(a, ctx->sm_count, ctx->smem_optin);
            if (dp.ok) {
                cudaError_t e = launch_gemv_decode(a, dp, stream);
                if (e != cudaSuccess) return cuda_fail(e, "launch decode MatVec");
                continue;
            }
        }
        if (epilogue == kEpiSwiGlu || norm_w || xp || xw)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "fused SwiGLU / RmsNorm / exchange need the decode rows kernel");
        GemvPlan plan = plan_gemv(rows, cols, format, np, ctx->sm_count, ctx->smem_optin);
        if (!plan.ok) return set_error(SATORI_ERR_ARGUMENT, "no MatVec plan fits shared memory for %dx%d", rows, cols);
        GemvArgs a = {};
        a.payload = d_payload;
        a.rows = rows;
        a.cols = cols;
        a.format = format;
        a.order = order;
        a.x = dx + (size_t)p0 * cols;
        a.y = dy + (size_t)p0 * rows;
        a.positions = np;
        a.epilogue = epilogue;
        a.bias = bias;
        a.residual = residual;
        a.err = ctx->d_err;
        a.use_pdl = use_pdl;
        cudaError_t e = launch_gemv(a, plan, stream);
        if (e != cudaSuccess) return cuda_fail(e, "launch MatVec");
    }
    return SATORI_OK;
}

}  // namespace satori

using namespace satori;

// ============================================================================ context
extern "C" int satori_last_error(char *buf, size_t n)
{
    if (!buf || n == 0) return SATORI_ERR_ARGUMENT;
    snprintf(buf, n, "%s", g_last_error.c_str());
    return SATORI_OK;
}

extern "C" int satori_version(char *buf, size_t n)
{
    if (!buf || n == 0) return SATORI_ERR_ARGUMENT;
    snprintf(buf, n, "satori-b200 %s sm_100a", SATORI_VERSION);
    return SATORI_OK;
}

extern "C" int satori_init(int device, satori_ctx **out)
{
    if (!out) return set_error(SATORI_ERR_ARGUMENT, "out is null");
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) return set_error(SATORI_ERR_ARGUMENT, "device %d out of range (%d)", device, count);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "device %d is sm_%d%d; this build is sm_100a only", device,
                         prop.major, prop.minor);
    satori_ctx *ctx = new satori_ctx();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->smem_optin = prop.sharedMemPerBlockOptin;
    e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    ctx->stream = ctx->own_stream;
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(unsigned));
    if (e != cudaSuccess) {
        int rc = cuda_fail(e, "initialise context");
        satori_destroy(ctx);
        return rc;
    }
    *out = ctx;
    return SATORI_OK;
}

extern "C" int satori_destroy(satori_ctx *ctx)
{
    if (!ctx) return SATORI_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_status);
    cudaFree(ctx->attn_scratch);
    cudaFree(ctx->tc_scratch);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return SATORI_OK;
}

extern "C" void *satori_stream(satori_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

extern "C" int satori_set_stream(satori_ctx *ctx, void *stream)
{
    if (!ctx) return set_error(SATORI_ERR_ARGUMENT, "ctx is null");
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return SATORI_OK;
}

extern "C" int satori_synchronize(satori_ctx *ctx)
{
    if (!ctx) return set_error(SATORI_ERR_ARGUMENT, "ctx is null");
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    return check_dev_error(ctx);
}

// ============================================================================ matrices
static int matrix_create(satori_ctx *ctx, const uint8_t *payload, bool dev, size_t bytes, int rows, int cols,
                         int format, satori_matrix **out)
{
    if (!ctx || !out) return set_error(SATORI_ERR_ARGUMENT, "ctx/out is null");
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    uint8_t *d = nullptr;
    int rc = upload_payload(ctx, payload, dev, bytes, rows, cols, format, &d);
    if (rc) return rc;
    satori_matrix *m = new satori_matrix();
    m->ctx = ctx;
    m->d_payload = d;
    m->bytes = bytes;
    m->rows = rows;
    m->cols = cols;
    m->format = format;
    *out = m;
    return SATORI_OK;
}

extern "C" int satori_matrix_create(satori_ctx *ctx, const uint8_t *payload, size_t bytes, int rows, int cols,
                                    int format, satori_matrix **out)
{
    return matrix_create(ctx, payload, false, bytes, rows, cols, format, out);
}

extern "C" int satori_matrix_create_device(satori_ctx *ctx, const uint8_t *payload, size_t bytes, int rows, int cols,
                                           int format, satori_matrix **out)
{
    return matrix_create(ctx, payload, true, bytes, rows, cols, format, out);
}

static int ensure_work(satori_matrix *m, int positions)
{
    if ((size_t)positions <= m->cap_positions) return SATORI_OK;
    cudaFree(m->d_x);
    cudaFree(m->d_y);
    cudaFreeHost(m->h_x);
    cudaFreeHost(m->h_y);
    m->d_x = m->d_y = m->h_x = m->h_y = nullptr;
    m->cap_positions = 0;
    const size_t nx = (size_t)positions * m->cols, ny = (size_t)positions * m->rows;
    cudaError_t e = cudaMalloc(&m->d_x, nx * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->d_y, ny * 4);
    if (e == cudaSuccess) e = cudaHostAlloc(&m->h_x, nx * 4, cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaHostAlloc(&m->h_y, ny * 4, cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_fail(e, "allocate MatVec work vectors");
    m->cap_positions = positions;
    return SATORI_OK;
}

static int matrix_execute_host(satori_matrix *m, const float *x, float *y, int positions, int order)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (!x || !y) return set_error(SATORI_ERR_ARGUMENT, "vector is null");
    if (positions <= 0) return set_error(SATORI_ERR_ARGUMENT, "positions must be positive");
    // Input and output must not overlap (QuantizedMatVec.cs:84, Ternary2MatVec.cs:34-35).
    const char *xb = (const char *)x, *xe = xb + (size_t)positions * m->cols * 4;
    const char *yb = (const char *)y, *ye = yb + (size_t)positions * m->rows * 4;
    if (xb < ye && yb < xe) return set_error(SATORI_ERR_ARGUMENT, "output must not overlap input");
    satori_ctx *ctx = m->ctx;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    int rc = ensure_work(m, positions);
    if (rc) return rc;
    memcpy(m->h_x, x, (size_t)positions * m->cols * 4);
    cudaError_t e = clear_dev_error(ctx);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->d_x, m->h_x, (size_t)positions * m->cols * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy input");
    rc = run_gemv(ctx, m->d_payload, m->rows, m->cols, m->format, order, m->d_x, m->d_y, positions, kEpiNone, nullptr,
                  nullptr, ctx->stream, 0);
    if (rc) return rc;
    e = cudaMemcpyAsync(m->h_y, m->d_y, (size_t)positions * m->rows * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy output");
    rc = check_dev_error(ctx);
    if (rc) return rc;
    memcpy(y, m->h_y, (size_t)positions * m->rows * 4);  // commit only on success
    return SATORI_OK;
}

extern "C" int satori_matrix_execute(satori_matrix *m, const float *x, float *y)
{
    return matrix_execute_host(m, x, y, 1, SATORI_ORDER_EXECUTE);
}

extern "C" int satori_matrix_execute_scalar(satori_matrix *m, const float *x, float *y)
{
    return matrix_execute_host(m, x, y, 1, SATORI_ORDER_SCALAR);
}

extern "C" int satori_matrix_execute_batch(satori_matrix *m, const float *x, int positions, float *y)
{
    if (m && m->format >= 64)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "ExecuteBatch is defined for the GGUF formats only");
    return matrix_execute_host(m, x, y, positions, SATORI_ORDER_BATCH);
}

extern "C" int satori_matrix_execute_tensor(satori_matrix *m, const float *x, int positions, float *y)
{
    if (m && m->format != SATORI_Q8_0 && m->format != SATORI_Q4_0)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "the tensor order is defined for Q8_0 / Q4_0");
    return matrix_execute_host(m, x, y, positions, SATORI_ORDER_TENSOR);
}

extern "C" int satori_matrix_execute_device(satori_matrix *m, const float *dx, float *dy, int positions, int order)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (!dx || !dy || positions <= 0) return set_error(SATORI_ERR_ARGUMENT, "bad device vectors/positions");
    if (order < 0 || order > 3) return set_error(SATORI_ERR_ARGUMENT, "bad order %d", order);
    if (order == SATORI_ORDER_TENSOR && m->format != SATORI_Q8_0 && m->format != SATORI_Q4_0)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "the tensor order is defined for Q8_0 / Q4_0");
    if (order < SATORI_ORDER_BATCH && positions != 1)
        return set_error(SATORI_ERR_ARGUMENT, "only the batch order takes several positions");
    if (order == SATORI_ORDER_BATCH && m->format >= 64)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "ExecuteBatch is defined for the GGUF formats only");
    // Launched with programmatic dependent launch: the kernel streams its weights while the previous
    // kernel on the stream finishes, and waits for it before reading x or writing y.
    return run_gemv(m->ctx, m->d_payload, m->rows, m->cols, m->format, order, dx, dy, positions, kEpiNone, nullptr,
                    nullptr, m->ctx->stream, 1);
}

extern "C" int satori_matrix_read_row(satori_matrix *m, int row, float *out)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (m->format == SATORI_Q4_0) return set_error(SATORI_ERR_NOT_SUPPORTED, "Q4_0 embedding rows are not supported");
    if (row < 0 || row >= m->rows || !out) return set_error(SATORI_ERR_ARGUMENT, "row %d out of range", row);
    DeviceScope scope(m->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    int rc = ensure_work(m, 1);
    if (rc) return rc;
    satori_ctx *ctx = m->ctx;
    cudaError_t e = launch_decode_row(m->d_payload, m->rows, m->cols, m->format, nullptr, row, m->d_x, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->h_x, m->d_x, (size_t)m->cols * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "decode row");
    memcpy(out, m->h_x, (size_t)m->cols * 4);
    return SATORI_OK;
}

extern "C" int satori_matrix_info(const satori_matrix *m, int *rows, int *cols, int *format, size_t *bytes)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (rows) *rows = m->rows;
    if (cols) *cols = m->cols;
    if (format) *format = m->format;
    if (bytes) *bytes = m->bytes;
    return SATORI_OK;
}

extern "C" const uint8_t *satori_matrix_device_payload(const satori_matrix *m) { return m ? m->d_payload : nullptr; }

extern "C" int satori_matrix_destroy(satori_matrix *m)
{
    if (!m) return SATORI_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(m->d_payload);
    cudaFree(m->d_x);
    cudaFree(m->d_y);
    cudaFreeHost(m->h_x);
    cudaFreeHost(m->h_y);
    delete m;
    return SATORI_OK;
}

// ============================================================================ quantizers
extern "C" int satori_ternary2_quantize(satori_ctx *ctx, const float *weights, int rows, int cols, int block_size,
                                        uint8_t *payload)
{
    if (!ctx || !weights || !payload) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (block_size != 64 && block_size != 128 && block_size != 256)
        return set_error(SATORI_ERR_ARGUMENT, "Supported block sizes: 64, 128, 256.");
    int rc = validate_shape(rows, cols, block_size);
    if (rc) return rc;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    const size_t n = (size_t)rows * cols, bytes = payload_bytes(rows, cols, block_size);
    float *dw = nullptr;
    uint8_t *dp = nullptr;
    int status = 0;
    cudaError_t e = cudaMalloc(&dw, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dp, bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dw, weights, n * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_status, 0, sizeof(int), ctx->stream);
    if (e == cudaSuccess) e = launch_t2_quantize(dw, rows, cols, block_size, dp, ctx->d_status, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
    std::vector<uint8_t> host(bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host.data(), dp, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(dw);
    cudaFree(dp);
    if (e != cudaSuccess) return cuda_fail(e, "quantize");
    if (status) return set_error(SATORI_ERR_ARGUMENT, "Weights must be finite.");
    memcpy(payload, host.data(), bytes);
    return SATORI_OK;
}

extern "C" int satori_quantize_q_device(satori_ctx *ctx, const float *d_weights, int rows, int cols, int format,
                                        uint8_t *d_payload)
{
    if (!ctx || !d_weights || !d_payload) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (format != SATORI_Q8_0 && format != SATORI_Q4_0) return set_error(SATORI_ERR_ARGUMENT, "Q8_0/Q4_0 only");
    int rc = validate_shape(rows, cols, format);
    if (rc) return rc;
    cudaError_t e = launch_q_quantize(d_weights, rows, cols, format, d_payload, ctx->stream);
    return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "quantize");
}

// ============================================================================ attention
static int attention_args_ok(int q_heads, int kv_heads, int head_dim, int tokens)
{
    // TransformerOps.GroupedAttention's dimension checks (TransformerOps.cs:143-151).
    if (head_dim <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || tokens <= 0)
        return set_error(SATORI_ERR_ARGUMENT, "Invalid grouped-attention dimensions.");
    if (head_dim > 256) return set_error(SATORI_ERR_NOT_SUPPORTED, "head_dim > 256 is not supported");
    return SATORI_OK;
}

int satori::ensure_tc_scratch(satori_ctx *ctx, size_t bytes)
{
    if (bytes <= ctx->tc_scratch_bytes) return SATORI_OK;
    // Earlier launches on the stream may still read the old buffer.
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "synchronise before growing scratch");
    cudaFree(ctx->tc_scratch);
    ctx->tc_scratch = nullptr;
    ctx->tc_scratch_bytes = 0;
    e = cudaMalloc(&ctx->tc_scratch, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "allocate tensor-order scratch");
    ctx->tc_scratch_bytes = bytes;
    return SATORI_OK;
}

static int ensure_attn_scratch(satori_ctx *ctx, size_t floats)
{
    if (floats <= ctx->attn_scratch_floats) return SATORI_OK;
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->attn_scratch);
    ctx->attn_scratch = nullptr;
    ctx->attn_scratch_floats = 0;
    cudaError_t e = cudaMalloc(&ctx->attn_scratch, floats * 4);
    if (e != cudaSuccess) return cuda_fail(e, "allocate attention scratch");

    ctx->attn_scratch_floats = floats;
    return SATORI_OK;
}

extern "C" int satori_grouped_attention_device(satori_ctx *ctx, const float *q, const float *keys,
                                               const float *values, int q_heads, int kv_heads, int head_dim,
                                               int tokens, float *out)
{
    if (!ctx || !q || !keys || !values || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    int rc = attention_args_ok(q_heads, kv_heads, head_dim, tokens);
    if (rc) return rc;
    rc = ensure_attn_scratch(ctx, attn_scratch_floats(q_heads, kv_heads, head_dim, tokens, ctx->sm_count));
    if (rc) return rc;
    AttnArgs a = {};
    a.q = q;
    a.keys = keys;
    a.values = values;
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.tokens = tokens;
    a.max_tokens = tokens;
    a.out = out;
    a.scratch = ctx->attn_scratch;
    a.err = ctx->d_err;
    a.use_pdl = 1;
    cudaError_t e = launch_attention(a, ctx->sm_count, ctx->stream);
    return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "launch attention");
}

extern "C" int satori_grouped_attention(satori_ctx *ctx, const float *q, const float *keys, const float *values,
                                        int q_heads, int kv_heads, int head_dim, int tokens, float *out)
{
    if (!ctx || !q || !keys || !values || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    int rc = attention_args_ok(q_heads, kv_heads, head_dim, tokens);
    if (rc) return rc;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    const size_t nq = (size_t)q_heads * head_dim, nkv = (size_t)tokens * kv_heads * head_dim;
    float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
    cudaError_t e = cudaMalloc(&dq, nq * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dk, nkv * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dv, nkv * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dout, nq * 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dk, keys, nkv * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv, values, nkv * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = clear_dev_error(ctx);
    std::vector<float> host(nq);
    if (e == cudaSuccess) {
        rc = satori_grouped_attention_device(ctx, dq, dk, dv, q_heads, kv_heads, head_dim, tokens, dout);
        if (rc == SATORI_OK) {
            e = cudaMemcpyAsync(host.data(), dout, nq * 4, cudaMemcpyDeviceToHost, ctx->stream);
            if (e == cudaSuccess) rc = check_dev_error(ctx);
        }
    }
    cudaStreamSynchronize(ctx->stream);
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dout);
    if (e != cudaSuccess) return cuda_fail(e, "grouped attention");
    if (rc) return rc;
    memcpy(out, host.data(), nq * 4);
    return SATORI_OK;
}

extern "C" int satori_rope_half(satori_ctx *ctx, float *vector, int n, int head_dim, int position, double base,
                                int rotary)
{
    if (!ctx || !vector) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    // TransformerOps.RopeHalf argument checks (TransformerOps.cs:101-105).
    if (head_dim <= 0 || n % head_dim != 0 || position < 0) return set_error(SATORI_ERR_ARGUMENT, "headDimension");
    if (!(base > 0) || isinf(base)) return set_error(SATORI_ERR_ARGUMENT, "frequencyBase");
    if (rotary <= 0 || rotary > head_dim || rotary % 2 != 0) return set_error(SATORI_ERR_ARGUMENT, "rotaryDimensions");
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    float *d = nullptr;
    std::vector<float> host(n);
    cudaError_t e = cudaMalloc(&d, (size_t)n * 4 + 4);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d, vector, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = launch_rope_half(d, n, head_dim, position, base, rotary, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host.data(), d, (size_t)n * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e, "rope");
    memcpy(vector, host.data(), (size_t)n * 4);
    return SATORI_OK;
}

// ============================================================================ KV cache + attention step
struct satori_attn {
    satori_ctx *ctx = nullptr;
    int layers = 0, context = 0, q_heads = 0, kv_heads = 0, head_dim = 0;
    double rope_base = 0;
    float *d_k = nullptr, *d_v = nullptr;  // [layers][context][kv_width]
    float *d_q = nullptr, *d_kin = nullptr, *d_vin = nullptr, *d_qrot = nullptr, *d_out = nullptr;
    float *d_scratch = nullptr;
};

extern "C" int satori_attn_create(satori_ctx *ctx, int layers, int context, int q_heads, int kv_heads, int head_dim,
                                  double rope_base, satori_attn **out)
{
    if (!ctx || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (layers <= 0 || context <= 0) return set_error(SATORI_ERR_ARGUMENT, "layers/context must be positive");
    int rc = attention_args_ok(q_heads, kv_heads, head_dim, 1);
    if (rc) return rc;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    satori_attn *a = new satori_attn();
    a->ctx = ctx;
    a->layers = layers;
    a->context = context;
    a->q_heads = q_heads;
    a->kv_heads = kv_heads;
    a->head_dim = head_dim;
    a->rope_base = rope_base;
    const size_t kvw = (size_t)kv_heads * head_dim, qw = (size_t)q_heads * head_dim;
    const size_t cache = (size_t)layers * context * kvw;
    cudaError_t e = cudaMalloc(&a->d_k, cache * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_v, cache * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_q, qw * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_qrot, qw * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_out, qw * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_kin, kvw * 4);
    if (e == cudaSuccess) e = cudaMalloc(&a->d_vin, kvw * 4);
    if (e == cudaSuccess)
        e = cudaMalloc(&a->d_scratch, attn_scratch_floats(q_heads, kv_heads, head_dim, context, ctx->sm_count) * 4);
    if (e != cudaSuccess) {
        rc = cuda_fail(e, "allocate attention state");
        satori_attn_destroy(a);
        return rc;
    }
    *out = a;
    return SATORI_OK;
}

extern "C" int satori_attn_append(satori_attn *a, int layer, int position, const float *q, const float *k,
                                  const float *v, float *out)
{
    if (!a) return set_error(SATORI_ERR_DISPOSED, "attention state is disposed");
    if (!q || !k || !v || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (layer < 0 || layer >= a->layers) return set_error(SATORI_ERR_ARGUMENT, "layer out of range");
    if (position < 0) return set_error(SATORI_ERR_ARGUMENT, "position out of range");
    if (position >= a->context)
        return set_error(SATORI_ERR_CONTEXT_FULL, "Context limit %d reached; reset or enlarge the session.", a->context);
    satori_ctx *ctx = a->ctx;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    const size_t kvw = (size_t)a->kv_heads * a->head_dim, qw = (size_t)a->q_heads * a->head_dim;
    float *kc = a->d_k + (size_t)layer * a->context * kvw, *vc = a->d_v + (size_t)layer * a->context * kvw;
    cudaError_t e = clear_dev_error(ctx);
    if (e == cudaSuccess) e = cudaMemcpyAsync(a->d_q, q, qw * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(a->d_kin, k, kvw * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(a->d_vin, v, kvw * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy q/k/v");
    RopeAppendArgs r = {};
    r.q = a->d_q;
    r.k = a->d_kin;
    r.v = a->d_vin;
    r.q_out = a->d_qrot;
    r.k_cache = kc;
    r.v_cache = vc;
    r.q_heads = a->q_heads;
    r.kv_heads = a->kv_heads;
    r.head_dim = a->head_dim;
    r.rotary = a->head_dim;
    r.base = a->rope_base;
    r.position = position;
    e = launch_rope_append(r, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "rope/append");
    AttnArgs at = {};
    at.q = a->d_qrot;
    at.keys = kc;
    at.values = vc;
    at.q_heads = a->q_heads;
    at.kv_heads = a->kv_heads;
    at.head_dim = a->head_dim;
    at.tokens = position + 1;
    at.max_tokens = a->context;
    at.out = a->d_out;
    at.scratch = a->d_scratch;
    at.err = ctx->d_err;
    e = launch_attention(at, ctx->sm_count, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "attention");
    std::vector<float> host(qw);
    e = cudaMemcpyAsync(host.data(), a->d_out, qw * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy output");
    int rc = check_dev_error(ctx);
    if (rc) return rc;
    memcpy(out, host.data(), qw * 4);
    return SATORI_OK;
}

extern "C" int satori_attn_destroy(satori_attn *a)
{
    if (!a) return SATORI_OK;
    cudaSetDevice(a->ctx->device);
    cudaStreamSynchronize(a->ctx->stream);
    cudaFree(a->d_k);
    cudaFree(a->d_v);
    cudaFree(a->d_q);
    cudaFree(a->d_qrot);
    cudaFree(a->d_out);
    cudaFree(a->d_kin);
    cudaFree(a->d_vin);
    cudaFree(a->d_scratch);
    delete a;
    return SATORI_OK;
}
