// matrix_sharded.cu -- one large MatVec split by rows over the GPUs of a node, one process per GPU.
//
// Rank r of `world` holds rows [r*S, min((r+1)*S, rows)) of the matrix, S = ceil(rows / world): a
// contiguous byte range of the GGUF / STQ2 payload, uploaded and validated like any matrix.  Every rank
// computes its rows with the single-GPU kernels (so each row keeps the reference's FP32 operation order
// bit for bit) into its slice of the output, and an NCCL all-gather gives every rank the full vector.
// When S does not divide `rows` the gather runs on a padded buffer and the first `rows` values are
// copied out.  All ranks call execute together, in the same order (it is a collective).
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "capi_internal.h"
#include "nccl_api.h"

using namespace satori;

struct satori_matrix_sharded {
    satori_ctx *ctx = nullptr;
    satori_matrix *local = nullptr;      // this rank's row block
    int rows = 0, cols = 0, format = 0, rank = 0, world = 1;
    int r0 = 0, r1 = 0, slice = 0;       // this rank's rows [r0, r1); every slice is `slice` rows long
    ncclComm_t comm = nullptr;
    float *d_gather = nullptr;           // [world * slice] when slice * world != rows
    float *d_x = nullptr, *d_y = nullptr;  // work vectors of the host-pointer call
    float *h_x = nullptr, *h_y = nullptr;
};

extern "C" int satori_matrix_sharded_destroy(satori_matrix_sharded *m)
{
    if (!m) return SATORI_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->local) satori_matrix_destroy(m->local);
    const NcclApi *api = nccl_api();
    if (api && m->comm) api->CommDestroy(m->comm);
    cudaFree(m->d_gather);
    cudaFree(m->d_x);
    cudaFree(m->d_y);
    cudaFreeHost(m->h_x);
    cudaFreeHost(m->h_y);
    delete m;
    return SATORI_OK;
}

extern "C" int satori_matrix_create_sharded(satori_ctx *ctx, const uint8_t *payload, size_t bytes, int rows, int cols,
                                            int format, int payload_on_device, int rank, int world,
                                            const void *nccl_unique_id, satori_matrix_sharded **out)
{
    if (!ctx || !payload || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (world < 1 || rank < 0 || rank >= world) return set_error(SATORI_ERR_ARGUMENT, "bad rank %d / world %d", rank, world);
    int rc = validate_shape(rows, cols, format);
    if (rc) return rc;
    if (bytes != payload_bytes(rows, cols, format))
        return set_error(SATORI_ERR_ARGUMENT, "Payload length must match matrix dimensions.");
    const int slice = (rows + world - 1) / world;
    if ((long long)slice * (world - 1) >= rows)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "%d rows leave rank %d of %d without rows", rows, world - 1, world);
    if (world > 1 && !nccl_unique_id) return set_error(SATORI_ERR_ARGUMENT, "nccl_unique_id is null");
    const size_t row_bytes = payload_bytes(1, cols, format);
    satori_matrix_sharded *m = new satori_matrix_sharded();
    m->ctx = ctx;
    m->rows = rows;
    m->cols = cols;
    m->format = format;
    m->rank = rank;
    m->world = world;
    m->slice = slice;
    m->r0 = rank * slice;
    m->r1 = std::min(rows, m->r0 + slice);
    const uint8_t *mine = payload + row_bytes * (size_t)m->r0;
    const size_t mine_bytes = row_bytes * (size_t)(m->r1 - m->r0);
    rc = payload_on_device ? satori_matrix_create_device(ctx, mine, mine_bytes, m->r1 - m->r0, cols, format, &m->local)
                           : satori_matrix_create(ctx, mine, mine_bytes, m->r1 - m->r0, cols, format, &m->local);
    if (rc) {
        delete m;
        return rc;
    }
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess && (size_t)slice * world != (size_t)rows) e = cudaMalloc(&m->d_gather, (size_t)slice * world * 4);
    if (e != cudaSuccess) {
        const int f = cuda_fail(e, "allocate gather buffer");
        satori_matrix_sharded_destroy(m);
        return f;
    }
    if (world > 1) {
        const NcclApi *api = nccl_api();
        if (!api) {
            satori_matrix_sharded_destroy(m);
            return set_error(SATORI_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
        }
        ncclUniqueId id;
        memcpy(&id, nccl_unique_id, sizeof id);
        const ncclResult_t r = api->CommInitRank(&m->comm, world, id, rank);
        if (r != ncclSuccess) {
            m->comm = nullptr;
            const int f = nccl_fail(api, r, "communicator");
            satori_matrix_sharded_destroy(m);
            return f;
        }
    }
    *out = m;
    return SATORI_OK;
}

extern "C" int satori_matrix_sharded_info(const satori_matrix_sharded *m, int *row_begin, int *row_end)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (row_begin) *row_begin = m->r0;
    if (row_end) *row_end = m->r1;
    return SATORI_OK;
}

extern "C" int satori_matrix_sharded_execute_device(satori_matrix_sharded *m, const float *dx, float *dy, int order)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (!dx || !dy) return set_error(SATORI_ERR_ARGUMENT, "bad device vectors");
    if (order < 0 || order > SATORI_ORDER_BATCH) return set_error(SATORI_ERR_ARGUMENT, "bad order %d", order);
    float *gathered = m->d_gather ? m->d_gather : dy;
    int rc = satori_matrix_execute_device(m->local, dx, gathered + (size_t)m->rank * m->slice, 1, order);
    if (rc) return rc;
    cudaStream_t st = m->ctx->stream;
    if (m->world > 1) {
        const NcclApi *api = nccl_api();
        const ncclResult_t r = api->AllGather(gathered + (size_t)m->rank * m->slice, gathered, (size_t)m->slice,
                                              ncclFloat32, m->comm, st);
        if (r != ncclSuccess) return nccl_fail(api, r, "all-gather");
    }
    if (m->d_gather) {
        cudaError_t e = cudaMemcpyAsync(dy, m->d_gather, (size_t)m->rows * 4, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "copy gathered output");
    }
    return SATORI_OK;
}

extern "C" int satori_matrix_sharded_execute(satori_matrix_sharded *m, const float *x, float *y, int order)
{
    if (!m) return set_error(SATORI_ERR_DISPOSED, "matrix is disposed");
    if (!x || !y) return set_error(SATORI_ERR_ARGUMENT, "vector is null");
    satori_ctx *ctx = m->ctx;
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    cudaError_t e = cudaSuccess;
    if (!m->d_x) {
        e = cudaMalloc(&m->d_x, (size_t)m->cols * 4);
        if (e == cudaSuccess) e = cudaMalloc(&m->d_y, (size_t)m->rows * 4);
        if (e == cudaSuccess) e = cudaHostAlloc(&m->h_x, (size_t)m->cols * 4, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaHostAlloc(&m->h_y, (size_t)m->rows * 4, cudaHostAllocDefault);
        if (e != cudaSuccess) {
            cudaFree(m->d_x);
            cudaFree(m->d_y);
            cudaFreeHost(m->h_x);
            cudaFreeHost(m->h_y);
            m->d_x = m->d_y = m->h_x = m->h_y = nullptr;
            return cuda_fail(e, "allocate MatVec work vectors");
        }
    }
    memcpy(m->h_x, x, (size_t)m->cols * 4);
    e = clear_dev_error(ctx);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->d_x, m->h_x, (size_t)m->cols * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy input");
    int rc = satori_matrix_sharded_execute_device(m, m->d_x, m->d_y, order);
    if (rc) return rc;
    e = cudaMemcpyAsync(m->h_y, m->d_y, (size_t)m->rows * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "copy output");
    rc = check_dev_error(ctx);
    if (rc) return rc;
    memcpy(y, m->h_y, (size_t)m->rows * 4);   // commit only on success
    return SATORI_OK;
}
