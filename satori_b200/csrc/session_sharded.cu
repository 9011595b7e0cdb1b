// session_sharded.cu -- one rank of a decode session sharded over GPUs (one process per GPU).
//
// Every projection is sharded by rows: rank r computes a contiguous block of output rows, so every
// row's FP32 chain (QuantizedMatVec.cs:300-365) runs whole on one GPU and the logits stay identical
// to a single-GPU session.  Attention is sharded by query heads (each rank computes, appends and
// caches only the KV heads its query heads read).  After each sharded operator the result the next
// operator needs in full is all-gathered in place with NCCL over NVLink, inside the same CUDA graph:
// the attention context, the residual after attn_output and after ffn_down, the SwiGLU activations,
// and the logits -- four exchanges per layer plus one per token.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2) when the first sharded session is created, so a
// process that already loaded NCCL (for example through torch.distributed) shares that copy.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <algorithm>

#include "capi_internal.h"
#include "session_internal.h"

using namespace satori;

namespace {

struct NcclApi {
    void *lib = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi *nccl_api()
{
    static NcclApi api = [] {
        NcclApi a;
        a.lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!a.lib) return a;
        a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(a.lib, "ncclGetUniqueId"));
        a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(dlsym(a.lib, "ncclCommInitRank"));
        a.AllGather = reinterpret_cast<decltype(a.AllGather)>(dlsym(a.lib, "ncclAllGather"));
        a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(a.lib, "ncclCommDestroy"));
        a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(a.lib, "ncclGetErrorString"));
        if (!a.GetUniqueId || !a.CommInitRank || !a.AllGather || !a.CommDestroy || !a.GetErrorString) a.lib = nullptr;
        return a;
    }();
    return api.lib ? &api : nullptr;
}

int nccl_fail(const NcclApi *api, ncclResult_t r, const char *what)
{
    return set_error(SATORI_ERR_CUDA, "%s: %s", what, api ? api->GetErrorString(r) : "NCCL unavailable");
}

// Context blocks of rank i (query heads [i*qH/W, (i+1)*qH/W)) sit at pad + i*qmax*hd.
__global__ void ctx_compact_kernel(const float *pad, float *ctx, int world, int q_heads, int head_dim, int qmax)
{
    const int n = q_heads * head_dim;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
        const int h = idx / head_dim, d = idx - h * head_dim;
        int i = world - 1;
        while (i > 0 && (long long)i * q_heads / world > h) --i;
        const int qa = (int)((long long)i * q_heads / world);
        ctx[idx] = pad[((size_t)i * qmax + (h - qa)) * head_dim + d];
    }
}

}  // namespace

struct ShardState {
    ncclComm_t comm = nullptr;
};

int session_plan_shards(satori_session *s)
{
    const int W = s->world, r = s->rank, hd = s->head_dim, group = s->q_heads / s->kv_heads;
    if (W == 1) {
        s->qa = 0;
        s->qb = s->q_heads;
        s->ka = 0;
        s->kb = s->kv_heads;
        s->h0 = 0;
        s->h1 = s->hidden;
        s->f0 = 0;
        s->f1 = s->ffn;
        s->v0 = 0;
        s->v1 = s->vocab;
        s->q_local = s->q_width;
        s->kv_local = s->kv_width;
        s->qmax = 0;
        return SATORI_OK;
    }
    if (s->hidden % W || s->ffn % W || s->vocab % W)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "hidden (%d), ffn (%d) and vocab (%d) must be multiples of the %d ranks",
                         s->hidden, s->ffn, s->vocab, W);
    if (s->q_heads < W)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "%d query heads cannot be shared by %d ranks", s->q_heads, W);
    s->h0 = r * (s->hidden / W);
    s->h1 = s->h0 + s->hidden / W;
    s->f0 = r * (s->ffn / W);
    s->f1 = s->f0 + s->ffn / W;
    s->v0 = r * (s->vocab / W);
    s->v1 = s->v0 + s->vocab / W;
    s->qa = (int)((long long)r * s->q_heads / W);
    s->qb = (int)((long long)(r + 1) * s->q_heads / W);
    s->ka = s->qa / group;
    s->kb = (s->qb - 1) / group + 1;
    s->q_local = (s->qb - s->qa) * hd;
    s->kv_local = (s->kb - s->ka) * hd;
    s->qmax = s->q_heads % W ? (s->q_heads + W - 1) / W : 0;
    return SATORI_OK;
}

int session_allgather(satori_session *s, float *buf, size_t count, cudaStream_t st)
{
    if (s->world == 1) return SATORI_OK;
    const NcclApi *api = nccl_api();
    if (!api || !s->shard) return set_error(SATORI_ERR_NOT_SUPPORTED, "NCCL is not available");
    const ncclResult_t r = api->AllGather(buf + (size_t)s->rank * count, buf, count, ncclFloat32, s->shard->comm, st);
    return r == ncclSuccess ? SATORI_OK : nccl_fail(api, r, "all-gather");
}

cudaError_t launch_ctx_compact(const float *pad, float *ctx, int world, int q_heads, int head_dim, int qmax,
                               cudaStream_t st)
{
    const int n = q_heads * head_dim;
    ctx_compact_kernel<<<(n + 255) / 256, 256, 0, st>>>(pad, ctx, world, q_heads, head_dim, qmax);
    return cudaGetLastError();
}

void session_destroy_sharding(satori_session *s)
{
    if (!s->shard) return;
    const NcclApi *api = nccl_api();
    if (api && s->shard->comm) api->CommDestroy(s->shard->comm);
    delete s->shard;
    s->shard = nullptr;
}

extern "C" int satori_nccl_unique_id(void *out128)
{
    if (!out128) return set_error(SATORI_ERR_ARGUMENT, "out is null");
    const NcclApi *api = nccl_api();
    if (!api) return set_error(SATORI_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    const ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(api, r, "unique id");
    memcpy(out128, &id, sizeof id);
    return SATORI_OK;
}

extern "C" int satori_session_create_sharded(satori_ctx *ctx, const satori_model_desc *desc, int context, int rank,
                                             int world, const void *nccl_unique_id, satori_session **out)
{
    if (!ctx || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    if (world < 1 || rank < 0 || rank >= world) return set_error(SATORI_ERR_ARGUMENT, "bad rank %d / world %d", rank, world);
    int rc = session_check_desc(desc, context);
    if (rc) return rc;
    if (world == 1) return satori_session_create(ctx, desc, context, out);
    if (!nccl_unique_id) return set_error(SATORI_ERR_ARGUMENT, "nccl_unique_id is null");
    if (desc->hidden % world || desc->ffn % world || desc->vocab % world)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "hidden (%d), ffn (%d) and vocab (%d) must be multiples of the %d ranks",
                         desc->hidden, desc->ffn, desc->vocab, world);
    if (desc->q_heads < world)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "%d query heads cannot be shared by %d ranks", desc->q_heads, world);
    const NcclApi *api = nccl_api();
    if (!api) return set_error(SATORI_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_fail(e, "set device");
    ncclUniqueId id;
    memcpy(&id, nccl_unique_id, sizeof id);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api->CommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) return nccl_fail(api, r, "communicator");
    satori_session *s = session_new(ctx, desc, context);
    s->world = world;
    s->rank = rank;
    s->shard = new ShardState();
    s->shard->comm = comm;
    return session_build(s, desc, out);
}
