// session_sharded.cu -- one rank of a decode session sharded over GPUs (one process per GPU).
//
// Every projection is sharded by rows: rank r computes a contiguous block of output rows, so every
// row's FP32 chain (QuantizedMatVec.cs:300-365) runs whole on one GPU and the logits stay identical
// to a single-GPU session.  Attention is sharded by query heads (each rank computes, appends and
// caches only the KV heads its query heads read).  After each sharded operator the result the next
// operator needs in full is all-gathered in place, inside the same CUDA graph: the attention context,
// the residual after attn_output and after ffn_down, the SwiGLU activations, and the logits -- four
// exchanges per layer plus one per token.
//
// Two exchange backends:
//  * P2P (default): the four gathered vectors live in one device arena per rank that every peer maps
//    (CUDA IPC).  Where the vector comes out of a row-MatVec launch, that launch stores its rows into
//    every peer's copy as it writes them and signals from its last CTA, and the next launch waits
//    (xchg.cuh); otherwise one small kernel per exchange stores this rank's slice into every peer's
//    copy over NVLink, then signals each peer with a release store of the exchange's sequence number
//    and waits (bounded) until every peer has signalled it (SATORI_EXCHANGE_CARRY=0 uses the kernel
//    for every exchange).  Slices may differ in length, so an uneven query-head split needs no
//    padding.
//  * NCCL (SATORI_EXCHANGE=nccl): in-place ncclAllGather; an uneven query-head split goes through a
//    padded context buffer and a compaction kernel.
// NCCL also carries the IPC handles at creation.  It is loaded at run time (dlopen of libnccl.so.2),
// so a process that already loaded NCCL (for example through torch.distributed) shares that copy.
//
// Ordering argument for the P2P backend: a peer writes exchange n's slice into this rank's arena only
// after it has seen this rank's signal for exchange n-1, and every buffer's remote slices are last read
// here before this rank signals the exchange preceding the one that rewrites them (the step reads the
// gathered residual in the norm before the next exchange, the context and activations in the
// projection right after their own exchange).
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"
#include "session_internal.h"
#include "nccl_api.h"
#include "xchg.cuh"

namespace satori {

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

}  // namespace satori

using namespace satori;

namespace {

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

constexpr int kMaxRanks = kXchgMaxRanks;
constexpr int kPushThreads = 256;
constexpr int kPushMaxCtas = 16;
// Default wait for a peer's signal: about four seconds of SM clock at 1.965 GHz, far above any step, so
// only a lost peer reaches it.  SATORI_PEER_TIMEOUT_MS overrides it when a session is created.
constexpr long long kPeerWaitCycles = 8000000000LL;

// Arena header (one 256-byte line): the peers' signals, then this rank's own bookkeeping.
struct ArenaHeader {
    unsigned long long flag[kMaxRanks];   // flag[src] = last exchange sequence number rank src signalled
    unsigned long long seq;               // exchanges completed here
    unsigned ticket;                      // CTAs of the running exchange that finished their stores
};
constexpr size_t kHeaderBytes = 256;
static_assert(sizeof(ArenaHeader) <= kHeaderBytes, "arena header");

struct PushArgs {
    const float *src;                      // this rank's slice in its own arena
    float *dst[kMaxRanks];                 // the same slice in each peer's arena (null for this rank)
    unsigned long long *signal[kMaxRanks]; // &peer header->flag[rank] (null for this rank)
    ArenaHeader *own;
    unsigned *err;
    size_t count;                          // floats
    long long budget;                      // SM cycles to wait for the peers' signals
    int rank, world;
};

// One exchange: copy this rank's slice to every peer, then signal and wait (last CTA to finish).
__global__ void __launch_bounds__(kPushThreads) p2p_push_kernel(PushArgs a)
{
    pdl_launch_dependents();
    pdl_wait();
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (size_t)gridDim.x * blockDim.x;
    if (((uintptr_t)a.src & 15) == 0 && (a.count & 3) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(a.src);
        for (size_t i = tid; i < a.count / 4; i += nth) {
            const float4 v = s4[i];
            for (int p = 0; p < a.world; ++p)
                if (p != a.rank) reinterpret_cast<float4 *>(a.dst[p])[i] = v;
        }
    } else {
        for (size_t i = tid; i < a.count; i += nth) {
            const float v = a.src[i];
            for (int p = 0; p < a.world; ++p)
                if (p != a.rank) a.dst[p][i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();   // this CTA's peer stores are visible system-wide before its ticket
    if (atomicAdd(&a.own->ticket, 1u) != gridDim.x - 1) return;
    a.own->ticket = 0;
    const unsigned long long n = a.own->seq + 1;
    __threadfence_system();
    for (int p = 0; p < a.world; ++p)
        if (p != a.rank) xchg_store_release_sys(a.signal[p], n);
    const long long start = clock64();
    for (int p = 0; p < a.world; ++p) {
        if (p == a.rank) continue;
        while (xchg_load_acquire_sys(&a.own->flag[p]) < n) {
            // After one expired wait the rest of the step does not wait again: the step already failed.
            if (clock64() - start > a.budget || (*(volatile unsigned *)a.err & kDevErrTimeout)) {
                atomicOr(a.err, kDevErrTimeout);
                a.own->seq = n;
                return;
            }
            __nanosleep(64);
        }
    }
    a.own->seq = n;
}

// The wait of an exchange carried by its producer, for a consumer that cannot carry it.
__global__ void xwait_kernel(XWait w, unsigned *err)
{
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) xwait_peers(w, err);
}

}  // namespace

struct ShardState {
    ncclComm_t comm = nullptr;
    bool p2p = false;
    char *arena = nullptr;                 // this rank's exchange arena (IPC-exported)
    char *peer[kMaxRanks] = {};            // every rank's arena as mapped here (peer[rank] == arena)
    size_t arena_bytes = 0;
    long long wait_cycles = kPeerWaitCycles;
    bool carry = true;                     // producing MatVec launches carry their exchanges
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
    s->qmax = s->q_heads % W && !(s->shard && s->shard->p2p) ? (s->q_heads + W - 1) / W : 0;
    return SATORI_OK;
}

bool session_p2p(const satori_session *s) { return s->shard && s->shard->p2p; }

namespace {

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

int session_exchange_alloc(satori_session *s)
{
    ShardState *sh = s->shard;
    const size_t oh = kHeaderBytes, oc = oh + align256((size_t)s->hidden * 4), oa = oc + align256((size_t)s->q_width * 4),
                 ol = oa + align256((size_t)s->ffn * 4), total = ol + align256((size_t)s->vocab * 4);
    TRYCUDA(cudaMalloc(&sh->arena, total), "exchange arena");
    sh->arena_bytes = total;
    // Cleared (and synchronised) before any peer can learn the handle, so no early signal is lost.
    TRYCUDA(cudaMemset(sh->arena, 0, total), "clear exchange arena");
    TRYCUDA(cudaDeviceSynchronize(), "clear exchange arena");
    s->d_hidden = reinterpret_cast<float *>(sh->arena + oh);
    s->d_ctx = reinterpret_cast<float *>(sh->arena + oc);
    s->d_act = reinterpret_cast<float *>(sh->arena + oa);
    s->d_logits = reinterpret_cast<float *>(sh->arena + ol);

    const NcclApi *api = nccl_api();
    const int W = s->world;
    cudaIpcMemHandle_t mine;
    TRYCUDA(cudaIpcGetMemHandle(&mine, sh->arena), "export exchange arena");
    std::vector<cudaIpcMemHandle_t> all(W);
    void *dbuf = nullptr;
    TRYCUDA(cudaMalloc(&dbuf, sizeof(cudaIpcMemHandle_t) * W), "handle buffer");
    char *db = static_cast<char *>(dbuf);
    cudaError_t e = cudaMemcpy(db + sizeof mine * s->rank, &mine, sizeof mine, cudaMemcpyHostToDevice);
    ncclResult_t r = ncclSuccess;
    if (e == cudaSuccess) {
        r = api->AllGather(db + sizeof mine * s->rank, db, sizeof mine, ncclUint8, sh->comm, s->ctx->stream);
        if (r == ncclSuccess) e = cudaStreamSynchronize(s->ctx->stream);
        if (r == ncclSuccess && e == cudaSuccess) e = cudaMemcpy(all.data(), db, sizeof mine * W, cudaMemcpyDeviceToHost);
    }
    cudaFree(dbuf);
    if (r != ncclSuccess) return nccl_fail(api, r, "handle exchange");
    if (e != cudaSuccess) return cuda_fail(e, "handle exchange");
    for (int p = 0; p < W; ++p) {
        if (p == s->rank) {
            sh->peer[p] = sh->arena;
            continue;
        }
        void *m = nullptr;
        e = cudaIpcOpenMemHandle(&m, all[p], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(SATORI_ERR_NOT_SUPPORTED,
                             "rank %d cannot map rank %d's exchange arena (%s); SATORI_EXCHANGE=nccl selects NCCL",
                             s->rank, p, cudaGetErrorString(e));
        sh->peer[p] = static_cast<char *>(m);
    }
    return SATORI_OK;
}

bool session_xchg_fusable(const satori_session *s)
{
    return s->world > 1 && s->shard && s->shard->p2p && s->shard->carry;
}

XPush session_xpush(satori_session *s, float *local_out)
{
    ShardState *sh = s->shard;
    XPush x = {};
    const size_t at = (size_t)(reinterpret_cast<char *>(local_out) - sh->arena);
    for (int p = 0; p < s->world; ++p) {
        if (p == s->rank) continue;
        x.dst[p] = reinterpret_cast<float *>(sh->peer[p] + at);
        x.signal[p] = &reinterpret_cast<ArenaHeader *>(sh->peer[p])->flag[s->rank];
    }
    ArenaHeader *own = reinterpret_cast<ArenaHeader *>(sh->arena);
    x.ticket = &own->ticket;
    x.seq = &own->seq;
    x.world = s->world;
    x.rank = s->rank;
    return x;
}

XWait session_xwait(satori_session *s)
{
    ArenaHeader *own = reinterpret_cast<ArenaHeader *>(s->shard->arena);
    XWait w = {};
    w.flags = own->flag;
    w.seq = &own->seq;
    w.budget = s->shard->wait_cycles;
    w.world = s->world;
    w.rank = s->rank;
    return w;
}

int launch_xwait(satori_session *s, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = s->use_pdl ? 1 : 0;
    TRYCUDA(cudaLaunchKernelEx(&cfg, xwait_kernel, session_xwait(s), s->ctx->d_err), "exchange wait");
    return SATORI_OK;
}

int session_exchange(satori_session *s, float *buf, size_t off, size_t count, cudaStream_t st)
{
    if (s->world == 1) return SATORI_OK;
    ShardState *sh = s->shard;
    if (!sh->p2p) {
        if (off != (size_t)s->rank * count)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "NCCL exchange needs equal slices");
        return session_allgather(s, buf, count, st);
    }
    const size_t at = (size_t)(reinterpret_cast<char *>(buf + off) - sh->arena);
    PushArgs a = {};
    a.src = buf + off;
    for (int p = 0; p < s->world; ++p) {
        if (p == s->rank) continue;
        a.dst[p] = reinterpret_cast<float *>(sh->peer[p] + at);
        a.signal[p] = &reinterpret_cast<ArenaHeader *>(sh->peer[p])->flag[s->rank];
    }
    a.own = reinterpret_cast<ArenaHeader *>(sh->arena);
    a.err = s->ctx->d_err;
    a.count = count;
    a.budget = sh->wait_cycles;
    a.rank = s->rank;
    a.world = s->world;
    const int ctas = (int)std::min<size_t>(kPushMaxCtas, std::max<size_t>(1, (count / 4 + kPushThreads - 1) / kPushThreads));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kPushThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = s->use_pdl ? 1 : 0;
    TRYCUDA(cudaLaunchKernelEx(&cfg, p2p_push_kernel, a), "exchange");
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
    for (int p = 0; p < kMaxRanks; ++p)
        if (s->shard->peer[p] && s->shard->peer[p] != s->shard->arena) cudaIpcCloseMemHandle(s->shard->peer[p]);
    if (s->shard->arena) cudaFree(s->shard->arena);
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
    const char *backend = getenv("SATORI_EXCHANGE");
    const bool p2p = !(backend && strcmp(backend, "nccl") == 0);
    if (backend && strcmp(backend, "nccl") != 0 && strcmp(backend, "p2p") != 0)
        return set_error(SATORI_ERR_ARGUMENT, "SATORI_EXCHANGE must be p2p or nccl, not '%s'", backend);
    if (p2p && world > kMaxRanks)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "the P2P exchange serves at most %d ranks", kMaxRanks);
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
    s->shard->p2p = p2p;
    if (const char *c = getenv("SATORI_EXCHANGE_CARRY")) s->shard->carry = strcmp(c, "0") != 0;
    if (const char *ms = getenv("SATORI_PEER_TIMEOUT_MS")) {
        const long long v = atoll(ms);
        if (v > 0) s->shard->wait_cycles = v * 2000000LL;   // 2 GHz: at most the B200's SM clock
    }
    return session_build(s, desc, out);
}
