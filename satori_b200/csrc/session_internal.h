// session_internal.h -- state of a decode session (single GPU or one rank of a sharded model).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "capi_internal.h"

#define TRY(x)               \
    do {                     \
        int rc_ = (x);       \
        if (rc_) return rc_; \
    } while (0)
#define TRYCUDA(x, what)                                   \
    do {                                                   \
        cudaError_t e_ = (x);                              \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

struct DevMatrix {
    const uint8_t *payload = nullptr;
    int rows = 0, cols = 0, format = 0;
};

struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    DevMatrix q, k, v, o, gate, up, down;
    // Fused forms (when the formats agree): q, k, v rows stacked (one launch, biases stacked alike) and
    // ffn_gate / ffn_up rows interleaved (one launch with the SwiGLU epilogue).  The parts are then freed.
    DevMatrix qkv, gu;
    float *qkv_bias = nullptr;
    bool qkv_norm = false;           // attn_norm runs inside the q/k/v launch (the rows kernel takes it)
};

struct ShardState;  // multi-GPU exchange state (session_sharded.cu)

struct satori_session {
    satori_ctx *ctx = nullptr;
    int layers = 0, hidden = 0, ffn = 0, q_heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
    int q_width = 0, kv_width = 0;
    float eps = 0;
    double rope_base = 0;
    int context = 0;
    int position = 0;
    int use_pdl = 1;
    int fuse = 1;                    // stack q/k/v and interleave gate/up (SATORI_FUSE=0 keeps them apart)
    int prefetch_next = 1;           // each projection prefetches the next one's weights into L2
                                     // (SATORI_PREFETCH_NEXT=0 turns it off)
    size_t weight_bytes = 0;

    std::vector<Layer> layer;
    DevMatrix embd, output;
    float *output_norm = nullptr;

    float *d_kcache = nullptr, *d_vcache = nullptr;
    float *d_hidden = nullptr, *d_normed = nullptr, *d_final = nullptr, *d_proj = nullptr;
    float *d_q = nullptr, *d_qrot = nullptr, *d_ctx = nullptr, *d_k = nullptr, *d_v = nullptr;
    float *d_qkv = nullptr;          // [q_local | kv_local | kv_local]: d_q, d_k, d_v point into it
    float *d_gate = nullptr, *d_up = nullptr, *d_act = nullptr, *d_logits = nullptr;
    float *d_attn_scratch = nullptr;
    double *d_rope = nullptr;        // this step's RoPE cos/sin per pair (written by the embed kernel)
    int *d_ints = nullptr;
    int *d_token = nullptr, *d_pos = nullptr, *d_tokens = nullptr, *d_argmax = nullptr, *d_nonfinite = nullptr;
    int *h_ints = nullptr;
    float *h_logits = nullptr;

    cudaGraphExec_t graph_exec = nullptr;
    int kernels_per_step = 0;        // kernel nodes of the captured step
    int *d_gen = nullptr;            // generated tokens of satori_session_generate ([context])
    std::vector<void *> allocations;

    // This rank's share of every dimension (a single-GPU session is world 1, rank 0, full ranges).
    // Rows stay whole on one rank, so every projection keeps the reference's per-row FP32 order.
    int world = 1, rank = 0;
    int qa = 0, qb = 0;              // query heads computed here
    int ka = 0, kb = 0;              // KV heads computed and cached here (those of qa .. qb-1)
    int h0 = 0, h1 = 0;              // rows of attn_output / ffn_down (hidden)
    int f0 = 0, f1 = 0;              // rows of ffn_gate / ffn_up
    int v0 = 0, v1 = 0;              // rows of the logits matrix
    int q_local = 0, kv_local = 0;   // floats of this rank's q and k (or v) vectors
    int qmax = 0;                    // query heads per rank in the padded context exchange (0: none)
    float *d_ctx_pad = nullptr;      // [world][qmax * head_dim] when query heads do not split evenly

    ShardState *shard = nullptr;
    bool failed = false;             // a peer stopped answering: every later step is refused

    // Tensor-core prefill (session_prefill.cu): chunk buffers, allocated by the first such call.
    int pf_ready = 0;                // 1 allocated, -1 the weights do not qualify
    int *pf_tokens = nullptr;        // [context] tokens of the call
    float *pf_hidden = nullptr, *pf_normed = nullptr, *pf_qkv = nullptr, *pf_qrot = nullptr, *pf_ctx = nullptr;
    float *pf_act = nullptr, *pf_gate = nullptr, *pf_up = nullptr, *pf_attn = nullptr;
    double *pf_rope = nullptr;       // [chunk][rotary/2][cos, sin]
};

satori_session *session_new(satori_ctx *ctx, const satori_model_desc *d, int context);
int session_check_desc(const satori_model_desc *d, int context);
int session_build(satori_session *s, const satori_model_desc *d, satori_session **out);
int session_alloc_state(satori_session *s);
// Device buffer owned by the session (freed with it), zeroed.
int session_dalloc_bytes(satori_session *s, void **p, size_t bytes);
void session_destroy_sharding(satori_session *s);
// Fills the rank's ranges (world 1: everything).  Returns a satori_status.
int session_plan_shards(satori_session *s);
// In-place NCCL all-gather of `count` floats per rank: rank r's slice is buf + r * count.  No-op for world 1.
int session_allgather(satori_session *s, float *buf, size_t count, cudaStream_t st);
// True when the gathered vectors are exchanged by peer stores (the default sharded backend).
bool session_p2p(const satori_session *s);
// Places d_hidden, d_ctx, d_act and d_logits in this rank's exchange arena and maps every peer's.
int session_exchange_alloc(satori_session *s);
// Gathers buf[off, off + count) from every rank (each rank its own slice) into every rank's buf.
int session_exchange(satori_session *s, float *buf, size_t off, size_t count, cudaStream_t st);
// P2P backend: a producing row-MatVec launch can carry the exchange itself (xchg.cuh).  session_xpush
// describes the push of an output whose element 0 is `local_out` (inside the exchange arena);
// session_xwait the wait of its consumer; launch_xwait runs that wait alone, for a consumer that
// cannot carry it.
bool session_xchg_fusable(const satori_session *s);
satori::XPush session_xpush(satori_session *s, float *local_out);
satori::XWait session_xwait(satori_session *s);
int launch_xwait(satori_session *s, cudaStream_t st);
// Copies every rank's query-head block out of the padded exchange buffer into d_ctx.
cudaError_t launch_ctx_compact(const float *pad, float *ctx, int world, int q_heads, int head_dim, int qmax,
                               cudaStream_t st);
