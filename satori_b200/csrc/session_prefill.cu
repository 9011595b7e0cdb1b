// session_prefill.cu -- DenseSession.Forward's chunked prefill with the projections on the tensor cores.
//
// DenseSession.Forward (src/Satori.Core/Model/DenseSession.cs:136-181) embeds a chunk of positions and runs
// it through DenseForward.LayerBatch (DenseForward.cs:178-262) layer by layer: RmsNorm of every position,
// the q/k/v projections over the whole chunk, bias / head norms / RoPE / cache append per position, then
// every position's causal attention, the output projection and residual, RmsNorm, gate/up projections,
// SwiGLU, the down projection and residual.  Only the last position's logits are formed.
//
// Here every projection of a chunk is one tensor-core GEMM (prefill_gemm.cu; Q8_0 / Q4_0 weights) with the
// bias, residual or SwiGLU in its epilogue, and every per-position phase is one launch over the whole chunk
// (the decode step's kernels with a position dimension).  Chunks hold up to 128 positions.  The projections
// accumulate in tensor memory rather than in ExecuteBatch's order, so the cache rows this path writes match
// the per-token path to FP32 rounding, not bit for bit; everything else is the decode step's arithmetic.
// The last token of the call runs through the captured decode step, which forms its logits and greedy
// token exactly as satori_session_append_tokens does.
#include "attention.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "session_internal.h"

#include <algorithm>

using namespace satori;

namespace {

constexpr int kPrefillChunk = 128;

bool takes(const DevMatrix &m, int epilogue)
{
    return m.payload && tc_gemm_takes(m.rows, m.cols, m.format, 1, epilogue);
}

// Whether every projection of every layer can run on the tensor-core path (single-GPU sessions only).
bool prefill_qualifies(const satori_session *s)
{
    if (s->world != 1) return false;
    for (const Layer &L : s->layer) {
        const bool qkv = L.qkv.payload ? takes(L.qkv, kEpiBias)
                                       : takes(L.q, kEpiBias) && takes(L.k, kEpiBias) && takes(L.v, kEpiBias);
        const bool ffn = L.gu.payload ? takes(L.gu, kEpiSwiGlu) : takes(L.gate, kEpiNone) && takes(L.up, kEpiNone);
        if (!qkv || !ffn || !takes(L.o, kEpiResidual) || !takes(L.down, kEpiResidual)) return false;
    }
    return true;
}

template <typename T>
int palloc(satori_session *s, T **p, size_t n)
{
    void *v = nullptr;
    TRY(session_dalloc_bytes(s, &v, n * sizeof(T)));
    *p = static_cast<T *>(v);
    return SATORI_OK;
}

int prefill_alloc(satori_session *s)
{
    const size_t P = kPrefillChunk;
    const int qkv_rows = s->q_local + 2 * s->kv_local;
    TRY(palloc(s, &s->pf_tokens, (size_t)s->context));
    TRY(palloc(s, &s->pf_hidden, P * s->hidden));
    TRY(palloc(s, &s->pf_normed, P * s->hidden));
    TRY(palloc(s, &s->pf_qkv, P * qkv_rows));
    TRY(palloc(s, &s->pf_qrot, P * s->q_local));
    TRY(palloc(s, &s->pf_ctx, P * s->q_width));
    TRY(palloc(s, &s->pf_act, P * s->ffn));
    if (std::any_of(s->layer.begin(), s->layer.end(), [](const Layer &L) { return !L.gu.payload; })) {
        TRY(palloc(s, &s->pf_gate, P * s->ffn));
        TRY(palloc(s, &s->pf_up, P * s->ffn));
    }
    TRY(palloc(s, &s->pf_rope, P * s->head_dim));
    // Partial records for the largest batch x split product any chunk size can ask for.
    size_t attn = 0;
    for (int b = 1; b <= kPrefillChunk; ++b)
        attn = std::max(attn, attn_scratch_floats(s->q_heads, s->kv_heads, s->head_dim, s->context,
                                                  s->ctx->sm_count, b));
    TRY(palloc(s, &s->pf_attn, attn));
    // The tensor-order scratch is the context's; grow it once for the largest projection.
    size_t tc = 0;
    auto need = [&](const DevMatrix &m) {
        if (m.payload) tc = std::max(tc, tc_scratch_bytes(m.rows, m.cols, kPrefillChunk, s->ctx->sm_count));
    };
    for (const Layer &L : s->layer) {
        need(L.qkv), need(L.q), need(L.k), need(L.v), need(L.o), need(L.gu), need(L.gate), need(L.up);
        need(L.down);
    }
    TRY(ensure_tc_scratch(s->ctx, tc));
    s->pf_ready = 1;
    return SATORI_OK;
}

int project(satori_session *s, const DevMatrix &m, const float *x, int positions, int epilogue, float *y, int ldy,
            const float *bias, float *residual, int ldr, cudaStream_t st)
{
    TcGemm g = {};
    g.payload = m.payload;
    g.rows = m.rows;
    g.cols = m.cols;
    g.format = m.format;
    g.x = x;
    g.positions = positions;
    g.epilogue = epilogue == kEpiBias && !bias ? kEpiNone : epilogue;
    g.y = y;
    g.ldy = ldy;
    g.bias = bias;
    g.residual = residual;
    g.ldr = ldr;
    g.scratch = s->ctx->tc_scratch;
    g.scratch_bytes = s->ctx->tc_scratch_bytes;
    g.err = s->ctx->d_err;
    TRYCUDA(launch_tc_gemm(g, s->ctx->sm_count, st), "prefill projection");
    return SATORI_OK;
}

// One chunk: positions pos0 .. pos0 + P - 1 with tokens pf_tokens[t0 ..].
int enqueue_chunk(satori_session *s, int t0, int P, int pos0, cudaStream_t st)
{
    const int H = s->hidden, hd = s->head_dim, nf = s->ffn;
    const int ql = s->q_local, kvl = s->kv_local, qkv_rows = ql + 2 * kvl;
    TRYCUDA(launch_embed_batch(s->embd.payload, H, s->pf_tokens + t0, P, pos0, s->pf_hidden, s->pf_rope,
                               s->rope_base, hd, st),
            "prefill embed");
    for (int l = 0; l < s->layers; ++l) {
        const Layer &L = s->layer[l];
        TRYCUDA(launch_rmsnorm_batch(s->pf_hidden, L.attn_norm, H, s->eps, s->pf_normed, P, st), "prefill norm");
        if (L.qkv.payload) {
            TRY(project(s, L.qkv, s->pf_normed, P, kEpiBias, s->pf_qkv, qkv_rows, L.qkv_bias, nullptr, 0, st));
        } else {
            TRY(project(s, L.q, s->pf_normed, P, kEpiBias, s->pf_qkv, qkv_rows, L.q_bias, nullptr, 0, st));
            TRY(project(s, L.k, s->pf_normed, P, kEpiBias, s->pf_qkv + ql, qkv_rows, L.k_bias, nullptr, 0, st));
            TRY(project(s, L.v, s->pf_normed, P, kEpiBias, s->pf_qkv + ql + kvl, qkv_rows, L.v_bias, nullptr, 0,
                        st));
        }
        if (L.q_norm) {
            TRYCUDA(launch_rmsnorm_heads_batch(s->pf_qkv, ql, L.q_norm, s->eps, hd, qkv_rows, P, st), "q norm");
            TRYCUDA(launch_rmsnorm_heads_batch(s->pf_qkv + ql, kvl, L.k_norm, s->eps, hd, qkv_rows, P, st), "k norm");
        }
        RopeAppendArgs r = {};
        r.q = s->pf_qkv;
        r.k = s->pf_qkv + ql;
        r.v = s->pf_qkv + ql + kvl;
        r.q_out = s->pf_qrot;
        r.k_cache = s->d_kcache + (size_t)l * s->context * kvl;
        r.v_cache = s->d_vcache + (size_t)l * s->context * kvl;
        r.q_heads = s->q_heads;
        r.kv_heads = s->kv_heads;
        r.head_dim = hd;
        r.rotary = hd;
        r.base = s->rope_base;
        r.position = pos0;
        r.table = s->pf_rope;
        r.batch = P;
        r.in_stride = qkv_rows;
        TRYCUDA(launch_rope_append(r, st), "prefill rope/append");
        AttnArgs a = {};
        a.q = s->pf_qrot;
        a.keys = r.k_cache;
        a.values = r.v_cache;
        a.q_heads = s->q_heads;
        a.kv_heads = s->kv_heads;
        a.head_dim = hd;
        a.kv_stride = kvl;
        a.tokens = pos0 + 1;
        a.max_tokens = s->context;
        a.out = s->pf_ctx;
        a.scratch = s->pf_attn;
        a.err = s->ctx->d_err;
        a.batch = P;
        a.q_pstride = ql;
        a.out_pstride = s->q_width;
        TRYCUDA(launch_attention(a, s->ctx->sm_count, st), "prefill attention");
        TRY(project(s, L.o, s->pf_ctx, P, kEpiResidual, nullptr, 0, nullptr, s->pf_hidden, H, st));
        TRYCUDA(launch_rmsnorm_batch(s->pf_hidden, L.ffn_norm, H, s->eps, s->pf_normed, P, st), "prefill norm");
        if (L.gu.payload) {
            TRY(project(s, L.gu, s->pf_normed, P, kEpiSwiGlu, s->pf_act, nf, nullptr, nullptr, 0, st));
        } else {
            TRY(project(s, L.gate, s->pf_normed, P, kEpiNone, s->pf_gate, nf, nullptr, nullptr, 0, st));
            TRY(project(s, L.up, s->pf_normed, P, kEpiNone, s->pf_up, nf, nullptr, nullptr, 0, st));
            TRYCUDA(launch_swiglu(s->pf_gate, s->pf_up, P * nf, s->pf_act, st, 0), "prefill swiglu");
        }
        TRY(project(s, L.down, s->pf_act, P, kEpiResidual, nullptr, 0, nullptr, s->pf_hidden, H, st));
    }
    return SATORI_OK;
}

}  // namespace

extern "C" int satori_session_forward_tensor(satori_session *s, const int *tokens, int count, float *logits,
                                             int *argmax)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    if (!tokens) return set_error(SATORI_ERR_ARGUMENT, "tokens is null");
    if (count <= 0) return set_error(SATORI_ERR_ARGUMENT, "count must be positive");
    for (int i = 0; i < count; ++i)
        if (tokens[i] < 0 || tokens[i] >= s->vocab)
            return set_error(SATORI_ERR_ARGUMENT, "Token %d is outside the vocabulary.", tokens[i]);
    if (s->position + count > s->context)
        return set_error(SATORI_ERR_CONTEXT_FULL, "Context limit %d reached; reset or enlarge the session.", s->context);
    if (s->pf_ready == 0) s->pf_ready = prefill_qualifies(s) ? 0 : -1;
    // One token, a sharded session or weights outside Q8_0 / Q4_0: the per-token step does it all.
    if (count == 1 || s->pf_ready < 0) return satori_session_append_tokens(s, tokens, count, logits, argmax);
    if (s->failed) return set_error(SATORI_ERR_TIMEOUT, "a peer rank stopped answering; destroy the sharded session");
    if (s->pf_ready == 0) TRY(prefill_alloc(s));
    satori_ctx *ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    const int n = count - 1;
    TRYCUDA(clear_dev_error(ctx), "clear error");
    TRYCUDA(cudaMemcpyAsync(s->pf_tokens, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, st), "prefill tokens");
    for (int t0 = 0; t0 < n; t0 += kPrefillChunk)
        TRY(enqueue_chunk(s, t0, std::min(kPrefillChunk, n - t0), s->position + t0, st));
    TRY(check_dev_error(ctx));
    // Commit the prefix, then the last token through the decode step (its logits and greedy token).
    s->position += n;
    s->h_ints[6] = s->position;
    TRYCUDA(cudaMemcpyAsync(s->d_pos, &s->h_ints[6], sizeof(int), cudaMemcpyHostToDevice, st), "position");
    TRYCUDA(cudaStreamSynchronize(st), "position");
    return satori_session_append_tokens(s, tokens + n, 1, logits, argmax);
}
