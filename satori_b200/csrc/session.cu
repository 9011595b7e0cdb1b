// session.cu -- the dense decode session: DenseSession.Append (src/Satori.Core/Model/DenseSession.cs:111-131)
// with DenseForward.Embed/Step/Final (src/Satori.Core/Model/DenseForward.cs:87-162, 298-306) and greedy
// selection, entirely on the device.
//
// All weights are uploaded once at creation (unchanged GGUF layout) and the KV cache lives in HBM
// ([layer][context][kv_heads*head_dim], DenseSession.cs:80-84).  One decode step is a fixed
// sequence of kernels whose only varying inputs -- the token and the position -- live in device
// memory, so the step is captured once into a CUDA graph and replayed for every token; the greedy
// argmax kernel writes the next token and advances the position on the device, so a generation
// loop needs no host round trip between tokens.
#include "attention.cuh"
#include "capi_internal.h"
#include "common.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "session_internal.h"

#include <string.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <initializer_list>
#include <utility>
#include <string>
#include <vector>

using namespace satori;

namespace {

const satori_tensor *find_tensor(const satori_model_desc *d, const std::string &name)
{
    for (int i = 0; i < d->n_tensors; ++i)
        if (d->tensors[i].name && name == d->tensors[i].name) return &d->tensors[i];
    return nullptr;
}

// Uploads rows [r0, r1) of the named matrix (all rows when r1 <= r0).  Rows are contiguous in the
// GGUF payload, so a row slice is one contiguous byte range.
int fetch_matrix(satori_session *s, const satori_model_desc *d, const std::string &name, int rows, int cols,
                 DevMatrix *out, int r0 = 0, int r1 = 0)
{
    const satori_tensor *t = find_tensor(d, name);
    if (!t) return set_error(SATORI_ERR_ARGUMENT, "missing tensor %s", name.c_str());
    if (t->format < 0 || t->rows != rows || t->cols != cols)
        return set_error(SATORI_ERR_ARGUMENT, "tensor %s has shape %dx%d (format %d), expected %dx%d matrix",
                         name.c_str(), t->rows, t->cols, t->format, rows, cols);
    if (t->bytes != payload_bytes(rows, cols, t->format))
        return set_error(SATORI_ERR_ARGUMENT, "tensor %s has %zu bytes, expected %zu", name.c_str(), t->bytes,
                         payload_bytes(rows, cols, t->format));
    if (r1 <= r0) {
        r0 = 0;
        r1 = rows;
    }
    const size_t row_bytes = payload_bytes(1, cols, t->format);
    uint8_t *dp = nullptr;
    TRY(upload_payload(s->ctx, (const uint8_t *)t->data + (size_t)r0 * row_bytes, false, (size_t)(r1 - r0) * row_bytes,
                       r1 - r0, cols, t->format, &dp));
    s->allocations.push_back(dp);
    out->payload = dp;
    out->rows = r1 - r0;
    out->cols = cols;
    out->format = t->format;
    s->weight_bytes += (size_t)(r1 - r0) * row_bytes;
    return SATORI_OK;
}

// Uploads elements [e0, e0 + count) of the named float vector of length n (all of it when count <= 0).
int fetch_vector(satori_session *s, const satori_model_desc *d, const std::string &name, int n, float **out,
                 bool optional = false, int e0 = 0, int count = 0)
{
    const satori_tensor *t = find_tensor(d, name);
    if (!t) {
        if (optional) {
            *out = nullptr;
            return SATORI_OK;
        }
        return set_error(SATORI_ERR_ARGUMENT, "missing tensor %s", name.c_str());
    }
    if (t->format != -1 || t->rows != n || t->bytes != (size_t)n * 4)
        return set_error(SATORI_ERR_ARGUMENT, "tensor %s must be %d float32 values", name.c_str(), n);
    if (count <= 0) {
        e0 = 0;
        count = n;
    }
    float *dv = nullptr;
    TRYCUDA(cudaMalloc(&dv, (size_t)count * 4), "upload vector");
    s->allocations.push_back(dv);
    TRYCUDA(cudaMemcpy(dv, (const float *)t->data + e0, (size_t)count * 4, cudaMemcpyDefault), "upload vector");
    *out = dv;
    return SATORI_OK;
}

void release(satori_session *s, void *p)
{
    if (!p) return;
    cudaFree(p);
    s->allocations.erase(std::find(s->allocations.begin(), s->allocations.end(), p));
}

// One payload holding the rows of `parts` stacked in order (interleave = false) or, for two parts of
// equal height, row i of part 0 then row i of part 1 (interleave = true).  The parts are freed.
int combine_rows(satori_session *s, std::initializer_list<DevMatrix *> parts, bool interleave, DevMatrix *out)
{
    const DevMatrix &p0 = **parts.begin();
    const size_t rb = payload_bytes(1, p0.cols, p0.format);
    int rows = 0;
    for (const DevMatrix *p : parts) rows += p->rows;
    uint8_t *d = nullptr;
    const size_t bytes = (size_t)rows * rb;
    TRYCUDA(cudaMalloc(&d, bytes + 256), "allocate fused payload");
    s->allocations.push_back(d);
    TRYCUDA(cudaMemset(d + bytes, 0, 256), "clear payload padding");
    if (interleave) {
        int k = 0;
        for (const DevMatrix *p : parts)
            TRYCUDA(cudaMemcpy2D(d + rb * k++, 2 * rb, p->payload, rb, rb, p->rows, cudaMemcpyDeviceToDevice),
                    "interleave rows");
    } else {
        size_t off = 0;
        for (const DevMatrix *p : parts) {
            TRYCUDA(cudaMemcpy(d + off, p->payload, (size_t)p->rows * rb, cudaMemcpyDeviceToDevice), "stack rows");
            off += (size_t)p->rows * rb;
        }
    }
    for (DevMatrix *p : parts) {
        release(s, const_cast<uint8_t *>(p->payload));
        p->payload = nullptr;
    }
    out->payload = d;
    out->rows = rows;
    out->cols = p0.cols;
    out->format = p0.format;
    return SATORI_OK;
}

int stack_vectors(satori_session *s, std::initializer_list<std::pair<float **, int>> parts, float **out)
{
    int n = 0;
    for (const auto &p : parts) n += p.second;
    float *d = nullptr;
    TRYCUDA(cudaMalloc(&d, (size_t)n * 4), "allocate fused bias");
    s->allocations.push_back(d);
    int off = 0;
    for (const auto &p : parts) {
        TRYCUDA(cudaMemcpy(d + off, *p.first, (size_t)p.second * 4, cudaMemcpyDeviceToDevice), "stack bias");
        off += p.second;
        release(s, *p.first);
        *p.first = nullptr;
    }
    *out = d;
    return SATORI_OK;
}

template <typename T>
int dalloc(satori_session *s, T **p, size_t n)
{
    TRYCUDA(cudaMalloc(p, n * sizeof(T) + 16), "allocate session buffer");
    s->allocations.push_back(*p);
    TRYCUDA(cudaMemset(*p, 0, n * sizeof(T) + 16), "clear session buffer");
    return SATORI_OK;
}

}  // namespace

// Enqueues one decode step on `st` (captured into the graph).  A sharded rank computes its rows of
// every projection and its query heads' attention, and all-gathers each result the next operator
// needs in full (context, residual after attn_output and after ffn_down, SwiGLU activations, logits).
static int enqueue_step(satori_session *s, cudaStream_t st)
{
    const int pdl = s->use_pdl;
    const int H = s->hidden, qw = s->q_width, hd = s->head_dim;
    const int group = s->q_heads / s->kv_heads;
    const int nq = s->qb - s->qa, nkv = s->kb - s->ka;
    // Sharded P2P step: a row-MatVec launch that produces a gathered vector carries the exchange (its
    // epilogue stores the rows into the peers' copies and signals), and the launch that reads the vector
    // next waits for the peers' signals; `pending` tracks an exchange whose wait is still owed.
    const bool xf = session_xchg_fusable(s);
    const XWait xw = xf ? session_xwait(s) : XWait{};
    bool pending = false;
    auto take_wait = [&]() -> const XWait * {
        if (!pending) return nullptr;
        pending = false;
        return &xw;
    };
    auto flush_wait = [&]() -> int {
        if (!pending) return SATORI_OK;
        pending = false;
        return launch_xwait(s, st);
    };
    // The head of the next projection's weights goes into L2 while the current one finishes.
    auto hint = [&](const DevMatrix &m) {
        s->ctx->next_payload = s->prefetch_next ? m.payload : nullptr;
        s->ctx->next_bytes = m.payload ? payload_bytes(m.rows, m.cols, m.format) : 0;
    };
    auto first_projection = [&](const Layer &L) -> const DevMatrix & { return L.qkv.payload ? L.qkv : L.q; };
    auto carries = [&](int rows, int cols, int fmt, int epi) {
        return xf && gemv_fused_takes(rows, cols, fmt, epi, s->ctx->sm_count, s->ctx->smem_optin);
    };
    TRYCUDA(launch_embed(s->embd.payload, H, s->d_token, s->d_pos, s->d_tokens, s->d_hidden, s->d_rope, s->rope_base,
                         hd, st, pdl),
            "embed");
    for (int l = 0; l < s->layers; ++l) {
        const Layer &L = s->layer[l];
        if (!L.qkv_norm) {
            TRY(flush_wait());
            TRYCUDA(launch_rmsnorm(s->d_hidden, L.attn_norm, H, s->eps, s->d_normed, st, pdl), "rmsnorm");
        }
        if (L.qkv.payload) {
            hint(L.o);
            TRY(run_gemv(s->ctx, L.qkv.payload, L.qkv.rows, H, L.qkv.format, SATORI_ORDER_BATCH,
                         L.qkv_norm ? s->d_hidden : s->d_normed, s->d_qkv, 1, L.qkv_bias ? kEpiBias : kEpiNone,
                         L.qkv_bias, nullptr, st, pdl, L.qkv_norm ? L.attn_norm : nullptr, s->eps, nullptr,
                         L.qkv_norm ? take_wait() : nullptr));
        } else {
            TRY(run_gemv(s->ctx, L.q.payload, L.q.rows, H, L.q.format, SATORI_ORDER_BATCH, s->d_normed, s->d_q, 1,
                         L.q_bias ? kEpiBias : kEpiNone, L.q_bias, nullptr, st, pdl));
            TRY(run_gemv(s->ctx, L.k.payload, L.k.rows, H, L.k.format, SATORI_ORDER_BATCH, s->d_normed, s->d_k, 1,
                         L.k_bias ? kEpiBias : kEpiNone, L.k_bias, nullptr, st, pdl));
            TRY(run_gemv(s->ctx, L.v.payload, L.v.rows, H, L.v.format, SATORI_ORDER_BATCH, s->d_normed, s->d_v, 1,
                         L.v_bias ? kEpiBias : kEpiNone, L.v_bias, nullptr, st, pdl));
        }
        if (L.q_norm) {
            TRYCUDA(launch_rmsnorm_heads(s->d_q, s->q_local, L.q_norm, s->eps, hd, st, pdl), "q norm");
            TRYCUDA(launch_rmsnorm_heads(s->d_k, s->kv_local, L.k_norm, s->eps, hd, st, pdl), "k norm");
        }
        RopeAppendArgs r = {};
        r.q = s->d_q;
        r.k = s->d_k;
        r.v = s->d_v;
        r.q_out = s->d_qrot;
        r.k_cache = s->d_kcache + (size_t)l * s->context * s->kv_local;
        r.v_cache = s->d_vcache + (size_t)l * s->context * s->kv_local;
        r.q_heads = nq;
        r.kv_heads = nkv;
        r.head_dim = hd;
        r.rotary = hd;
        r.base = s->rope_base;
        r.position_dev = s->d_pos;
        r.table = s->d_rope;
        r.use_pdl = pdl;
        TRYCUDA(launch_rope_append(r, st), "rope/append");
        float *ctx_out = s->qmax ? s->d_ctx_pad + (size_t)s->rank * s->qmax * hd : s->d_ctx + (size_t)s->qa * hd;
        // One launch when this rank's query heads are whole groups; otherwise one per KV head touched.
        const bool whole = s->qa % group == 0 && s->qb % group == 0;
        for (int g = whole ? s->ka : s->ka; g < (whole ? s->ka + 1 : s->kb); ++g) {
            const int qs = whole ? s->qa : std::max(s->qa, g * group);
            const int qe = whole ? s->qb : std::min(s->qb, (g + 1) * group);
            const int kg = whole ? s->ka : g;
            AttnArgs a = {};
            a.q = s->d_qrot + (size_t)(qs - s->qa) * hd;
            a.keys = r.k_cache + (size_t)(kg - s->ka) * hd;
            a.values = r.v_cache + (size_t)(kg - s->ka) * hd;
            a.q_heads = qe - qs;
            a.kv_heads = whole ? nkv : 1;
            a.head_dim = hd;
            a.kv_stride = s->kv_local;
            a.tokens_dev = s->d_tokens;
            a.max_tokens = s->context;
            a.out = ctx_out + (size_t)(qs - s->qa) * hd;
            a.scratch = s->d_attn_scratch;
            a.err = s->ctx->d_err;
            a.use_pdl = pdl;
            TRYCUDA(launch_attention(a, s->ctx->sm_count, st), "attention");
        }
        if (s->qmax) {
            TRY(session_allgather(s, s->d_ctx_pad, (size_t)s->qmax * hd, st));
            TRYCUDA(launch_ctx_compact(s->d_ctx_pad, s->d_ctx, s->world, s->q_heads, hd, s->qmax, st), "ctx");
        } else {
            TRY(session_exchange(s, s->d_ctx, (size_t)s->qa * hd, (size_t)s->q_local, st));
        }
        if (carries(s->h1 - s->h0, qw, L.o.format, kEpiResidual)) {
            const XPush xp = session_xpush(s, s->d_hidden + s->h0);
            hint(L.gu.payload ? L.gu : L.gate);
            TRY(run_gemv(s->ctx, L.o.payload, s->h1 - s->h0, qw, L.o.format, SATORI_ORDER_BATCH, s->d_ctx,
                         s->d_proj + s->h0, 1, kEpiResidual, nullptr, s->d_hidden + s->h0, st, pdl, nullptr, 0.0f,
                         &xp));
            pending = true;
        } else {
            hint(L.gu.payload ? L.gu : L.gate);
            TRY(run_gemv(s->ctx, L.o.payload, s->h1 - s->h0, qw, L.o.format, SATORI_ORDER_BATCH, s->d_ctx,
                         s->d_proj + s->h0, 1, kEpiResidual, nullptr, s->d_hidden + s->h0, st, pdl));
            TRY(session_exchange(s, s->d_hidden, (size_t)s->h0, (size_t)(s->h1 - s->h0), st));
        }
        const int nf = s->f1 - s->f0;
        if (L.gu.payload) {
            // ffn_norm runs inside the launch: every CTA forms the same norm of the residual.
            const XPush xp = xf ? session_xpush(s, s->d_act + s->f0) : XPush{};
            hint(L.down);
            TRY(run_gemv(s->ctx, L.gu.payload, 2 * nf, H, L.gu.format, SATORI_ORDER_BATCH, s->d_hidden,
                         s->d_act + s->f0, 1, kEpiSwiGlu, nullptr, nullptr, st, pdl, L.ffn_norm, s->eps,
                         xf ? &xp : nullptr, take_wait()));
            if (xf)
                pending = true;
            else
                TRY(session_exchange(s, s->d_act, (size_t)s->f0, (size_t)nf, st));
        } else {
            TRY(flush_wait());
            TRYCUDA(launch_rmsnorm(s->d_hidden, L.ffn_norm, H, s->eps, s->d_normed, st, pdl), "rmsnorm");
            TRY(run_gemv(s->ctx, L.gate.payload, nf, H, L.gate.format, SATORI_ORDER_BATCH, s->d_normed, s->d_gate, 1,
                         kEpiNone, nullptr, nullptr, st, pdl));
            TRY(run_gemv(s->ctx, L.up.payload, nf, H, L.up.format, SATORI_ORDER_BATCH, s->d_normed, s->d_up, 1,
                         kEpiNone, nullptr, nullptr, st, pdl));
            TRYCUDA(launch_swiglu(s->d_gate, s->d_up, nf, s->d_act + s->f0, st, pdl), "swiglu");
            TRY(session_exchange(s, s->d_act, (size_t)s->f0, (size_t)nf, st));
        }
        const DevMatrix &after_down = l + 1 < s->layers ? first_projection(s->layer[l + 1]) : s->output;
        if (carries(s->h1 - s->h0, s->ffn, L.down.format, kEpiResidual)) {
            const XPush xp = session_xpush(s, s->d_hidden + s->h0);
            hint(after_down);
            TRY(run_gemv(s->ctx, L.down.payload, s->h1 - s->h0, s->ffn, L.down.format, SATORI_ORDER_BATCH,
                         s->d_act, s->d_proj + s->h0, 1, kEpiResidual, nullptr, s->d_hidden + s->h0, st, pdl,
                         nullptr, 0.0f, &xp, take_wait()));
            pending = true;
        } else {
            TRY(flush_wait());
            hint(after_down);
            TRY(run_gemv(s->ctx, L.down.payload, s->h1 - s->h0, s->ffn, L.down.format, SATORI_ORDER_BATCH,
                         s->d_act, s->d_proj + s->h0, 1, kEpiResidual, nullptr, s->d_hidden + s->h0, st, pdl));
            TRY(session_exchange(s, s->d_hidden, (size_t)s->h0, (size_t)(s->h1 - s->h0), st));
        }
    }
    TRY(flush_wait());
    TRYCUDA(launch_rmsnorm(s->d_hidden, s->output_norm, H, s->eps, s->d_final, st, pdl), "final norm");
    if (carries(s->v1 - s->v0, H, s->output.format, kEpiNone)) {
        const XPush xp = session_xpush(s, s->d_logits + s->v0);
        hint(first_projection(s->layer[0]));
        TRY(run_gemv(s->ctx, s->output.payload, s->v1 - s->v0, H, s->output.format, SATORI_ORDER_BATCH, s->d_final,
                     s->d_logits + s->v0, 1, kEpiNone, nullptr, nullptr, st, pdl, nullptr, 0.0f, &xp));
        pending = true;
    } else {
        hint(first_projection(s->layer[0]));
        TRY(run_gemv(s->ctx, s->output.payload, s->v1 - s->v0, H, s->output.format, SATORI_ORDER_BATCH, s->d_final,
                     s->d_logits + s->v0, 1, kEpiNone, nullptr, nullptr, st, pdl));
        TRY(session_exchange(s, s->d_logits, (size_t)s->v0, (size_t)(s->v1 - s->v0), st));
    }
    TRY(flush_wait());
    TRYCUDA(launch_argmax_advance(s->d_logits, s->vocab, s->d_argmax, s->d_nonfinite, s->d_pos, s->d_token,
                                  reinterpret_cast<unsigned *>(s->d_ints + 8), s->ctx->sm_count, st, pdl),
            "argmax");
    return SATORI_OK;
}

static int build_graph(satori_session *s)
{
    cudaStream_t st = s->ctx->stream;
    TRYCUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture");
    int rc = enqueue_step(s, st);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "end capture");
    size_t nodes = 0;
    e = cudaGraphGetNodes(g, nullptr, &nodes);
    if (e == cudaSuccess && nodes) {
        std::vector<cudaGraphNode_t> list(nodes);
        e = cudaGraphGetNodes(g, list.data(), &nodes);
        s->kernels_per_step = 0;
        for (size_t i = 0; e == cudaSuccess && i < nodes; ++i) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(list[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++s->kernels_per_step;
        }
    }
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        return cuda_fail(e, "graph nodes");
    }
    e = cudaGraphInstantiate(&s->graph_exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "instantiate graph");
    return SATORI_OK;
}

static int session_upload(satori_session *s, const satori_model_desc *d)
{
    const int H = d->hidden, F = d->ffn;
    s->layer.resize(d->layers);
    for (int l = 0; l < d->layers; ++l) {
        Layer &L = s->layer[l];
        const std::string p = "blk." + std::to_string(l) + ".";
        TRY(fetch_vector(s, d, p + "attn_norm.weight", H, &L.attn_norm));
        TRY(fetch_vector(s, d, p + "ffn_norm.weight", H, &L.ffn_norm));
        const int hd = s->head_dim;
        TRY(fetch_matrix(s, d, p + "attn_q.weight", s->q_width, H, &L.q, s->qa * hd, s->qb * hd));
        TRY(fetch_matrix(s, d, p + "attn_k.weight", s->kv_width, H, &L.k, s->ka * hd, s->kb * hd));
        TRY(fetch_matrix(s, d, p + "attn_v.weight", s->kv_width, H, &L.v, s->ka * hd, s->kb * hd));
        TRY(fetch_matrix(s, d, p + "attn_output.weight", H, s->q_width, &L.o, s->h0, s->h1));
        TRY(fetch_matrix(s, d, p + "ffn_gate.weight", F, H, &L.gate, s->f0, s->f1));
        TRY(fetch_matrix(s, d, p + "ffn_up.weight", F, H, &L.up, s->f0, s->f1));
        TRY(fetch_matrix(s, d, p + "ffn_down.weight", H, F, &L.down, s->h0, s->h1));
        TRY(fetch_vector(s, d, p + "attn_q.bias", s->q_width, &L.q_bias, true, s->qa * hd, s->q_local));
        TRY(fetch_vector(s, d, p + "attn_k.bias", s->kv_width, &L.k_bias, true, s->ka * hd, s->kv_local));
        TRY(fetch_vector(s, d, p + "attn_v.bias", s->kv_width, &L.v_bias, true, s->ka * hd, s->kv_local));
        // Qwen2 carries all three biases or none; a partial set is rejected.
        if (!!L.q_bias != !!L.k_bias || !!L.q_bias != !!L.v_bias)
            return set_error(SATORI_ERR_ARGUMENT, "layer %d has a partial q/k/v bias set", l);
        TRY(fetch_vector(s, d, p + "attn_q_norm.weight", s->head_dim, &L.q_norm, true));
        TRY(fetch_vector(s, d, p + "attn_k_norm.weight", s->head_dim, &L.k_norm, true));
        if (!!L.q_norm != !!L.k_norm) return set_error(SATORI_ERR_ARGUMENT, "layer %d has a partial q/k norm set", l);
        if (s->fuse && L.q.format == L.k.format && L.q.format == L.v.format) {
            TRY(combine_rows(s, {&L.q, &L.k, &L.v}, false, &L.qkv));
            if (L.q_bias)
                TRY(stack_vectors(s, {{&L.q_bias, s->q_local}, {&L.k_bias, s->kv_local}, {&L.v_bias, s->kv_local}},
                                  &L.qkv_bias));
            L.qkv_norm = gemv_fused_takes(L.qkv.rows, H, L.qkv.format, L.qkv_bias ? kEpiBias : kEpiNone,
                                         s->ctx->sm_count, s->ctx->smem_optin);
        }
        const int nf = s->f1 - s->f0;
        if (s->fuse && L.gate.format == L.up.format &&
            gemv_fused_takes(2 * nf, H, L.gate.format, kEpiSwiGlu, s->ctx->sm_count, s->ctx->smem_optin))
            TRY(combine_rows(s, {&L.gate, &L.up}, true, &L.gu));
    }
    const satori_tensor *e = find_tensor(d, "token_embd.weight");
    // GgufQuantizedMatrix.ReadRow rejects Q4_0 embedding rows (GgufQuantizedMatrix.cs:56).
    if (e && e->format == SATORI_Q4_0)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "Q4_0 embedding rows are not supported");
    TRY(fetch_matrix(s, d, "token_embd.weight", d->vocab, H, &s->embd));
    if (s->embd.format != SATORI_Q8_0)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "embedding rows must be Q8_0");
    TRY(fetch_vector(s, d, "output_norm.weight", H, &s->output_norm));
    if (d->tied_embeddings && s->world == 1) s->output = s->embd;
    else if (d->tied_embeddings) TRY(fetch_matrix(s, d, "token_embd.weight", d->vocab, H, &s->output, s->v0, s->v1));
    else TRY(fetch_matrix(s, d, "output.weight", d->vocab, H, &s->output, s->v0, s->v1));
    return SATORI_OK;
}

int session_alloc_state(satori_session *s)
{
    const size_t kv = (size_t)s->layers * s->context * s->kv_local;
    TRY(dalloc(s, &s->d_kcache, kv));
    TRY(dalloc(s, &s->d_vcache, kv));
    // The vectors a sharded rank gathers live in the IPC-mapped exchange arena under the P2P backend.
    if (session_p2p(s)) {
        TRY(session_exchange_alloc(s));
    } else {
        TRY(dalloc(s, &s->d_hidden, s->hidden));
        TRY(dalloc(s, &s->d_ctx, s->q_width));
        TRY(dalloc(s, &s->d_act, s->ffn));
        TRY(dalloc(s, &s->d_logits, s->vocab));
    }
    TRY(dalloc(s, &s->d_normed, s->hidden));
    TRY(dalloc(s, &s->d_final, s->hidden));
    TRY(dalloc(s, &s->d_proj, s->hidden));
    TRY(dalloc(s, &s->d_qkv, (size_t)s->q_local + 2 * s->kv_local));
    s->d_q = s->d_qkv;
    s->d_k = s->d_qkv + s->q_local;
    s->d_v = s->d_k + s->kv_local;
    TRY(dalloc(s, &s->d_qrot, s->q_local));
    if (s->qmax) TRY(dalloc(s, &s->d_ctx_pad, (size_t)s->world * s->qmax * s->head_dim));
    TRY(dalloc(s, &s->d_gate, s->f1 - s->f0));
    TRY(dalloc(s, &s->d_up, s->f1 - s->f0));
    TRY(dalloc(s, &s->d_ints, 12));   // 0-6 step state (read back), 8-11 argmax scratch
    TRY(dalloc(s, &s->d_gen, (size_t)s->context));
    TRY(dalloc(s, &s->d_rope, (size_t)s->head_dim));
    s->d_token = s->d_ints + 0;
    s->d_pos = s->d_ints + 1;
    s->d_tokens = s->d_ints + 2;
    s->d_argmax = s->d_ints + 3;
    s->d_nonfinite = s->d_ints + 4;
    // Enough partial records for any launch shape the step uses (a single KV head has the most splits).
    TRY(dalloc(s, &s->d_attn_scratch,
               std::max(attn_scratch_floats(s->q_heads, s->kv_heads, s->head_dim, s->context, s->ctx->sm_count),
                        attn_scratch_floats(s->q_heads, 1, s->head_dim, s->context, s->ctx->sm_count))));
    TRYCUDA(cudaHostAlloc(&s->h_ints, 8 * sizeof(int), cudaHostAllocDefault), "pinned ints");
    TRYCUDA(cudaHostAlloc(&s->h_logits, (size_t)s->vocab * 4, cudaHostAllocDefault), "pinned logits");
    return SATORI_OK;
}

static int check_desc(const satori_model_desc *d, int context)
{
    if (!d) return set_error(SATORI_ERR_ARGUMENT, "desc is null");
    if (d->layers <= 0 || d->hidden <= 0 || d->ffn <= 0 || d->q_heads <= 0 || d->kv_heads <= 0 || d->head_dim <= 0 ||
        d->vocab <= 0 || context <= 0)
        return set_error(SATORI_ERR_ARGUMENT, "model dimensions and context must be positive");
    if (d->q_heads % d->kv_heads != 0) return set_error(SATORI_ERR_ARGUMENT, "q_heads must be a multiple of kv_heads");
    if (d->head_dim % 2 != 0 || d->head_dim > 256) return set_error(SATORI_ERR_ARGUMENT, "unsupported head_dim");
    if (!(d->rms_epsilon > 0) || !(d->rope_base > 0)) return set_error(SATORI_ERR_ARGUMENT, "bad epsilon/rope base");
    return SATORI_OK;
}

satori_session *session_new(satori_ctx *ctx, const satori_model_desc *d, int context)
{
    satori_session *s = new satori_session();
    s->ctx = ctx;
    s->layers = d->layers;
    s->hidden = d->hidden;
    s->ffn = d->ffn;
    s->q_heads = d->q_heads;
    s->kv_heads = d->kv_heads;
    s->head_dim = d->head_dim;
    s->vocab = d->vocab;
    s->eps = d->rms_epsilon;
    s->rope_base = d->rope_base;
    s->context = context;
    s->q_width = d->q_heads * d->head_dim;
    s->kv_width = d->kv_heads * d->head_dim;
    s->use_pdl = 1;
    const char *fuse = getenv("SATORI_FUSE");
    s->fuse = !(fuse && strcmp(fuse, "0") == 0);
    const char *pf = getenv("SATORI_PREFETCH_NEXT");
    s->prefetch_next = !(pf && strcmp(pf, "0") == 0);
    return s;
}

// Uploads this rank's weights, allocates the state and captures the decode step.  On failure the
// session is destroyed and the error of the failing call is kept.
int session_build(satori_session *s, const satori_model_desc *d, satori_session **out)
{
    int rc = session_plan_shards(s);
    if (!rc) rc = session_upload(s, d);
    if (!rc) rc = session_alloc_state(s);
    if (!rc) rc = build_graph(s);
    if (rc) {
        char buf[512];
        satori_last_error(buf, sizeof buf);
        std::string msg = buf;
        satori_session_destroy(s);
        return set_error(rc, "%s", msg.c_str());
    }
    *out = s;
    return SATORI_OK;
}

int session_check_desc(const satori_model_desc *d, int context) { return check_desc(d, context); }

int session_dalloc_bytes(satori_session *s, void **p, size_t bytes)
{
    uint8_t *b = nullptr;
    TRY(dalloc(s, &b, bytes));
    *p = b;
    return SATORI_OK;
}

extern "C" int satori_session_create(satori_ctx *ctx, const satori_model_desc *d, int context, satori_session **out)
{
    if (!ctx || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    DeviceScope scope(ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    TRY(check_desc(d, context));
    return session_build(session_new(ctx, d, context), d, out);
}

// Runs `count` steps fed from host tokens `feed` (one step per token).
static int peer_lost(satori_session *s)
{
    return set_error(SATORI_ERR_TIMEOUT, "a peer rank stopped answering; destroy the sharded session");
}

// A bounded wait that expired in a sharded step means a peer is gone: the ranks are out of step.
static int step_status(satori_session *s)
{
    const int rc = check_dev_error(s->ctx);
    if (rc == SATORI_ERR_TIMEOUT && s->world > 1) {
        s->failed = true;
        return peer_lost(s);
    }
    return rc;
}

static int run_steps(satori_session *s, const int *feed, int count, float *logits, int *argmax)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    if (s->failed) return peer_lost(s);
    if (count <= 0) return set_error(SATORI_ERR_ARGUMENT, "count must be positive");
    for (int i = 0; i < count; ++i)
        if (feed[i] < 0 || feed[i] >= s->vocab)
            return set_error(SATORI_ERR_ARGUMENT, "Token %d is outside the vocabulary.", feed[i]);
    if (s->position + count > s->context)
        return set_error(SATORI_ERR_CONTEXT_FULL, "Context limit %d reached; reset or enlarge the session.", s->context);
    satori_ctx *ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    TRYCUDA(clear_dev_error(ctx), "clear error");
    for (int i = 0; i < count; ++i) {
        s->h_ints[7] = feed[i];
        TRYCUDA(cudaMemcpyAsync(s->d_token, &s->h_ints[7], sizeof(int), cudaMemcpyHostToDevice, st), "token");
        TRYCUDA(cudaGraphLaunch(s->graph_exec, st), "graph launch");
        // The pinned token slot is reused by the next step: wait until this one has been read.
        if (i + 1 < count) TRYCUDA(cudaStreamSynchronize(st), "sync");
    }
    TRYCUDA(cudaMemcpyAsync(s->h_ints, s->d_ints, 7 * sizeof(int), cudaMemcpyDeviceToHost, st), "state");
    if (logits)
        TRYCUDA(cudaMemcpyAsync(s->h_logits, s->d_logits, (size_t)s->vocab * 4, cudaMemcpyDeviceToHost, st), "logits");
    int rc = step_status(s);
    s->position += count;
    if (rc) return rc;
    if (s->h_ints[4]) {
        cudaMemsetAsync(s->d_nonfinite, 0, sizeof(int), st);
        return set_error(SATORI_ERR_INVALID_DATA, "Non-finite logit.");
    }
    if (logits) memcpy(logits, s->h_logits, (size_t)s->vocab * 4);
    if (argmax) *argmax = s->h_ints[3];
    return SATORI_OK;
}

extern "C" int satori_session_append(satori_session *s, int token, float *logits, int *argmax)
{
    return run_steps(s, &token, 1, logits, argmax);
}

extern "C" int satori_session_append_tokens(satori_session *s, const int *tokens, int count, float *logits, int *argmax)
{
    if (!tokens) return set_error(SATORI_ERR_ARGUMENT, "tokens is null");
    return run_steps(s, tokens, count, logits, argmax);
}

extern "C" int satori_session_generate(satori_session *s, int first, int count, int *tokens_out)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    if (s->failed) return peer_lost(s);
    if (!tokens_out) return set_error(SATORI_ERR_ARGUMENT, "tokens_out is null");
    if (first < 0 || first >= s->vocab) return set_error(SATORI_ERR_ARGUMENT, "Token %d is outside the vocabulary.", first);
    if (count <= 0) return set_error(SATORI_ERR_ARGUMENT, "count must be positive");
    if (s->position + count > s->context)
        return set_error(SATORI_ERR_CONTEXT_FULL, "Context limit %d reached; reset or enlarge the session.", s->context);
    cudaStream_t st = s->ctx->stream;
    std::vector<int> out(count);
    int *d_out = s->d_gen;            // count <= context - position <= context
    s->h_ints[7] = first;
    cudaError_t e = cudaMemcpyAsync(s->d_token, &s->h_ints[7], sizeof(int), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = clear_dev_error(s->ctx);
    // First step consumes `first`; later steps consume the device-side argmax of the step before.
    for (int i = 0; i < count && e == cudaSuccess; ++i) {
        e = cudaGraphLaunch(s->graph_exec, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_out + i, s->d_argmax, sizeof(int), cudaMemcpyDeviceToDevice, st);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(out.data(), d_out, sizeof(int) * count, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->h_ints, s->d_ints, 7 * sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "generate");
    int rc = step_status(s);
    s->position += count;
    if (rc) return rc;
    if (s->h_ints[4]) {
        cudaMemsetAsync(s->d_nonfinite, 0, sizeof(int), st);
        return set_error(SATORI_ERR_INVALID_DATA, "Non-finite logit.");
    }
    memcpy(tokens_out, out.data(), sizeof(int) * count);
    return SATORI_OK;
}

extern "C" int satori_session_position(const satori_session *s, int *position)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    if (position) *position = s->position;
    return SATORI_OK;
}

extern "C" int satori_session_reset(satori_session *s)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    s->position = 0;
    cudaError_t e = cudaMemsetAsync(s->d_pos, 0, sizeof(int), s->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->ctx->stream);
    return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "reset");
}

extern "C" int satori_session_rewind(satori_session *s, int position)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    if (position < 0 || position > s->position)
        return set_error(SATORI_ERR_ARGUMENT, "position %d is outside the committed range [0, %d]", position,
                         s->position);
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    // The cache rows below `position` are untouched; the next step overwrites row `position`.
    s->position = position;
    s->h_ints[6] = position;
    cudaError_t e = cudaMemcpyAsync(s->d_pos, &s->h_ints[6], sizeof(int), cudaMemcpyHostToDevice, s->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->ctx->stream);
    return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "rewind");
}

extern "C" int satori_session_info(const satori_session *s, int *kernels_per_step, size_t *weight_bytes,
                                   size_t *kv_bytes_per_position)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    if (kernels_per_step) *kernels_per_step = s->kernels_per_step;
    if (weight_bytes) *weight_bytes = s->weight_bytes;
    if (kv_bytes_per_position) *kv_bytes_per_position = (size_t)s->layers * 2 * s->kv_local * sizeof(float);
    return SATORI_OK;
}

extern "C" int satori_session_stage(const satori_session *s, int which, float *out, size_t n)
{
    if (!s) return set_error(SATORI_ERR_DISPOSED, "session is disposed");
    const float *src = which == 0 ? s->d_hidden : which == 1 ? s->d_final : which == 2 ? s->d_logits : nullptr;
    const size_t len = which == 2 ? (size_t)s->vocab : (size_t)s->hidden;
    if (!src || !out || n != len) return set_error(SATORI_ERR_ARGUMENT, "bad stage %d / length %zu", which, n);
    DeviceScope scope(s->ctx->device);
    if (scope.status != cudaSuccess) return cuda_fail(scope.status, "cudaSetDevice");
    cudaError_t e = cudaMemcpyAsync(out, src, len * 4, cudaMemcpyDeviceToHost, s->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->ctx->stream);
    return e == cudaSuccess ? SATORI_OK : cuda_fail(e, "stage");
}

extern "C" int satori_session_destroy(satori_session *s)
{
    if (!s) return SATORI_OK;
    cudaSetDevice(s->ctx->device);
    cudaStreamSynchronize(s->ctx->stream);
    if (s->graph_exec) cudaGraphExecDestroy(s->graph_exec);
    session_destroy_sharding(s);
    for (void *p : s->allocations) cudaFree(p);
    if (s->h_ints) cudaFreeHost(s->h_ints);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    delete s;
    return SATORI_OK;
}
