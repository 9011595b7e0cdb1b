// session_internal.h -- state of a decode session (single GPU or one rank of a sharded model).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "capi_internal.h"

struct DevMatrix {
    const uint8_t *payload = nullptr;
    int rows = 0, cols = 0, format = 0;
};

struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    float *q_bias = nullptr, *k_bias = nullptr, *v_bias = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
    DevMatrix q, k, v, o, gate, up, down;
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
    size_t weight_bytes = 0;

    std::vector<Layer> layer;
    DevMatrix embd, output;
    float *output_norm = nullptr;

    float *d_kcache = nullptr, *d_vcache = nullptr;
    float *d_hidden = nullptr, *d_normed = nullptr, *d_final = nullptr, *d_proj = nullptr;
    float *d_q = nullptr, *d_qrot = nullptr, *d_ctx = nullptr, *d_k = nullptr, *d_v = nullptr;
    float *d_gate = nullptr, *d_up = nullptr, *d_act = nullptr, *d_logits = nullptr;
    float *d_attn_scratch = nullptr;
    int *d_ints = nullptr;
    int *d_token = nullptr, *d_pos = nullptr, *d_tokens = nullptr, *d_argmax = nullptr, *d_nonfinite = nullptr;
    int *h_ints = nullptr;
    float *h_logits = nullptr;

    cudaGraphExec_t graph_exec = nullptr;
    std::vector<void *> allocations;

    ShardState *shard = nullptr;
};

int session_alloc_state(satori_session *s);
void session_destroy_sharding(satori_session *s);
