// attention.cuh -- decode grouped-query attention (split-K flash decoding) launch interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace satori {

struct AttnArgs {
    const float *q;       // [q_heads * head_dim], RoPE already applied
    const float *keys;    // token-major [tokens][kv_heads * head_dim]
    const float *values;
    int q_heads, kv_heads, head_dim;
    int kv_stride;        // floats between consecutive tokens' rows; 0 = kv_heads * head_dim
    int tokens;           // used when tokens_dev == nullptr
    const int *tokens_dev;  // device-side token count (decode graphs: position + 1)
    int max_tokens;       // upper bound of tokens (sizes the split plan)
    float *out;           // [q_heads * head_dim]
    float *scratch;       // partial records, attn_scratch_floats() floats
    unsigned *err;
    int use_pdl;
    // Prefill chunk of `batch` positions (0 or 1: one position): position z reads q + z * q_pstride,
    // attends to the first tokens + z tokens (the causal prefix; tokens_dev must be null) and writes
    // out + z * out_pstride.
    int batch;
    long long q_pstride, out_pstride;
};

// Number of split-K work units (CTAs along the sequence) for a given shape.
int attn_splits(int q_heads, int kv_heads, int head_dim, int max_tokens, int sm_count, int batch = 1);
// Scratch the partial records need: batch * splits * q_heads * (head_dim + 2) floats.
size_t attn_scratch_floats(int q_heads, int kv_heads, int head_dim, int max_tokens, int sm_count, int batch = 1);
cudaError_t launch_attention(const AttnArgs &a, int sm_count, cudaStream_t stream);

// RopeHalf on q and k at `position`, then append k and v at slot `position` of the cache; the
// rotated q goes to q_out.  position comes from *position_dev when non-null.
struct RopeAppendArgs {
    const float *q, *k, *v;
    float *q_out;
    float *k_cache, *v_cache;   // [context][kv_heads*head_dim] of one layer
    int q_heads, kv_heads, head_dim, rotary;
    double base;
    int position;
    const int *position_dev;
    const double *table;        // optional [rotary/2][cos, sin] for this position (launch_embed writes it)
    int use_pdl;
    // Prefill chunk of `batch` positions (0 or 1: one): position z = position + z reads q/k/v + z * in_stride,
    // writes q_out + z * q_heads * head_dim and its cache slot, and takes table + z * rotary when a table
    // is given.  position_dev must be null.
    int batch;
    long long in_stride;
};
cudaError_t launch_rope_append(const RopeAppendArgs &a, cudaStream_t stream);

// RopeHalf alone, in place on a device vector (n floats).
cudaError_t launch_rope_half(float *v, int n, int head_dim, int position, double base, int rotary,
                             cudaStream_t stream);

}  // namespace satori
