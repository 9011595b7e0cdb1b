// ops.cuh -- decode-step glue kernels (TransformerOps restated for the device).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace satori {

// TransformerOps.RmsNorm (src/Satori.Core/TransformerOps.cs:13-22): FP64 sum of squares,
// scale = 1/sqrt(sum/n + eps), out = (float)(x * scale * w).
cudaError_t launch_rmsnorm(const float *x, const float *w, int n, float eps, float *out, cudaStream_t s, int pdl);
// TransformerOps.RmsNormHeads (:122-135), in place.
cudaError_t launch_rmsnorm_heads(float *v, int n, const float *w, float eps, int head_dim, cudaStream_t s, int pdl);
// TransformerOps.SwiGlu (:41-51): FP64 sigmoid.
cudaError_t launch_swiglu(const float *gate, const float *up, int n, float *out, cudaStream_t s, int pdl);
// DenseForward.Embed via GgufQuantizedMatrix.ReadRow (Q8_0 rows): token from *token_dev; also writes
// *tokens_dev = *pos_dev + 1 (the attention prefix length of this step).  With rope_table non-null it
// also writes the step's RoPE factors (cos, sin of TransformerOps.RopeHalf's angle for pair k at
// position *pos_dev, k < rotary/2) for every layer's rope_append to read.
cudaError_t launch_embed(const uint8_t *embd, int cols, const int *token_dev, const int *pos_dev, int *tokens_dev,
                         float *hidden, double *rope_table, double rope_base, int rotary, cudaStream_t s, int pdl);
// Prefill chunk forms (`positions` vectors, one after another unless a stride is given; no PDL):
// RmsNorm of each position's vector, RmsNormHeads of each position's heads (vectors `stride` floats
// apart), and the embedding rows of tokens_dev[0..positions) with the RoPE factors of positions
// pos0 .. pos0 + positions - 1 ([positions][rotary/2][cos, sin]).
cudaError_t launch_rmsnorm_batch(const float *x, const float *w, int n, float eps, float *out, int positions,
                                 cudaStream_t s);
cudaError_t launch_rmsnorm_heads_batch(float *v, int n, const float *w, float eps, int head_dim, long long stride,
                                       int positions, cudaStream_t s);
cudaError_t launch_embed_batch(const uint8_t *embd, int cols, const int *tokens_dev, int positions, int pos0,
                               float *hidden, double *rope_table, double rope_base, int rotary, cudaStream_t s);
// GreedyTokenSelector.Select (src/Satori.Core/GreedyTokenSelector.cs:6-16): smallest index of the
// maximum; a non-finite logit sets *nonfinite_dev.  Then advances *pos_dev and feeds *token_dev.
// `scratch` = 4 zeroed words (8-byte aligned) the launch leaves zeroed again.
cudaError_t launch_argmax_advance(const float *logits, int n, int *argmax_dev, int *nonfinite_dev, int *pos_dev,
                                  int *token_dev, unsigned *scratch, int sm_count, cudaStream_t s, int pdl);

}  // namespace satori
