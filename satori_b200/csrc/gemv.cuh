// gemv.cuh -- quantized MatVec (Q8_0, Q4_0, Ternary2) launch interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "xchg.cuh"

namespace satori {

// Optional fused epilogue of the MatVec (decode-step glue; each reproduces the reference op):
//   y = acc                       (kEpiNone)
//   y = acc + bias                (kEpiBias: TransformerOps.Add(query, bias, query), DenseForward.cs:124-129)
//   y = residual + acc, residual := y  (kEpiResidual: TransformerOps.Add(residual, projected, residual),
//                                      DenseForward.cs:148,160)
//   y[r/2] = SwiGlu(acc[r], acc[r+1]) for even r  (kEpiSwiGlu: rows interleave ffn_gate and ffn_up row by
//                                      row; TransformerOps.SwiGlu, DenseForward.cs:151-153; gemv_rows only)
enum Epilogue : int { kEpiNone = 0, kEpiBias = 1, kEpiResidual = 2, kEpiSwiGlu = 3 };

struct GemvArgs {
    const uint8_t *payload;  // device, 256-byte aligned, readable 16 bytes past the end
    int rows, cols, format;  // format: 0 Q8_0, 1 Q4_0, 64/128/256 Ternary2
    int order;               // satori_order
    const float *x;          // device [positions][cols]
    float *y;                // device [positions][rows]
    int positions;
    int epilogue;
    const float *bias;       // [rows] for kEpiBias
    float *residual;         // [rows] for kEpiResidual (positions == 1)
    unsigned *err;           // device error word
    int use_pdl;             // launched with programmatic stream serialization
    const float *norm_w;     // non-null: x is RmsNorm'ed on the fly with these weights (gemv_rows only)
    float norm_eps;
    XPush xp;                // sharded step: push the epilogue's output to the peers (gemv_rows only)
    XWait xw;                // sharded step: wait for the peers' slices of x first (gemv_rows only)
    const uint8_t *next_payload;  // gemv_stream: weights of the next MatVec, whose head this launch
    size_t next_bytes;            // prefetches into L2 once its own last stage has landed (0: none)
};

// Geometry the host chooses for one launch.
struct GemvPlan {
    int grid, threads, rows_per_cta, chunk_blocks, nchunks, stages, seg_stride, dstride;
    size_t smem;
    int ok;
};

GemvPlan plan_gemv(int rows, int cols, int format, int positions, int sm_count, size_t smem_limit);

// Decode-order MatVec of one position for Q8_0 / Q4_0 with cols % 256 == 0: gemv_rows.cu (up to
// 24576 columns, kind 1) and gemv_decode.cu (column chunks, any width, kind 2).  A plan function returns
// ok = 0 for any argument set its kernel does not take.
struct DecodePlan {
    int ok, kind, grid, rc, stages, nchunks, rs;
    int cw, nb, fold;     // gemv_rows: compute warps, block columns per lane, rows per fold batch
    size_t smem;
};
DecodePlan plan_gemv_rows(const GemvArgs &a, int sm_count, size_t smem_limit);
// True when the decode-order rows kernel takes this shape with this epilogue (and so the fused SwiGLU
// epilogue and the fused RmsNorm of x).
bool gemv_rows_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit);
cudaError_t launch_gemv_rows(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream);
// gemv_stream.cu: the same order for the decode configurations' row widths with the width fixed at
// compile time (kind 3); preferred over gemv_rows where it takes the shape.
DecodePlan plan_gemv_stream(const GemvArgs &a, int sm_count, size_t smem_limit);
bool gemv_stream_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit);
cudaError_t launch_gemv_stream(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream);
// True when one of the two decode row kernels takes the shape (and with it the fused RmsNorm of x, the
// SwiGLU epilogue and a carried peer exchange).
bool gemv_fused_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit);
DecodePlan plan_gemv_decode(const GemvArgs &a, int sm_count, size_t smem_limit);
cudaError_t launch_gemv_decode(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream);
cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &plan, cudaStream_t stream);
// gemv_kquant.cu: GGUF Q4_K / Q6_K (batch order: Q8_K activations and exact integer products; scalar and
// execute orders in FP32), their row decode and validation.
bool is_kquant(int format);
cudaError_t launch_kq_gemv(const GemvArgs &a, cudaStream_t stream);
cudaError_t launch_kq_decode_row(const uint8_t *payload, int cols, int format, const int *row_dev, int row_host,
                                 float *out, cudaStream_t stream);
cudaError_t launch_kq_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                               cudaStream_t stream);
// gemv_ternary.cu: the row-streaming ternary MatVec in the AVX2 order for Ternary2 and bitplane matrices
// (*taken = false when the shape does not qualify; nothing is launched then), and the bitplane fallbacks.
bool is_bitplane(int format);
int ternary_block_size(int format);
cudaError_t launch_ternary_stream(const GemvArgs &a, int sm_count, size_t smem_limit, cudaStream_t stream,
                                  bool *taken);
cudaError_t launch_bitplane_rowwise(const GemvArgs &a, cudaStream_t stream);
cudaError_t launch_bitplane_decode_row(const uint8_t *payload, int cols, int format, const int *row_dev,
                                       int row_host, float *out, cudaStream_t stream);
cudaError_t launch_bitplane_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                                     cudaStream_t stream);
// prefill_gemm.cu: the projection of a chunk of up to 128 positions on the tensor cores (Q8_0 / Q4_0,
// cols % 64 == 0).  Not the reference's FP32 order: exact products, FP32 accumulation in tensor memory.
struct TcGemm {
    const uint8_t *payload;
    int rows, cols, format;
    const float *x;          // [positions][cols]
    int positions;
    int epilogue;            // kEpiNone / kEpiBias / kEpiResidual / kEpiSwiGlu
    float *y;                // y[p * ldy + r] (SwiGlu: y[p * ldy + r / 2]); unused by kEpiResidual when null
    int ldy;                 // 0: rows (SwiGlu: rows / 2)
    const float *bias;
    float *residual;         // residual[p * ldr + r] += acc
    int ldr;                 // 0: rows
    uint8_t *scratch;        // tc_scratch_bytes(); 256-byte aligned
    size_t scratch_bytes;
    unsigned *err;
};
bool tc_gemm_takes(int rows, int cols, int format, int positions, int epilogue);
size_t tc_scratch_bytes(int rows, int cols, int positions, int sm_count);
cudaError_t launch_tc_gemm(const TcGemm &g, int sm_count, cudaStream_t stream);
int gemv_block_bytes(int format);
int gemv_block_elems(int format);

// Row decode (GgufQuantizedMatrix.ReadRow / Ternary2Matrix.Dequantize), device pointers.
cudaError_t launch_decode_row(const uint8_t *payload, int rows, int cols, int format, const int *row_dev,
                              int row_host, float *out, cudaStream_t stream);

// Payload validation on the device: writes 0 or a satori_status into *status_dev.
cudaError_t launch_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                            cudaStream_t stream);

// Ternary2Matrix.Quantize on the device (bit-exact), and this library's own Q8_0/Q4_0 quantizer.
cudaError_t launch_t2_quantize(const float *w, int rows, int cols, int bs, uint8_t *out, int *status_dev,
                               cudaStream_t stream);
cudaError_t launch_q_quantize(const float *w, int rows, int cols, int format, uint8_t *out, cudaStream_t stream);

}  // namespace satori
