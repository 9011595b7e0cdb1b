/*
 * satori_oracle.h -- CPU restatement of the Satori decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against (tests/, __graft_entry__.smoke(), and the cpu_baseline /
 * --impl reference legs of bench.py).  Nothing in the product path
 * (satori_b200/, include/) links, loads or calls it.
 *
 * Parity is pinned against the reference's own golden vectors and known-answer
 * tests (fixtures/gguf/v1, fixtures/operators JSON files, the Ternary2 and STQ2
 * byte KATs of tests/Satori.Numerics.Tests); see tests/test_oracle_golden.py.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the reference project root).  The reference is C#/.NET; its FP32 arithmetic
 * is IEEE single precision with no contraction, so this file is compiled with
 * -ffp-contract=off and uses fmaf()/_mm256_fmadd_ps exactly where the
 * reference calls Fma.MultiplyAdd.
 */
#ifndef SATORI_ORACLE_H
#define SATORI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes, mirroring the C# exception the reference throws. */
#define SO_OK 0
#define SO_ERR_ARGUMENT 1      /* ArgumentException / ArgumentOutOfRangeException */
#define SO_ERR_INVALID_DATA 2  /* InvalidDataException */
#define SO_ERR_NOT_SUPPORTED 3 /* NotSupportedException */
#define SO_ERR_CONTEXT_FULL 4  /* InvalidOperationException (context limit) */

/* Block formats (BlockQuantization.cs:3 for Q8_0/Q4_0; Ternary2 block sizes). */
#define SO_Q8_0 0
#define SO_Q4_0 1
#define SO_Q4_K 12
#define SO_Q6_K 14
#define SO_T2_64 64
#define SO_T2_128 128
#define SO_T2_256 256

/* ---------------- numeric helpers ---------------- */
float so_half_to_float(uint16_t bits);          /* BitConverter.UInt16BitsToHalf then (float) */
uint16_t so_float_to_half(float value);         /* round-to-nearest-even, for fixtures/quantizer */

/* ---------------- Ternary2 (src/Satori.Core/Ternary2*.cs) ---------------- */
int so_t2_geometry(int rows, int cols, int bs, int *blocks_per_row, int *block_bytes, int64_t *byte_length);
int so_t2_quantize(const float *w, int rows, int cols, int bs, uint8_t *out);
int so_t2_validate(const uint8_t *data, int64_t len, int rows, int cols, int bs);
int so_t2_dequantize(const uint8_t *data, int rows, int cols, int bs, float *out);
int so_t2_matvec_scalar(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y);
int so_t2_matvec_avx2(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y, int threads);
int so_t2_matvec_avx2_emulated(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y);
void so_stq2_write_header(uint8_t header[32], int rows, int cols, int bs);
int so_stq2_read_header(const uint8_t *header, int64_t file_len, int *rows, int *cols, int *bs);

/* ---------------- GGUF Q8_0 / Q4_0 (src/Satori.Core/QuantizedMatVec.cs etc.) ---------------- */
int so_q_geometry(int rows, int cols, int fmt, int *block_bytes, int64_t *byte_length);
int so_q_validate(const uint8_t *data, int64_t len, int rows, int cols, int fmt);
int so_q_decode_row(const uint8_t *row_bytes, int cols, int fmt, float *out);
int so_q_matvec_scalar(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y);
int so_q_matvec_avx2(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y, int threads);
int so_q_matvec_avx2_emulated(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y);
int so_q_matvec_batch(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions,
                      float *y, int threads);
int so_q_matvec_batch_emulated(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions,
                               float *y);
/* Not in the reference (it only decodes): this repository's own deterministic quantizer. */
/* K-quants (Q4KCodec.cs, Q6KCodec.cs, Q8KCodec.cs, QuantizedKAvx2Kernel.cs) */
int so_k_geometry(int rows, int cols, int fmt, int *block_bytes, int64_t *byte_length);
int so_k_validate(const uint8_t *data, int64_t len, int rows, int cols, int fmt);
int so_k_decode_row(const uint8_t *row_bytes, int cols, int fmt, float *out);
int so_k_matvec_scalar(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y);
int so_k_matvec_avx2(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y, int threads);
int so_q8k_quantize_row(const float *x, int cols, uint8_t *out);
int so_k_int_dot(const uint8_t *block, int fmt, const uint8_t *activation, int32_t *dot, int32_t *min_total);
int so_k_matvec_batch(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions, float *y,
                      int threads);
/* Ternary bitplane STB1 (TernaryBitplaneMatrix.cs, TernaryBitplaneMatVec.cs, TernaryBitplaneAvx2Kernel.cs) */
int so_tb_from_t2(const uint8_t *t2, int rows, int cols, int bs, uint8_t *out);
int so_tb_to_t2(const uint8_t *tb, int rows, int cols, int bs, uint8_t *out);
int so_tb_validate(const uint8_t *data, int64_t len, int rows, int cols, int bs);
int so_tb_matvec_scalar(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y);
int so_tb_matvec_avx2(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y);
int so_q_quantize(const float *w, int rows, int cols, int fmt, uint8_t *out);

/* ---------------- operators (src/Satori.Core/TransformerOps.cs) ---------------- */
int so_rmsnorm(const float *x, const float *w, int n, float eps, float *out);
int so_rmsnorm_heads(float *v, int n, const float *w, float eps, int head_dim);
int so_rope_half(float *v, int n, int head_dim, int position, double base, int rotary);
int so_rope_interleaved(float *v, int n, int head_dim, int position);
int so_swiglu(const float *gate, const float *up, int n, float *out);
int so_add(const float *a, const float *b, int n, float *out);
int so_grouped_attention(const float *q, const float *keys, const float *values, int q_heads, int kv_heads,
                         int head_dim, int tokens, double *scores, float *out, int threads);
int so_greedy_select(const float *logits, int n, int *token);

/* ---------------- dense decode (src/Satori.Core/Model/DenseForward.cs, DenseSession.cs) ---------------- */
typedef struct so_layer {
    const float *attn_norm, *ffn_norm;        /* [hidden] */
    const float *q_bias, *k_bias, *v_bias;    /* optional, NULL when absent */
    const uint8_t *q, *k, *v, *o, *gate, *up, *down;
    int q_fmt, k_fmt, v_fmt, o_fmt, gate_fmt, up_fmt, down_fmt;
} so_layer;

typedef struct so_model {
    int layers, hidden, ffn, q_heads, kv_heads, head_dim, vocab;
    float eps;
    double rope_base;
    const uint8_t *embd; int embd_fmt;        /* token_embd.weight [vocab rows x hidden cols] */
    const uint8_t *output; int output_fmt;    /* output.weight [vocab rows x hidden cols] */
    const float *output_norm;
    const so_layer *layer;                    /* [layers] */
} so_model;

typedef struct so_session so_session;
so_session *so_session_create(const so_model *model, int context);
void so_session_destroy(so_session *s);
void so_session_reset(so_session *s);
int so_session_fill_cache(so_session *s, int position, uint32_t seed);
int so_session_position(const so_session *s);
/* Appends one token; writes logits [vocab] and the greedy token.  threads parallelises rows/heads only. */
int so_session_append(so_session *s, int token, float *logits, int *argmax, int threads);
/* Copy of a stage value of the last append (for stage parity): 0 = hidden after last layer,
 * 1 = final_norm output. */
int so_session_stage(const so_session *s, int which, float *out, int n);

#ifdef __cplusplus
}
#endif
#endif
