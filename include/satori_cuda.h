/*
 * satori_cuda.h -- C ABI of the B200 (sm_100a) decode hot path for Satori.
 *
 * Plain C types only: host/device pointers, sizes, ints.  Every function returns a
 * satori_status; on any error the caller's output buffers are left untouched (the
 * "commits output only on success" contract of IQuantizedMatrix.Execute,
 * src/Satori.Core/IQuantizedMatrix.cs:6) and satori_last_error() describes the failure.
 * Reference paths are relative to the Satori project root.
 *
 * Threading: a context serialises its calls on one CUDA stream; handles are not
 * thread-safe, exactly like DenseSession (src/Satori.Core/Model/DenseSession.cs:11-12).
 */
#ifndef SATORI_CUDA_H
#define SATORI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SATORI_API __attribute__((visibility("default")))
#else
#define SATORI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum satori_status {
    SATORI_OK = 0,
    SATORI_ERR_ARGUMENT = 1,      /* ArgumentException / ArgumentOutOfRangeException */
    SATORI_ERR_INVALID_DATA = 2,  /* InvalidDataException (non-finite scale, bad STQ2 payload) */
    SATORI_ERR_NOT_SUPPORTED = 3, /* NotSupportedException (e.g. Q4_0 embedding rows) */
    SATORI_ERR_CONTEXT_FULL = 4,  /* InvalidOperationException: context limit reached */
    SATORI_ERR_DISPOSED = 5,      /* ObjectDisposedException */
    SATORI_ERR_CUDA = 6,          /* device or driver failure (IOException-like fault) */
    SATORI_ERR_TIMEOUT = 7,       /* a bounded device-side wait expired */
    SATORI_ERR_OUT_OF_MEMORY = 8
} satori_status;

/* Weight formats: GGUF Q8_0 / Q4_0 (src/Satori.Core/BlockQuantization.cs:3) and Ternary2 blocks. */
typedef enum satori_format {
    SATORI_Q8_0 = 0,
    SATORI_Q4_0 = 1,
    SATORI_Q4_K = 12,   /* GGUF Q4_K: 256-weight super-blocks of 144 bytes (Q4KCodec.cs) */
    SATORI_Q6_K = 14,   /* GGUF Q6_K: 256-weight super-blocks of 210 bytes (Q6KCodec.cs) */
    SATORI_T2_64 = 64,
    SATORI_T2_128 = 128,
    SATORI_T2_256 = 256,
    /* Ternary bitplane (docs/ternary-bitplane-v1.md, src/Satori.Core/TernaryBitplaneMatrix.cs): the same blocks
     * as Ternary2 with a positive and a negative bit plane instead of 2-bit codes. */
    SATORI_TB_64 = 1064,
    SATORI_TB_128 = 1128,
    SATORI_TB_256 = 1256
} satori_format;

/* Which reference routine's FP32 operation order a MatVec reproduces (bit for bit). */
typedef enum satori_order {
    /* Q8_0/Q4_0: QuantizedMatVec.Execute -> QuantizedAvx2Kernel.Execute (QuantizedMatVec.cs:12-16);
       Ternary2:  Ternary2MatVec.Execute -> Ternary2Avx2Kernel.Execute (Ternary2MatVec.cs:9-22). */
    SATORI_ORDER_EXECUTE = 0,
    /* QuantizedMatVec.ExecuteScalar (:45-78); Ternary2MatVec.ExecuteScalar (Ternary2MatVec.cs:38-42). */
    SATORI_ORDER_SCALAR = 1,
    /* QuantizedMatVec.ExecuteBatch -> ExecuteBatchFloat/Dot with FMA (:104-120, 221-365): the decode path. */
    SATORI_ORDER_BATCH = 2,
    /* ExecuteBatch's result for a prefill chunk on the tensor cores (Q8_0 / Q4_0, cols % 64 == 0, any number
       of positions): NOT bit-exact.  Weights and activations are split exactly into bf16 parts, every product
       is exact, and the sum is accumulated in FP32 in tensor memory, so |y - y_ref| stays within a few FP32
       roundings of sum|w*x| (the prefill tests bound it at 2e-6 of sum|w*x| + 1e-30). */
    SATORI_ORDER_TENSOR = 3
} satori_order;

typedef struct satori_ctx satori_ctx;
typedef struct satori_matrix satori_matrix;
typedef struct satori_attn satori_attn;
typedef struct satori_session satori_session;

/* ------------------------------------------------------------------ context */
/* Opens device `device` (one context per caller; replaces VulkanContext.TryCreate,
 * src/Satori.Backends.Vulkan/VulkanContext.cs:57).  A process may hold contexts on several devices and
 * call from any thread: the entry points that take host buffers, allocate or run a session step make
 * the handle's device current for the call and then restore the caller's.  The device-pointer entry
 * points (..._device, satori_grouped_attention_noalloc) run on the calling thread's current device,
 * which must be the one that holds the pointers (and the context's device). */
SATORI_API int satori_init(int device, satori_ctx **out);
SATORI_API int satori_destroy(satori_ctx *ctx);
/* Copies the calling thread's last error message (NUL-terminated, truncated to n). */
SATORI_API int satori_last_error(char *buf, size_t n);
/* Library build identity: writes "satori-b200 <version> sm_100a". */
SATORI_API int satori_version(char *buf, size_t n);
/* The context's CUDA stream as an opaque pointer (cudaStream_t), for device-pointer calls. */
SATORI_API void *satori_stream(satori_ctx *ctx);
/* Routes the context's device work to a caller-owned cudaStream_t (NULL restores the context's own
 * stream), e.g. to capture device-pointer calls into the caller's CUDA graph. */
SATORI_API int satori_set_stream(satori_ctx *ctx, void *stream);
/* Waits for the work queued on the context's current stream; reports a device error a kernel recorded
 * (SATORI_ERR_TIMEOUT for an expired bounded wait) like the synchronous calls do. */
SATORI_API int satori_synchronize(satori_ctx *ctx);

/* ------------------------------------------------------------------ matrices */
/* IQuantizedMatrixFactory.Create (src/Satori.Core/IQuantizedMatrixFactory.cs:6) and
 * Ternary2Matrix.FromPacked (src/Satori.Core/Ternary2Matrix.cs:73-81): validates the payload
 * exactly like QuantizedMatVec.ValidatePayload (QuantizedMatVec.cs:28-42) /
 * Ternary2Matrix.ValidatePayload (Ternary2Matrix.cs:83-101), then uploads it once, unchanged in
 * layout.  `payload` is borrowed only for the duration of the call. */
SATORI_API int satori_matrix_create(satori_ctx *ctx, const uint8_t *payload, size_t bytes, int rows, int cols,
                                    int format, satori_matrix **out);
/* Same, from a payload already in device memory (copied, then validated on the device). */
SATORI_API int satori_matrix_create_device(satori_ctx *ctx, const uint8_t *device_payload, size_t bytes, int rows,
                                           int cols, int format, satori_matrix **out);
/* IQuantizedMatrix.Execute (IQuantizedMatrix.cs:6), GgufQuantizedMatrix.Execute
 * (src/Satori.Formats.Gguf/GgufQuantizedMatrix.cs:38-40), Ternary2MatVec.Execute /
 * MappedTernary2Matrix.Execute (Ternary2MatVec.cs:9, MappedTernary2Matrix.cs:43): host x[cols] ->
 * host y[rows], synchronous, SATORI_ORDER_EXECUTE arithmetic. */
SATORI_API int satori_matrix_execute(satori_matrix *m, const float *x, float *y);
/* ExecuteScalar twins (QuantizedMatrix.cs:18-19, GgufQuantizedMatrix.cs:50-52, Ternary2MatVec.cs:38). */
SATORI_API int satori_matrix_execute_scalar(satori_matrix *m, const float *x, float *y);
/* QuantizedMatVec.ExecuteBatch / GgufQuantizedMatrix.ExecuteBatch (GgufQuantizedMatrix.cs:43-48):
 * x[positions][cols] -> y[positions][rows], position-major, host pointers. Q8_0/Q4_0 only. */
SATORI_API int satori_matrix_execute_batch(satori_matrix *m, const float *x, int positions, float *y);
/* The same product in SATORI_ORDER_TENSOR (host x[positions][cols], y[positions][rows]). */
SATORI_API int satori_matrix_execute_tensor(satori_matrix *m, const float *x, int positions, float *y);
/* Device-pointer form of all three on the context stream (asynchronous). */
SATORI_API int satori_matrix_execute_device(satori_matrix *m, const float *dx, float *dy, int positions, int order);
/* GgufQuantizedMatrix.ReadRow (GgufQuantizedMatrix.cs:54-61): decodes one row to host memory,
 * bit-exact; Q4_0 rows are rejected with SATORI_ERR_NOT_SUPPORTED as in the reference.  For
 * Ternary2 it decodes one row like Ternary2Matrix.Dequantize (Ternary2Matrix.cs:103-120). */
SATORI_API int satori_matrix_read_row(satori_matrix *m, int row, float *out);
/* The matrix's shape, satori_format and payload length (IQuantizedMatrix.Rows / Columns). */
SATORI_API int satori_matrix_info(const satori_matrix *m, int *rows, int *cols, int *format, size_t *bytes);
/* Device address of the resident payload (read-only), e.g. for a caller-managed graph. */
SATORI_API const uint8_t *satori_matrix_device_payload(const satori_matrix *m);
SATORI_API int satori_matrix_destroy(satori_matrix *m);

/* ------------------------------------------------------------------ quantizers */
/* Ternary2Matrix.Quantize (Ternary2Matrix.cs:38-71), computed on the device, bit-exact:
 * host weights[rows*cols] -> host payload (Ternary2 geometry, Ternary2Shape.cs:14). */
SATORI_API int satori_ternary2_quantize(satori_ctx *ctx, const float *weights, int rows, int cols, int block_size,
                                        uint8_t *payload);
/* Not in the reference (it only decodes GGUF): this library's own Q8_0/Q4_0 quantizer, used to
 * build seeded synthetic weights.  Device pointers, on the context stream. */
SATORI_API int satori_quantize_q_device(satori_ctx *ctx, const float *d_weights, int rows, int cols, int format,
                                        uint8_t *d_payload);

/* ------------------------------------------------------------------ attention */
/* TransformerOps.GroupedAttention (src/Satori.Core/TransformerOps.cs:140-179) on device pointers:
 * q[q_heads*head_dim], keys/values token-major [tokens][kv_heads*head_dim] -> out[q_heads*head_dim].
 * Split-K flash decoding (FP32) with partial-softmax merge; asynchronous on the context stream. */
SATORI_API int satori_grouped_attention_device(satori_ctx *ctx, const float *q, const float *keys,
                                               const float *values, int q_heads, int kv_heads, int head_dim,
                                               int tokens, float *out);
/* Host-pointer twin (synchronous). */
SATORI_API int satori_grouped_attention(satori_ctx *ctx, const float *q, const float *keys, const float *values,
                                        int q_heads, int kv_heads, int head_dim, int tokens, float *out);
/* No counterpart in the reference.  Grouped attention for callers that cannot allocate device
 * memory (for example a host that has already given the whole GPU to its own memory pool, or a path
 * that cannot afford cudaMalloc's device-wide synchronisation): the same kernels and result as
 * satori_grouped_attention_device, with their split-K scratch in a fixed 4 MiB array inside the
 * library's device image instead of a context allocation.  No context: device pointers and a
 * cudaStream_t (NULL = legacy default stream) on the current device.  The call allocates nothing; its
 * first call on a device looks up that array's address, so make that first call before any stream
 * capture.  Shapes whose partial records exceed 1,048,576 floats are rejected with
 * SATORI_ERR_ARGUMENT.  Calls share the one array: two calls that overlap on the GPU race.  The call
 * returns before the GPU runs, so unlike the context entry point it reports no SATORI_ERR_TIMEOUT: a
 * bounded wait that expires inside the streaming kernel instead sends the affected heads to the FP64
 * recomputation from K and V. */
SATORI_API int satori_grouped_attention_noalloc(const float *q, const float *keys, const float *values,
                                                int q_heads, int kv_heads, int head_dim, int tokens, float *out,
                                                void *stream);
/* TransformerOps.RopeHalf (TransformerOps.cs:99-118) on a host vector, in place (FP64 angles). */
SATORI_API int satori_rope_half(satori_ctx *ctx, float *vector, int n, int head_dim, int position, double base,
                                int rotary);

/* A device-resident FP32 KV cache for `layers` layers (DenseSession.cs:80-84 layout:
 * [layer][context][kv_heads*head_dim], token-major). */
SATORI_API int satori_attn_create(satori_ctx *ctx, int layers, int context, int q_heads, int kv_heads, int head_dim,
                                  double rope_base, satori_attn **out);
/* The attention half of DenseForward.Step (DenseForward.cs:135-143): RopeHalf on q and k at
 * `position`, append k and v at slot `position` of `layer`, GroupedAttention over position+1
 * tokens.  Host pointers (q/k/v as projected, bias already added); out = context[q_heads*head_dim]. */
SATORI_API int satori_attn_append(satori_attn *a, int layer, int position, const float *q, const float *k,
                                  const float *v, float *out);
SATORI_API int satori_attn_destroy(satori_attn *a);

/* ------------------------------------------------------------------ dense decode session */
/* One tensor of the model description (names follow GGUF: token_embd.weight, blk.N.attn_q.weight ...). */
typedef struct satori_tensor {
    const char *name;
    const void *data;   /* host or device pointer (unified addressing): payload bytes, or float32 values */
    size_t bytes;
    int format;         /* satori_format for matrices, -1 for float32 vectors */
    int rows, cols;     /* matrices: rows x cols; vectors: rows = length, cols = 1 */
} satori_tensor;

typedef struct satori_model_desc {
    int layers, hidden, ffn, q_heads, kv_heads, head_dim, vocab;
    float rms_epsilon;   /* ModelShape.RmsNormEpsilon cast to float, as DenseForward.cs:49 */
    double rope_base;
    int tied_embeddings; /* output projection is token_embd.weight (DenseForward.cs:52) */
    int n_tensors;
    const satori_tensor *tensors;
} satori_model_desc;

/* DenseSession (DenseSession.cs:47-90) with every tensor uploaded once and the whole step
 * (embed, every layer, final norm, logits, greedy argmax) run on the device. */
SATORI_API int satori_session_create(satori_ctx *ctx, const satori_model_desc *desc, int context,
                                     satori_session **out);
/* Multi-GPU variant (no counterpart in the reference, which runs on one CPU): this process is `rank`
 * of `world`, one process per GPU, all ranks calling together.  Every projection is row-sharded (a
 * row's FP32 chain stays on one GPU, so logits equal the single-GPU session's); attention is sharded
 * by query heads, each rank caching only the KV heads its heads read; the context, the residual
 * after attn_output / ffn_down, the SwiGLU activations and the logits are all-gathered inside the
 * step's CUDA graph -- by default with peer stores over NVLink into IPC-mapped buffers, carried by the
 * producing MatVec launches where they can (SATORI_EXCHANGE=nccl selects NCCL all-gathers).  hidden,
 * ffn and vocab must be multiples of `world` (SATORI_ERR_NOT_SUPPORTED otherwise).  Every rank passes the full tensor table and uploads only
 * its rows.  `nccl_unique_id` is the 128-byte id from satori_nccl_unique_id on rank 0.  world = 1 is
 * satori_session_create. */
SATORI_API int satori_session_create_sharded(satori_ctx *ctx, const satori_model_desc *desc, int context, int rank,
                                             int world, const void *nccl_unique_id, satori_session **out);
/* ncclGetUniqueId through the NCCL library loaded at run time (128 bytes into out128). */
SATORI_API int satori_nccl_unique_id(void *out128);

/* One large MatVec split by rows over the GPUs of a node (the row-sharded GEMV with an all-gather of y):
 * IQuantizedMatrix.Execute (IQuantizedMatrix.cs:6) / QuantizedMatVec.ExecuteBatch (QuantizedMatVec.cs:104-120)
 * with rank r of `world` holding rows [r*S, min((r+1)*S, rows)), S = ceil(rows / world).  `payload` is the
 * WHOLE matrix (host, or device when payload_on_device), of which only this rank's rows are uploaded;
 * every rank passes the same NCCL id (satori_nccl_unique_id on rank 0).  Execute computes this rank's rows
 * with the single-GPU kernels (each row bit-exact to the reference in `order`) and all-gathers the full
 * y[rows] onto every rank over NCCL; all ranks call it together.  Every rank must receive at least one
 * row (SATORI_ERR_NOT_SUPPORTED otherwise). */
typedef struct satori_matrix_sharded satori_matrix_sharded;
SATORI_API int satori_matrix_create_sharded(satori_ctx *ctx, const uint8_t *payload, size_t bytes, int rows, int cols,
                                            int format, int payload_on_device, int rank, int world,
                                            const void *nccl_unique_id, satori_matrix_sharded **out);
/* dx [cols], dy [rows] on this rank's device; the context's stream. */
SATORI_API int satori_matrix_sharded_execute_device(satori_matrix_sharded *m, const float *dx, float *dy, int order);
/* Host vectors, synchronous; y committed only on success. */
SATORI_API int satori_matrix_sharded_execute(satori_matrix_sharded *m, const float *x, float *y, int order);
/* The rows [row_begin, row_end) this rank holds and computes. */
SATORI_API int satori_matrix_sharded_info(const satori_matrix_sharded *m, int *row_begin, int *row_end);
SATORI_API int satori_matrix_sharded_destroy(satori_matrix_sharded *m);
/* DenseSession.Append (DenseSession.cs:111-131) + GreedyTokenSelector.Select
 * (src/Satori.Core/GreedyTokenSelector.cs:6-16): logits (host, may be NULL) and argmax (may be NULL). */
SATORI_API int satori_session_append(satori_session *s, int token, float *logits, int *argmax);
/* Appends `count` tokens one decode step at a time (prefill by repeated decode); writes the last
 * position's logits/argmax. */
SATORI_API int satori_session_append_tokens(satori_session *s, const int *tokens, int count, float *logits,
                                            int *argmax);
/* DenseSession.Forward (DenseSession.cs:136-181) with the prefill on the tensor cores: all tokens but the
 * last run in chunks of up to 128 positions through DenseForward.LayerBatch's phases (DenseForward.cs:178-262),
 * each projection one tcgen05 GEMM (SATORI_ORDER_TENSOR, so the cache rows match the per-token path to FP32
 * rounding, not bit for bit); the last token runs through the decode step and yields logits/argmax as in
 * satori_session_append_tokens.  Sharded sessions, one token, and weights other than Q8_0 / Q4_0 with
 * multiples of 64 columns take the per-token path unchanged. */
SATORI_API int satori_session_forward_tensor(satori_session *s, const int *tokens, int count, float *logits,
                                             int *argmax);
/* Greedy generation: appends `first`, then feeds back the argmax `count - 1` more times; writes the
 * `count` greedy tokens (TextGenerator.GenerateFromTokens' decode loop, TextGenerator.cs:62-99). */
SATORI_API int satori_session_generate(satori_session *s, int first, int count, int *tokens_out);
/* DenseSession.Position (DenseSession.cs:96): the number of cached positions. */
SATORI_API int satori_session_position(const satori_session *s, int *position);
SATORI_API int satori_session_reset(satori_session *s);    /* DenseSession.Reset (:189) */
/* No counterpart in the reference (its DenseSession only resets to position 0): discards the
 * positions at and after `position` (0 <= position <= the current position), keeping the cached
 * K/V of the earlier ones, so a prompt's cache can be decoded from again without re-running it. */
SATORI_API int satori_session_rewind(satori_session *s, int position);
/* No counterpart in the reference: kernels launched per decode step (the captured graph's kernel
 * nodes), payload bytes of the weights this session (or rank) holds, and the bytes of K/V one cached
 * position occupies on this device (every decode step reads that much per position of context). */
SATORI_API int satori_session_info(const satori_session *s, int *kernels_per_step, size_t *weight_bytes,
                                   size_t *kv_bytes_per_position);
/* Copies a stage tensor of the last step to the host: 0 = hidden after the last layer,
 * 1 = final_norm output, 2 = logits (stage parity, ForwardObserver in DenseForward.cs:6). */
SATORI_API int satori_session_stage(const satori_session *s, int which, float *out, size_t n);
SATORI_API int satori_session_destroy(satori_session *s);  /* idempotent like DenseSession.Dispose */

/* ------------------------------------------------------------------ GGUF / STQ2 files */
typedef struct satori_gguf satori_gguf;
/* GgufFile(path) (src/Satori.Formats.Gguf/GgufFile.cs:18-176): maps the file read-only and validates
 * the GGUF v3 catalogue with the reference's rules; InvalidDataException -> SATORI_ERR_INVALID_DATA,
 * NotSupportedException -> SATORI_ERR_NOT_SUPPORTED.  Host code only (no GPU needed). */
SATORI_API int satori_gguf_open(const char *path, satori_gguf **out);
SATORI_API int satori_gguf_close(satori_gguf *g);
/* GgufFile.Tensors.Count / Metadata.Count. */
SATORI_API int satori_gguf_counts(const satori_gguf *g, int *tensors, int *metadata);
/* GgufTensor (GgufTensor.cs): name, GGUF type id, rank, dims (dims[0] = row length; unused dims 1),
 * absolute file offset and byte length of the payload. */
SATORI_API int satori_gguf_tensor_info(const satori_gguf *g, int index, char *name, size_t name_cap, int *type,
                                       int *rank, int64_t *dims, int64_t *offset, int64_t *bytes);
/* Index of a tensor by name, -1 when absent. */
SATORI_API int satori_gguf_find_tensor(const satori_gguf *g, const char *name, int *index);
/* GgufFile.ReadTensor (GgufFile.cs:42-49): the payload inside the mapping (valid until close). */
SATORI_API const void *satori_gguf_tensor_data(const satori_gguf *g, int index);
/* GgufMetadata (GgufMetadata.cs): key, value type, element type and count of entry `index` (arrays:
 * type 9; scalars: elem_type -1, count 1). */
SATORI_API int satori_gguf_metadata(const satori_gguf *g, int index, char *key, size_t key_cap, int *type,
                                    int *elem_type, int64_t *count);
/* GgufFile.ReadScalar (GgufFile.cs:56-76): the scalar's little-endian bytes (strings: their UTF-8 bytes,
 * no terminator) into out[cap]; *written = the value's byte length.  Arrays are refused. */
SATORI_API int satori_gguf_read_scalar(const satori_gguf *g, const char *key, int *type, void *out, size_t cap,
                                       size_t *written);
/* GgufModelLoader.Load + DenseTransformerAdapter.Validate (src/Satori.Core/Model/DenseTransformerAdapter.cs:
 * 12-121): the model description of a qwen2 / qwen3 file, with `tensors[capacity]` filled with the tensors a
 * session reads (host pointers into the mapping).  *needed = the entries required (call with capacity 0 to
 * size the table). */
SATORI_API int satori_gguf_model_desc(const satori_gguf *g, satori_model_desc *desc, satori_tensor *tensors,
                                      int capacity, int *needed);
/* DenseSession over a GGUF file: satori_gguf_model_desc then satori_session_create, every tensor uploaded
 * once from the mapping, unchanged in layout. */
SATORI_API int satori_session_create_from_gguf(satori_ctx *ctx, const satori_gguf *g, int context,
                                               satori_session **out);
/* MappedTernary2Matrix(path) (src/Satori.Core/MappedTernary2Matrix.cs:9-30) with Ternary2FileFormat.ReadHeader
 * (Ternary2FileFormat.cs:21-35): an STQ2 file mapped, its header, length and payload validated
 * (SATORI_ERR_INVALID_DATA on any defect), the payload uploaded once. */
SATORI_API int satori_stq2_open(satori_ctx *ctx, const char *path, satori_matrix **out);

#ifdef __cplusplus
}
#endif
#endif
