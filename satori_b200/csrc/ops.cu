// ops.cu -- decode-step glue kernels.  FP64 where the reference computes in FP64, with every
// multiply and add rounded separately (no contraction), as the reference does.
#include <algorithm>

#include "common.cuh"
#include "ops.cuh"

namespace satori {

namespace {

template <typename K, typename... Args>
cudaError_t launch_ex(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, int pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

__device__ double block_sum_double(double v, double *red)
{
    red[threadIdx.x] = v;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = __dadd_rn(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    const double r = red[0];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *w, int n, float eps, float *out,
                                                      int pdl)
{
    __shared__ double red[8];
    if (pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    x += (long long)blockIdx.x * n;     // one vector per CTA (a prefill chunk has several)
    out += (long long)blockIdx.x * n;
    rms_partial(x, n, threadIdx.x, red);
    __syncthreads();
    const double scale = rms_scale(red, n, eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = rms_apply(x[i], scale, w[i]);
}

__global__ void rmsnorm_heads_kernel(float *v, int n, const float *w, float eps, int hd, long long stride, int pdl)
{
    __shared__ double red[128];
    if (pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    float *h = v + (long long)blockIdx.y * stride + (long long)blockIdx.x * hd;
    double sum = 0;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sum = __dadd_rn(sum, __dmul_rn((double)h[i], (double)h[i]));
    sum = block_sum_double(sum, red);
    const double scale = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)hd), (double)eps)));
    for (int i = threadIdx.x; i < hd; i += blockDim.x)
        h[i] = (float)__dmul_rn(__dmul_rn((double)h[i], scale), (double)w[i]);
}

__global__ void swiglu_kernel(const float *gate, const float *up, int n, float *out, int pdl)
{
    if (pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = swiglu_value(gate[i], up[i]);
}

__global__ void embed_kernel(const uint8_t *embd, int cols, const int *token_dev, const int *pos_dev, int *tokens_dev,
                             float *hidden, double *rope_table, double rope_base, int rotary, int pdl)
{
    if (pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    if (rope_table) {
        // TransformerOps.RopeHalf (TransformerOps.cs:99-118): the FP64 angle of pair k and its sin/cos,
        // the same for every head and layer of this step.
        const int k = blockIdx.x * blockDim.x + threadIdx.x;
        if (k < rotary / 2) {
            const double angle = __ddiv_rn((double)*pos_dev, pow(rope_base, __ddiv_rn(2.0 * k, (double)rotary)));
            double sn, cs;
            sincos(angle, &sn, &cs);
            rope_table[2 * k] = cs;
            rope_table[2 * k + 1] = sn;
        }
    }
    const int token = *token_dev;
    const int bpr = cols / 32;
    const uint8_t *row = embd + (long long)token * bpr * 34;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
        const uint8_t *blk = row + (i / 32) * 34;
        const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        const float code = u8_to_f_minus((uint32_t)blk[2 + (i & 31)] ^ 0x80u, 128.0f);
        hidden[i] = fmul(d, code);  // QuantizedRow.DecodeQ8Block
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *tokens_dev = *pos_dev + 1;
}

// A prefill chunk's embedding rows (token of position z from tokens[z]) and RoPE factors of positions
// pos0 + z, z = blockIdx.y: the per-position work of embed_kernel.
__global__ void embed_batch_kernel(const uint8_t *embd, int cols, const int *tokens, int pos0, float *hidden,
                                   double *rope_table, double rope_base, int rotary)
{
    const int z = blockIdx.y;
    if (rope_table) {
        const int k = blockIdx.x * blockDim.x + threadIdx.x;
        if (k < rotary / 2) {
            const double angle = __ddiv_rn((double)(pos0 + z), pow(rope_base, __ddiv_rn(2.0 * k, (double)rotary)));
            double sn, cs;
            sincos(angle, &sn, &cs);
            rope_table[(long long)z * rotary + 2 * k] = cs;
            rope_table[(long long)z * rotary + 2 * k + 1] = sn;
        }
    }
    const int bpr = cols / 32;
    const uint8_t *row = embd + (long long)tokens[z] * bpr * 34;
    float *out = hidden + (long long)z * cols;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
        const uint8_t *blk = row + (i / 32) * 34;
        const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        const float code = u8_to_f_minus((uint32_t)blk[2 + (i & 31)] ^ 0x80u, 128.0f);
        out[i] = fmul(d, code);
    }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx)
{
    uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 ties with +0, as the reference's '>' does
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);       // order-preserving map of finite floats
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

constexpr int kArgmaxThreads = 256;

// Grid-wide: every CTA folds its share into one 64-bit key with atomicMax (the key orders by value,
// then by the smaller index, so the result does not depend on the CTA order); the last CTA to finish
// publishes the index and clears the scratch for the next launch.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float *logits, int n, int *argmax,
                                                                int *nonfinite, int *pos, int *token,
                                                                unsigned *scratch, int pdl)
{
    __shared__ unsigned long long red[kArgmaxThreads / 32];
    unsigned long long *best_dev = reinterpret_cast<unsigned long long *>(scratch);
    unsigned *ticket = scratch + 2;
    if (pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    unsigned long long best = 0;
    bool bad = false;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        bad |= !isfinite(v);
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
    }
    if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) *nonfinite = 1;
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_down_sync(0xFFFFFFFFu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < kArgmaxThreads / 32; ++w) best = red[w] > best ? red[w] : best;
    atomicMax(best_dev, best);
    __threadfence();
    if (atomicAdd(ticket, 1u) != gridDim.x - 1) return;
    __threadfence();
    const unsigned long long k = atomicExch(best_dev, 0ull);
    *ticket = 0;
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    *argmax = idx;
    *token = idx;
    *pos = *pos + 1;
}

}  // namespace

cudaError_t launch_rmsnorm(const float *x, const float *w, int n, float eps, float *out, cudaStream_t s, int pdl)
{
    return launch_ex(rmsnorm_kernel, dim3(1), dim3(256), 0, s, pdl, x, w, n, eps, out, pdl);
}

cudaError_t launch_rmsnorm_heads(float *v, int n, const float *w, float eps, int head_dim, cudaStream_t s, int pdl)
{
    return launch_ex(rmsnorm_heads_kernel, dim3(n / head_dim), dim3(128), 0, s, pdl, v, n, w, eps, head_dim, 0ll,
                     pdl);
}

cudaError_t launch_rmsnorm_batch(const float *x, const float *w, int n, float eps, float *out, int positions,
                                 cudaStream_t s)
{
    return launch_ex(rmsnorm_kernel, dim3(positions), dim3(256), 0, s, 0, x, w, n, eps, out, 0);
}

cudaError_t launch_rmsnorm_heads_batch(float *v, int n, const float *w, float eps, int head_dim, long long stride,
                                       int positions, cudaStream_t s)
{
    return launch_ex(rmsnorm_heads_kernel, dim3(n / head_dim, positions), dim3(128), 0, s, 0, v, n, w, eps, head_dim,
                     stride, 0);
}

cudaError_t launch_embed_batch(const uint8_t *embd, int cols, const int *tokens_dev, int positions, int pos0,
                               float *hidden, double *rope_table, double rope_base, int rotary, cudaStream_t s)
{
    const int blocks = (std::max(cols, rotary / 2) + 255) / 256;
    return launch_ex(embed_batch_kernel, dim3(blocks, positions), dim3(256), 0, s, 0, embd, cols, tokens_dev, pos0,
                     hidden, rope_table, rope_base, rotary);
}

cudaError_t launch_swiglu(const float *gate, const float *up, int n, float *out, cudaStream_t s, int pdl)
{
    const int blocks = (n + 255) / 256;
    return launch_ex(swiglu_kernel, dim3(blocks), dim3(256), 0, s, pdl, gate, up, n, out, pdl);
}

cudaError_t launch_embed(const uint8_t *embd, int cols, const int *token_dev, const int *pos_dev, int *tokens_dev,
                         float *hidden, double *rope_table, double rope_base, int rotary, cudaStream_t s, int pdl)
{
    const int blocks = (std::max(cols, rotary / 2) + 255) / 256;
    return launch_ex(embed_kernel, dim3(blocks), dim3(256), 0, s, pdl, embd, cols, token_dev, pos_dev, tokens_dev,
                     hidden, rope_table, rope_base, rotary, pdl);
}

cudaError_t launch_argmax_advance(const float *logits, int n, int *argmax_dev, int *nonfinite_dev, int *pos_dev,
                                  int *token_dev, unsigned *scratch, int sm_count, cudaStream_t s, int pdl)
{
    const int blocks = std::max(1, std::min(sm_count, (n + 4 * kArgmaxThreads - 1) / (4 * kArgmaxThreads)));
    return launch_ex(argmax_kernel, dim3(blocks), dim3(kArgmaxThreads), 0, s, pdl, logits, n, argmax_dev,
                     nonfinite_dev, pos_dev, token_dev, scratch, pdl);
}

}  // namespace satori
