// ops.cu -- decode-step glue kernels.  FP64 where the reference computes in FP64, with every
// multiply and add rounded separately (no contraction), as the reference does.
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

__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float *x, const float *w, int n, float eps, float *out,
                                                       int pdl)
{
    __shared__ double red[1024];
    if (pdl) pdl_wait();
    double sum = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) sum = __dadd_rn(sum, __dmul_rn((double)x[i], (double)x[i]));
    sum = block_sum_double(sum, red);
    const double scale = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)n), (double)eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = (float)__dmul_rn(__dmul_rn((double)x[i], scale), (double)w[i]);
    if (pdl) pdl_launch_dependents();
}

__global__ void rmsnorm_heads_kernel(float *v, int n, const float *w, float eps, int hd, int pdl)
{
    __shared__ double red[128];
    if (pdl) pdl_wait();
    float *h = v + (long long)blockIdx.x * hd;
    double sum = 0;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sum = __dadd_rn(sum, __dmul_rn((double)h[i], (double)h[i]));
    sum = block_sum_double(sum, red);
    const double scale = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)hd), (double)eps)));
    for (int i = threadIdx.x; i < hd; i += blockDim.x)
        h[i] = (float)__dmul_rn(__dmul_rn((double)h[i], scale), (double)w[i]);
    if (pdl) pdl_launch_dependents();
}

__global__ void swiglu_kernel(const float *gate, const float *up, int n, float *out, int pdl)
{
    if (pdl) pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const double x = gate[i];
        double sig;
        if (x >= 0) {
            sig = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
        } else {
            const double e = exp(x);
            sig = __ddiv_rn(e, __dadd_rn(1.0, e));
        }
        out[i] = (float)__dmul_rn(__dmul_rn(x, sig), (double)up[i]);
    }
    if (pdl) pdl_launch_dependents();
}

__global__ void embed_kernel(const uint8_t *embd, int cols, const int *token_dev, const int *pos_dev, int *tokens_dev,
                             float *hidden, int pdl)
{
    if (pdl) pdl_wait();
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
    if (pdl) pdl_launch_dependents();
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx)
{
    uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 ties with +0, as the reference's '>' does
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);       // order-preserving map of finite floats
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float *logits, int n, int *argmax, int *nonfinite, int *pos,
                                                      int *token, int pdl)
{
    __shared__ unsigned long long red[1024];
    __shared__ int bad;
    if (pdl) pdl_wait();
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    unsigned long long best = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (!isfinite(v)) bad = 1;
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
    }
    red[threadIdx.x] = best;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s && red[threadIdx.x + s] > red[threadIdx.x]) red[threadIdx.x] = red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int idx = (int)(0xFFFFFFFFu - (uint32_t)(red[0] & 0xFFFFFFFFull));
        *argmax = idx;
        *token = idx;
        if (bad) *nonfinite = 1;
        *pos = *pos + 1;
    }
    if (pdl) pdl_launch_dependents();
}

}  // namespace

cudaError_t launch_rmsnorm(const float *x, const float *w, int n, float eps, float *out, cudaStream_t s, int pdl)
{
    return launch_ex(rmsnorm_kernel, dim3(1), dim3(1024), 0, s, pdl, x, w, n, eps, out, pdl);
}

cudaError_t launch_rmsnorm_heads(float *v, int n, const float *w, float eps, int head_dim, cudaStream_t s, int pdl)
{
    return launch_ex(rmsnorm_heads_kernel, dim3(n / head_dim), dim3(128), 0, s, pdl, v, n, w, eps, head_dim, pdl);
}

cudaError_t launch_swiglu(const float *gate, const float *up, int n, float *out, cudaStream_t s, int pdl)
{
    const int blocks = (n + 255) / 256;
    return launch_ex(swiglu_kernel, dim3(blocks), dim3(256), 0, s, pdl, gate, up, n, out, pdl);
}

cudaError_t launch_embed(const uint8_t *embd, int cols, const int *token_dev, const int *pos_dev, int *tokens_dev,
                         float *hidden, cudaStream_t s, int pdl)
{
    const int blocks = (cols + 255) / 256;
    return launch_ex(embed_kernel, dim3(blocks), dim3(256), 0, s, pdl, embd, cols, token_dev, pos_dev, tokens_dev,
                     hidden, pdl);
}

cudaError_t launch_argmax_advance(const float *logits, int n, int *argmax_dev, int *nonfinite_dev, int *pos_dev,
                                  int *token_dev, cudaStream_t s, int pdl)
{
    return launch_ex(argmax_kernel, dim3(1), dim3(1024), 0, s, pdl, logits, n, argmax_dev, nonfinite_dev, pos_dev,
                     token_dev, pdl);
}

}  // namespace satori
