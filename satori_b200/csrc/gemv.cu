// gemv.cu -- sm_100a quantized MatVec for the Satori decode path.
//
// One kernel template covers GGUF Q8_0 / Q4_0 and Ternary2 (blocks of 64/128/256) in the three
// FP32 operation orders of the reference (satori_order):
//   EXECUTE  Ternary2Avx2Kernel.Execute (src/Satori.Core/Ternary2Avx2Kernel.cs:10-56) and
//            QuantizedAvx2Kernel.Execute (src/Satori.Core/QuantizedAvx2Kernel.cs:10-53);
//   SCALAR   Ternary2MatVec.ExecuteScalarCore (Ternary2MatVec.cs:52-76), QuantizedMatVec.ExecuteScalar
//            (QuantizedMatVec.cs:45-78);
//   BATCH    QuantizedMatVec.ExecuteBatchFloat -> ExecuteBatchRows -> Dot (QuantizedMatVec.cs:221-365),
//            the routine every decode projection runs.
// Each reference routine computes, per row, a left-to-right FP32 sum over blocks of one "term"
// per block (scale * lane-reduced partial, or the FMA dot).  The term of a block depends only
// on that block, so terms are computed in parallel by all compute warps, and a chain warp adds
// them in block order -- the result is bit-identical to the reference.
//
// Data movement: the CTA owns a contiguous range of rows.  The row range is streamed in column
// chunks; each chunk is one 1-D TMA bulk copy per row segment (cp.async.bulk, unicast) into a
// ring of shared-memory stages guarded by mbarriers.  The activation vector is staged once per
// CTA in shared memory, swizzled per block so lanes on consecutive blocks read distinct banks.
// Weights are read from HBM exactly once, in their original GGUF / STQ2 layout.
#include "common.cuh"
#include "gemv.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRowsPerCta = 64;
constexpr int kMaxPositions = 8;

__host__ __device__ constexpr int block_bytes_of(int fmt)
{
    return fmt == 0 ? 34 : fmt == 1 ? 18 : fmt == SATORI_Q4_K ? 144 : fmt == SATORI_Q6_K ? 210
         : fmt > 1000 ? 4 + (fmt - 1000) / 4 : 4 + fmt / 4;
}
__host__ __device__ constexpr int block_elems_of(int fmt)
{
    return fmt <= 1 ? 32 : (fmt == SATORI_Q4_K || fmt == SATORI_Q6_K) ? 256 : fmt > 1000 ? fmt - 1000 : fmt;
}

struct Geo {
    const uint8_t *payload;
    int rows, cols, bpr;
    long long row_bytes;
    const float *x;
    float *y;
    int P;
    int cb, nchunks, stages, seg_stride, dstride;
    int epilogue;
    const float *bias;
    float *residual;
    unsigned *err;
    int use_pdl;
};

// x swizzle: 16-byte chunk q of block b lives at chunk b*CPB + (q ^ (b & 7)).
template <int CPB>
__device__ __forceinline__ uint32_t xchunk(uint32_t xbase, int b, int q)
{
    return xbase + 16u * (uint32_t)(b * CPB + (q ^ (b & 7)));
}

// ---------------------------------------------------------------- Q8_0 / Q4_0 block term
// `qw` holds the block's quant bytes re-aligned into words, `d` its fp16 scale as float.
template <int FMT, int ORDER, int PMAX>
__device__ __forceinline__ void q_terms(const uint32_t qw[8], float d, uint32_t xbase, int b, int P,
                                        int xpos_stride, float (&terms)[PMAX])
{
    // Unscaled integer codes, exact in FP32: c[j] for weight j of the block.
    float c[32];
    if (FMT == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int m = 0; m < 4; ++m) c[4 * k + m] = u8_to_f_minus(((qw[k] >> (8 * m)) & 0xFFu) ^ 0x80u, 128.0f);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                uint32_t byte = (qw[k] >> (8 * m)) & 0xFFu;
                c[4 * k + m] = u8_to_f_minus(byte & 15u, 8.0f);
                c[4 * k + m + 16] = u8_to_f_minus(byte >> 4, 8.0f);
            }
    }
    if (ORDER == SATORI_ORDER_BATCH) {
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = fmul(d, c[j]);  // QuantizedRow.DecodeQ8Block/DecodeQ4Block
#pragma unroll
        for (int p = 0; p < PMAX; ++p) {
            if (p >= P) break;
            uint32_t xb = xbase + (uint32_t)(p * xpos_stride);
            float a[8];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                float4 x0 = lds128f(xchunk<8>(xb, b, 2 * g));
                float4 x1 = lds128f(xchunk<8>(xb, b, 2 * g + 1));
                float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int l = 0; l < 8; ++l) a[l] = g == 0 ? ffma(w[l], xv[l], 0.0f) : ffma(w[8 * g + l], xv[l], a[l]);
            }
            terms[p] = hsum8(a);
        }
    } else {
        // EXECUTE and SCALAR are single-position routines.
        float xv[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 t = lds128f(xchunk<8>(xbase, b, q));
            xv[4 * q] = t.x; xv[4 * q + 1] = t.y; xv[4 * q + 2] = t.z; xv[4 * q + 3] = t.w;
        }
        if (ORDER == SATORI_ORDER_EXECUTE) {
            float a[8];
            if (FMT == 0) {
#pragma unroll
                for (int l = 0; l < 8; ++l) a[l] = fadd(0.0f, fmul(c[l], xv[l]));
#pragma unroll
                for (int g = 1; g < 4; ++g)
#pragma unroll
                    for (int l = 0; l < 8; ++l) a[l] = fadd(a[l], fmul(c[8 * g + l], xv[8 * g + l]));
            } else {
                // j = 0: low nibbles 0..7 then high nibbles (weights 16..23); j = 8: 8..15 then 24..31.
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    a[l] = fadd(0.0f, fmul(c[l], xv[l]));
                    a[l] = fadd(a[l], fmul(c[16 + l], xv[16 + l]));
                    a[l] = fadd(a[l], fmul(c[8 + l], xv[8 + l]));
                    a[l] = fadd(a[l], fmul(c[24 + l], xv[24 + l]));
                }
            }
            terms[0] = fmul(d, hsum8(a));
        } else {
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) s = fadd(s, fmul(c[j], xv[j]));
            terms[0] = fmul(d, s);
        }
    }
}

// ---------------------------------------------------------------- decode-order fast path
// Dequantization in one FMA: PRMT places a code byte (biased int8, or a masked nibble) in bits 8..15
// under the 2^23 exponent, giving f = 2^23 + 256*u.  Then fma(f, d/256, -d*(2^15 + bias)) equals
// d*(u - bias) exactly: d has at most 11 significant bits, so d/256 and d*(2^15 + bias) are exact
// FP32 values, and the exact result d*(u - bias) is representable, so the single rounding is a no-op.
// This is the same value QuantizedRow.DecodeQ8Block/DecodeQ4Block computes as scale * code.
__device__ __forceinline__ float2 f2pair(uint32_t word, uint32_t sel_lo, uint32_t sel_hi)
{
    return make_float2(__uint_as_float(__byte_perm(word, 0x4B000000u, sel_lo)),
                       __uint_as_float(__byte_perm(word, 0x4B000000u, sel_hi)));
}

// Selector putting byte m of `word` at bits 8..15, 0x4B at bits 24..31, zeros elsewhere.
__host__ __device__ constexpr uint32_t byte_sel(int m) { return 0x7404u | ((uint32_t)m << 4); }

// Dot's eight FMA lanes for one 8-weight group (lanes l, l+1 as packed pairs), then
// QuantizedKAvx2Kernel.HorizontalSum as packed adds: ((a0+a4),(a1+a5)) + ((a2+a6),(a3+a7)), then g0 + g1.
template <int FMT, int PMAX>
__device__ __forceinline__ void q_terms_batch_fast(const uint32_t qw[8], float d, uint32_t xbase, int b, int P,
                                                   int xpos_stride, float (&terms)[PMAX])
{
    const float s8 = fmul(d, 0.00390625f);
    const float c8 = fmul(d, FMT == 0 ? -32896.0f : -32776.0f);  // -d*(2^15 + 128) / -d*(2^15 + 8)
    const float2 S = make_float2(s8, s8), Cc = make_float2(c8, c8);
    // Source word of each 4-weight quad q (weights 4q..4q+3).
    uint32_t src[8];
    if (FMT == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) src[k] = qw[k] ^ 0x80808080u;
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            src[k] = qw[k] & 0x0F0F0F0Fu;             // weights 4k..4k+3 (low nibbles)
            src[k + 4] = (qw[k] >> 4) & 0x0F0F0F0Fu;  // weights 16+4k.. (high nibbles)
        }
    }
    float2 w[16];  // w[2q + h]: weights (4q + 2h, 4q + 2h + 1), i.e. Dot lanes (l, l + 1)
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        w[2 * q] = __ffma2_rn(f2pair(src[q], byte_sel(0), byte_sel(1)), S, Cc);
        w[2 * q + 1] = __ffma2_rn(f2pair(src[q], byte_sel(2), byte_sel(3)), S, Cc);
    }
#pragma unroll
    for (int p = 0; p < PMAX; ++p) {
        if (p >= P) break;
        const uint32_t xb = xbase + (uint32_t)(p * xpos_stride);
        float2 A[4];  // lanes (0,1), (2,3), (4,5), (6,7)
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const float4 x0 = lds128f(xchunk<8>(xb, b, 2 * g));
            const float4 x1 = lds128f(xchunk<8>(xb, b, 2 * g + 1));
            const float2 X[4] = {make_float2(x0.x, x0.y), make_float2(x0.z, x0.w), make_float2(x1.x, x1.y),
                                 make_float2(x1.z, x1.w)};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                A[i] = __ffma2_rn(w[4 * g + i], X[i], g == 0 ? make_float2(0.0f, 0.0f) : A[i]);
        }
        const float2 h01 = __fadd2_rn(A[0], A[2]);  // (a0+a4, a1+a5)
        const float2 h23 = __fadd2_rn(A[1], A[3]);  // (a2+a6, a3+a7)
        const float2 g01 = __fadd2_rn(h01, h23);    // (h0+h2, h1+h3)
        terms[p] = fadd(g01.x, g01.y);
    }
}

// ---------------------------------------------------------------- Ternary2 block term
template <int BS, int ORDER>
__device__ __forceinline__ float t2_term(uint32_t blk, uint32_t xbase, int b, int count)
{
    constexpr int CPB = BS / 4;
    float scale = __uint_as_float(lds32(blk));
    float partial;
    int i = 0;
    if (ORDER == SATORI_ORDER_EXECUTE) {
        float a[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) a[l] = 0.0f;
        const int full = count & ~7;
        for (; i < full; i += 16) {
            uint32_t word = lds32(blk + 4 + (uint32_t)(i >> 2));  // two 8-code groups
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                int ii = i + 8 * half;
                if (ii < full) {
                    uint32_t packed = word >> (16 * half);
                    float4 x0 = lds128f(xchunk<CPB>(xbase, b, ii >> 2));
                    float4 x1 = lds128f(xchunk<CPB>(xbase, b, (ii >> 2) + 1));
                    float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int l = 0; l < 8; ++l) {
                        uint32_t code = (packed >> (2 * l)) & 3u;
                        // AndNot(zero, x ^ sign): +0 for code 0, -x for code 2, x otherwise.
                        float v = __uint_as_float((__float_as_uint(xv[l]) ^ (code == 2u ? 0x80000000u : 0u)) &
                                                  (code == 0u ? 0u : 0xFFFFFFFFu));
                        a[l] = fadd(a[l], v);
                    }
                }
            }
        }
        i = full;
        partial = hsum8(a);
    } else {
        partial = 0.0f;
    }
    // Scalar tail (EXECUTE) or the whole block (SCALAR): sequential +x / -x.
    for (; i < count; ++i) {
        uint32_t code = (lds32(blk + 4 + (uint32_t)((i >> 4) << 2)) >> (2 * (i & 15))) & 3u;
        if (code == 1u || code == 2u) {
            float4 xq = lds128f(xchunk<CPB>(xbase, b, i >> 2));
            float xv = (i & 3) == 0 ? xq.x : (i & 3) == 1 ? xq.y : (i & 3) == 2 ? xq.z : xq.w;
            partial = code == 1u ? fadd(partial, xv) : __fsub_rn(partial, xv);
        }
    }
    return fmul(partial, scale);
}

// ---------------------------------------------------------------- the kernel
template <int FMT, int ORDER, int PMAX>
__global__ void __launch_bounds__(kThreads) gemv_kernel(Geo g)
{
    constexpr int BB = block_bytes_of(FMT);
    constexpr int BE = block_elems_of(FMT);
    constexpr int CPB = BE / 4;                     // 16-byte x chunks per block
    extern __shared__ __align__(128) uint8_t smem[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const int r0 = (int)(((long long)g.rows * cta) / gridDim.x);
    const int r1 = (int)(((long long)g.rows * (cta + 1)) / gridDim.x);
    const int RC = r1 - r0;
    const int nchain = (RC + 31) >> 5;               // 1 or 2 chain warps (RC <= 64)
    const int ncompute_threads = (8 - nchain) * 32;
    const bool is_chain = warp >= 8 - nchain;
    const int S = g.stages;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem);                 // [S]
    const int xfloats = g.bpr * BE;                                          // per position, padded
    float *xs = reinterpret_cast<float *>(smem + 128);
    float *D = xs + (size_t)g.P * xfloats;                                   // [2][64][dstride]
    uint8_t *stage0 = reinterpret_cast<uint8_t *>(D + 2 * (size_t)kMaxRowsPerCta * g.dstride);
    stage0 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(stage0) + 127) & ~uintptr_t(127));
    const size_t stage_bytes = (size_t)RC * g.seg_stride;

    __shared__ int abort_flag;
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Producer: the last warp issues one bulk copy per row segment of a chunk.
    auto issue_chunk = [&](int c) {
        const int s = c % S;
        const int nb = min(g.cb, g.bpr - c * g.cb);
        uint32_t bytes = 0;
        const uint8_t *src[2] = {nullptr, nullptr};
        uint32_t sz[2] = {0u, 0u};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int r = lane + 32 * k;
            if (r < RC) {
                const uint8_t *p = g.payload + (long long)(r0 + r) * g.row_bytes + (long long)c * g.cb * BB;
                uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
                uintptr_t e = (reinterpret_cast<uintptr_t>(p) + (uintptr_t)nb * BB + 15) & ~uintptr_t(15);
                src[k] = reinterpret_cast<const uint8_t *>(a);
                sz[k] = (uint32_t)(e - a);
                bytes += sz[k];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xFFFFFFFFu, bytes, o);
        if (lane == 0) mbar_expect_tx(&full[s], bytes);
        __syncwarp();
        uint8_t *dst = stage0 + (size_t)s * stage_bytes;
#pragma unroll
        for (int k = 0; k < 2; ++k)
            if (sz[k]) bulk_g2s(dst + (size_t)(lane + 32 * k) * g.seg_stride, src[k], sz[k], &full[s]);
    };

    // Weights do not depend on the previous kernel: start streaming them before the PDL wait.
    if (warp == 7)
        for (int c = 0; c < min(S, g.nchunks); ++c) issue_chunk(c);

    if (g.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    // Stage the activation vector(s), swizzled.
    for (int p = 0; p < g.P; ++p) {
        const float *xsrc = g.x + (long long)p * g.cols;
        float *xdst = xs + (size_t)p * xfloats;
        for (int f = tid; f < xfloats; f += kThreads) {
            int chunk = f >> 2, b = chunk / CPB, q = chunk - b * CPB;
            int phys = (b * CPB + (q ^ (b & 7))) * 4 + (f & 3);
            xdst[phys] = f < g.cols ? xsrc[f] : 0.0f;
        }
    }
    __syncthreads();

    const uint32_t xbase = smem_u32(xs);
    const int xpos_stride = xfloats * 4;
    float acc[PMAX];
#pragma unroll
    for (int p = 0; p < PMAX; ++p) acc[p] = 0.0f;
    const int chain_row = (warp - (8 - nchain)) * 32 + lane;

    for (int c = 0; c <= g.nchunks; ++c) {
        const int buf = c & 1;
        if (!is_chain && c < g.nchunks) {
            const int s = c % S;
            const int nb = min(g.cb, g.bpr - c * g.cb);
            if (!abort_flag && !mbar_wait_bounded(&full[s], (uint32_t)((c / S) & 1))) {
                atomicOr(g.err, kDevErrTimeout);
                abort_flag = 1;
            }
            if (!abort_flag) {
                const uint32_t sbase = smem_u32(stage0 + (size_t)s * stage_bytes);
                const int items = RC * nb;
                // (row, block) of this thread's first item; later items advance by a fixed (dr, dj).
                int r = tid / nb, j = tid - (tid / nb) * nb;
                const int dr = ncompute_threads / nb, dj = ncompute_threads - dr * nb;
                const uint32_t chunk_ofs = (uint32_t)(c * g.cb * BB);
                for (int it = tid; it < items; it += ncompute_threads) {
                    const int b = c * g.cb + j;
                    // Low 4 bits of the segment's global offset = its offset inside the 16-byte-aligned copy.
                    const uint32_t seg_ofs = ((uint32_t)(r0 + r) * (uint32_t)g.row_bytes + chunk_ofs) & 15u;
                    const uint32_t blk = sbase + (uint32_t)(r * g.seg_stride) + seg_ofs + (uint32_t)(j * BB);
                    float *dst = D + ((size_t)buf * kMaxRowsPerCta + r) * g.dstride + (size_t)j * g.P;
                    if (FMT <= 1) {
                        // Bytes [0, BB) of a 2-byte aligned block span words 0..NW from the aligned base.
                        const uint32_t base = blk & ~3u, sh = (blk & 3u) * 8u;
                        constexpr int NW = FMT == 0 ? 8 : 4;
                        uint32_t w[NW + 1];
#pragma unroll
                        for (int k = 0; k <= NW; ++k) w[k] = lds32(base + 4u * k);
                        uint32_t qw[8];
                        const uint32_t shq = sh + 16u;  // quants start 2 bytes after the scale
#pragma unroll
                        for (int k = 0; k < (FMT == 0 ? 8 : 4); ++k) qw[k] = __funnelshift_rc(w[k], w[k + 1], shq);
                        const float d = half_bits_to_float(__funnelshift_rc(w[0], w[1], sh));
                        float terms[PMAX];
                        if (ORDER == SATORI_ORDER_BATCH)
                            q_terms_batch_fast<FMT, PMAX>(qw, d, xbase, b, g.P, xpos_stride, terms);
                        else
                            q_terms<FMT, ORDER, PMAX>(qw, d, xbase, b, g.P, xpos_stride, terms);
#pragma unroll
                        for (int p = 0; p < PMAX; ++p)
                            if (p < g.P) dst[p] = terms[p];
                    } else {
                        const int count = min(BE, g.cols - b * BE);
                        dst[0] = t2_term<BE, ORDER>(blk, xbase, b, count);
                    }
                    j += dj;
                    r += dr;
                    if (j >= nb) {
                        j -= nb;
                        ++r;
                    }
                }
            }
        }
        if (is_chain && c >= 1 && chain_row < RC) {
            const int cprev = c - 1;
            const int nb = min(g.cb, g.bpr - cprev * g.cb);
            const float *src = D + ((size_t)(cprev & 1) * kMaxRowsPerCta + chain_row) * g.dstride;
            for (int j = 0; j < nb; ++j)
#pragma unroll
                for (int p = 0; p < PMAX; ++p)
                    if (p < g.P) acc[p] = fadd(acc[p], src[j * g.P + p]);
        }
        __syncthreads();
        if (warp == 7 && c < g.nchunks && c + S < g.nchunks) issue_chunk(c + S);
    }


    if (is_chain && chain_row < RC && !abort_flag) {
        const int row = r0 + chain_row;
#pragma unroll
        for (int p = 0; p < PMAX; ++p) {
            if (p >= g.P) break;
            float v = acc[p];
            if (g.epilogue == kEpiBias) v = fadd(v, g.bias[row]);
            if (g.epilogue == kEpiResidual) {
                v = fadd(g.residual[row], v);
                g.residual[row] = v;
            }
            g.y[(long long)p * g.rows + row] = v;
        }
    }
}

template <int FMT, int ORDER, int PMAX = 1>
cudaError_t launch_one(const Geo &g, const GemvPlan &plan, cudaStream_t stream)
{
    auto kern = gemv_kernel<FMT, ORDER, PMAX>;
    // Opt in to exactly the dynamic shared memory this plan needs (the limit counts static smem too).
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(kern), plan.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, g);
}

}  // namespace

int gemv_block_bytes(int format) { return block_bytes_of(format); }
int gemv_block_elems(int format) { return block_elems_of(format); }

GemvPlan plan_gemv(int rows, int cols, int format, int positions, int sm_count, size_t smem_limit)
{
    GemvPlan p = {};
    const int BB = block_bytes_of(format), BE = block_elems_of(format);
    const int bpr = (cols + BE - 1) / BE;
    if (positions < 1 || positions > kMaxPositions) return p;
    int grid = std::min(rows, 2 * sm_count);
    int rc = (rows + grid - 1) / grid;
    if (rc > kMaxRowsPerCta) rc = kMaxRowsPerCta;
    grid = (rows + rc - 1) / rc;
    // Chunk: a whole number of rounds of the compute threads (rows x blocks <= k * threads) carrying
    // at least ~12 KB of payload per stage, so every compute thread has the same number of items.
    const int tc = (8 - (rc + 31) / 32) * 32;
    int cb = 1;
    for (int k = 1; k <= 16; ++k) {
        const int c = std::max(1, (k * tc) / rc);
        cb = std::min(c, bpr);
        if (c >= bpr || (size_t)c * rc * BB >= 12288) break;
    }
    cb = std::max(1, std::min(cb, 64));
    const int seg_stride = ((cb * BB + 32) + 15) & ~15;
    const int dstride = cb * positions + 1;
    const size_t xbytes = (size_t)positions * bpr * BE * 4;
    const size_t dbytes = 2ull * kMaxRowsPerCta * dstride * 4;
    int stages = 4;
    size_t smem = 0;
    for (; stages >= 2; --stages) {
        smem = 128 + xbytes + dbytes + 128 + (size_t)stages * rc * seg_stride;
        if (smem <= smem_limit) break;
    }
    if (stages < 2) return p;
    p.grid = grid;
    p.threads = kThreads;
    p.rows_per_cta = rc;
    p.chunk_blocks = cb;
    p.nchunks = (bpr + cb - 1) / cb;
    p.stages = stages;
    p.seg_stride = seg_stride;
    p.dstride = dstride;
    p.smem = smem;
    p.ok = 1;
    return p;
}

cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &plan, cudaStream_t stream)
{
    Geo g;
    const int BB = block_bytes_of(a.format), BE = block_elems_of(a.format);
    g.payload = a.payload;
    g.rows = a.rows;
    g.cols = a.cols;
    g.bpr = (a.cols + BE - 1) / BE;
    g.row_bytes = (long long)g.bpr * BB;
    g.x = a.x;
    g.y = a.y;
    g.P = a.order == SATORI_ORDER_BATCH ? a.positions : 1;
    g.cb = plan.chunk_blocks;
    g.nchunks = plan.nchunks;
    g.stages = plan.stages;
    g.seg_stride = plan.seg_stride;
    g.dstride = plan.dstride;
    g.epilogue = a.epilogue;
    g.bias = a.bias;
    g.residual = a.residual;
    g.err = a.err;
    g.use_pdl = a.use_pdl;
#define SATORI_GEMV_CASE(F)                                                                               \
    case F:                                                                                               \
        if (a.order == SATORI_ORDER_EXECUTE) return launch_one<F, SATORI_ORDER_EXECUTE>(g, plan, stream); \
        if (a.order == SATORI_ORDER_SCALAR) return launch_one<F, SATORI_ORDER_SCALAR>(g, plan, stream);   \
        break;
    switch (a.format) {
    case 0:
        if (a.order == SATORI_ORDER_BATCH && g.P == 1) return launch_one<0, SATORI_ORDER_BATCH, 1>(g, plan, stream);
        if (a.order == SATORI_ORDER_BATCH) return launch_one<0, SATORI_ORDER_BATCH, kMaxPositions>(g, plan, stream);
        if (a.order == SATORI_ORDER_EXECUTE) return launch_one<0, SATORI_ORDER_EXECUTE>(g, plan, stream);
        if (a.order == SATORI_ORDER_SCALAR) return launch_one<0, SATORI_ORDER_SCALAR>(g, plan, stream);
        break;
    case 1:
        if (a.order == SATORI_ORDER_BATCH && g.P == 1) return launch_one<1, SATORI_ORDER_BATCH, 1>(g, plan, stream);
        if (a.order == SATORI_ORDER_BATCH) return launch_one<1, SATORI_ORDER_BATCH, kMaxPositions>(g, plan, stream);
        if (a.order == SATORI_ORDER_EXECUTE) return launch_one<1, SATORI_ORDER_EXECUTE>(g, plan, stream);
        if (a.order == SATORI_ORDER_SCALAR) return launch_one<1, SATORI_ORDER_SCALAR>(g, plan, stream);
        break;
    SATORI_GEMV_CASE(64)
    SATORI_GEMV_CASE(128)
    SATORI_GEMV_CASE(256)
    default:
        break;
    }
#undef SATORI_GEMV_CASE
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- row decode, validation, quantizers
namespace {

__global__ void decode_row_kernel(const uint8_t *payload, int cols, int format, const int *row_dev, int row_host,
                                  float *out)
{
    const int row = row_dev ? *row_dev : row_host;
    const int BB = block_bytes_of(format), BE = block_elems_of(format);
    const int bpr = (cols + BE - 1) / BE;
    const uint8_t *rp = payload + (long long)row * bpr * BB;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
        const int b = i / BE, j = i - b * BE;
        const uint8_t *blk = rp + (long long)b * BB;
        float v;
        if (format <= 1) {
            const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            float code;
            if (format == 0) code = u8_to_f_minus((uint32_t)blk[2 + j] ^ 0x80u, 128.0f);
            else code = j < 16 ? u8_to_f_minus(blk[2 + j] & 15u, 8.0f) : u8_to_f_minus(blk[2 + j - 16] >> 4, 8.0f);
            v = fmul(d, code);  // QuantizedRow.DecodeQ8Block / DecodeQ4Block
        } else {
            float scale;
            memcpy(&scale, blk, 4);
            const uint32_t code = (blk[4 + j / 4] >> (2 * (j % 4))) & 3u;
            v = code == 1u ? scale : code == 2u ? -scale : 0.0f;  // Ternary2Matrix.Dequantize
        }
        out[i] = v;
    }
}

__global__ void validate_kernel(const uint8_t *payload, int rows, int cols, int format, int *status)
{
    const int BB = block_bytes_of(format), BE = block_elems_of(format);
    const int bpr = (cols + BE - 1) / BE;
    const long long nblocks = (long long)rows * bpr;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nblocks;
         k += (long long)gridDim.x * blockDim.x) {
        const uint8_t *blk = payload + k * BB;
        if (format <= 1) {
            // QuantizedMatVec.ValidatePayload (QuantizedMatVec.cs:28-42): the fp16 scale must be finite.
            const uint32_t h = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8);
            if ((h & 0x7C00u) == 0x7C00u) atomicMax(status, (int)SATORI_ERR_INVALID_DATA);
        } else {
            // Ternary2Matrix.ValidatePayload (Ternary2Matrix.cs:83-101).
            uint32_t sb = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) | ((uint32_t)blk[3] << 24);
            const int b = (int)(k % bpr);
            const int count = min(format, cols - b * format);
            const bool finite = (sb & 0x7F800000u) != 0x7F800000u;
            const float scale = __uint_as_float(sb);
            bool bad = !finite || scale < 0.0f || sb == 0x80000000u;
            for (int i = 0; i < format && !bad; ++i) {
                const uint32_t code = (blk[4 + i / 4] >> (2 * (i % 4))) & 3u;
                if (code == 3u || ((i >= count || scale == 0.0f) && code != 0u)) bad = true;
            }
            if (bad) atomicMax(status, (int)SATORI_ERR_INVALID_DATA);
        }
    }
}

// Ternary2Matrix.Quantize (Ternary2Matrix.cs:38-71): one thread per block, FP64 magnitude sum in
// column order, FP32 scale, FP64 threshold -- the same IEEE operations, so the bytes are identical.
__global__ void t2_quantize_kernel(const float *w, int rows, int cols, int bs, uint8_t *out, int *status)
{
    const int bpr = (cols + bs - 1) / bs;
    const int bb = 4 + bs / 4;
    const long long nblocks = (long long)rows * bpr;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nblocks;
         k += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(k / bpr), block = (int)(k % bpr);
        const int column = block * bs;
        const int count = min(bs, cols - column);
        const float *src = w + (long long)row * cols + column;
        uint8_t *t = out + k * bb;
        double magnitude = 0;
        bool finite = true;
        for (int i = 0; i < count; ++i) {
            const float v = src[i];
            finite &= isfinite(v);
            magnitude = __dadd_rn(magnitude, fabs((double)v));
        }
        if (!finite) atomicMax(status, (int)SATORI_ERR_ARGUMENT);
        const float scale = __double2float_rn(__ddiv_rn(magnitude, (double)count));
        const uint32_t sb = __float_as_uint(scale);
        t[0] = sb & 0xFF; t[1] = (sb >> 8) & 0xFF; t[2] = (sb >> 16) & 0xFF; t[3] = sb >> 24;
        for (int i = 0; i < bs / 4; ++i) t[4 + i] = 0;
        if (scale == 0.0f) continue;
        const double threshold = (double)scale / 2;
        for (int i = 0; i < count; ++i) {
            const double v = (double)src[i];
            const int code = v > threshold ? 1 : v < -threshold ? 2 : 0;
            t[4 + i / 4] |= (uint8_t)(code << (2 * (i % 4)));
        }
    }
}

__device__ uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// This library's own Q8_0/Q4_0 quantizer (the reference has none): see satori_cuda.h.
__global__ void q_quantize_kernel(const float *w, int rows, int cols, int format, uint8_t *out)
{
    const int bpr = cols / 32;
    const int bb = format == 0 ? 34 : 18;
    const long long nblocks = (long long)rows * bpr;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nblocks;
         k += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(k / bpr), blk = (int)(k % bpr);
        const float *src = w + (long long)row * cols + blk * 32;
        uint8_t *b = out + k * bb;
        if (format == 0) {
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(src[j]));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const uint16_t h = f32_to_f16_bits(d);
            b[0] = h & 0xFF; b[1] = h >> 8;
            for (int j = 0; j < 32; ++j) {
                float v = roundf(__fmul_rn(src[j], id));
                v = fminf(127.0f, fmaxf(-127.0f, v));
                b[2 + j] = (uint8_t)(int8_t)v;
            }
        } else {
            float amax = 0.0f, m = 0.0f;
            for (int j = 0; j < 32; ++j) {
                const float a = fabsf(src[j]);
                if (a > amax) { amax = a; m = src[j]; }
            }
            const float d = __fdiv_rn(m, -8.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const uint16_t h = f32_to_f16_bits(d);
            b[0] = h & 0xFF; b[1] = h >> 8;
            for (int j = 0; j < 16; ++j) {
                int lo = (int)floorf(__fadd_rn(__fmul_rn(src[j], id), 8.5f));
                int hi = (int)floorf(__fadd_rn(__fmul_rn(src[j + 16], id), 8.5f));
                lo = lo < 0 ? 0 : lo > 15 ? 15 : lo;
                hi = hi < 0 ? 0 : hi > 15 ? 15 : hi;
                b[2 + j] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

}  // namespace

cudaError_t launch_decode_row(const uint8_t *payload, int rows, int cols, int format, const int *row_dev,
                              int row_host, float *out, cudaStream_t stream)
{
    (void)rows;
    if (is_kquant(format)) return launch_kq_decode_row(payload, cols, format, row_dev, row_host, out, stream);
    if (is_bitplane(format)) return launch_bitplane_decode_row(payload, cols, format, row_dev, row_host, out, stream);
    const int threads = 256;
    const int blocks = std::min(64, (cols + threads - 1) / threads);
    decode_row_kernel<<<blocks, threads, 0, stream>>>(payload, cols, format, row_dev, row_host, out);
    return cudaGetLastError();
}

cudaError_t launch_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                            cudaStream_t stream)
{
    if (is_kquant(format)) return launch_kq_validate(payload, rows, cols, format, status_dev, stream);
    if (is_bitplane(format)) return launch_bitplane_validate(payload, rows, cols, format, status_dev, stream);
    validate_kernel<<<592, 256, 0, stream>>>(payload, rows, cols, format, status_dev);
    return cudaGetLastError();
}

cudaError_t launch_t2_quantize(const float *w, int rows, int cols, int bs, uint8_t *out, int *status_dev,
                               cudaStream_t stream)
{
    t2_quantize_kernel<<<592, 128, 0, stream>>>(w, rows, cols, bs, out, status_dev);
    return cudaGetLastError();
}

cudaError_t launch_q_quantize(const float *w, int rows, int cols, int format, uint8_t *out, cudaStream_t stream)
{
    q_quantize_kernel<<<1184, 128, 0, stream>>>(w, rows, cols, format, out);
    return cudaGetLastError();
}

}  // namespace satori
