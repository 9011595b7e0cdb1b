// gemv_kquant.cu -- GGUF K-quant matrices (Q4_K, Q6_K): validation, row decode and MatVec in each of the
// reference's three orders, bit-identical to it.
//
// * batch order (QuantizedMatVec.ExecuteBatch with AVX2 -> ExecuteBatchQuantized ->
//   QuantizedKAvx2Kernel.ExecuteQuantizedTiled, QuantizedMatVec.cs:122-220, QuantizedKAvx2Kernel.cs:46-95):
//   the activation is quantized to Q8_K (Q8KCodec.QuantizeBlock, Q8KCodec.cs:43-75); every (row, block)
//   product is an exact integer (dp4a on the GPU, any order), then combined in FP32 in the reference's
//   order -- (d*as)*isum - (dmin*as)*mins for Q4_K, (as*d)*isum for Q6_K -- and added to the row's sum
//   block by block; all-zero activation blocks are skipped.  This is what decode runs.
// * scalar order (QuantizedMatVec.ExecuteScalar with Q4KCodec.DotBlock / Q6KCodec.DotBlock) and
//   execute order (QuantizedKAvx2Kernel.ExecuteQ4K / ExecuteQ6K, eight FP32 lanes per step and the fixed
//   horizontal sum): one thread per row, every operation in the reference's sequence.
// * row decode (Q4KCodec.DecodeBlock / Q6KCodec.DecodeBlock) and the finite-scale validation
//   (Q4KCodec.AreScalesFinite / Q6KCodec.AreScalesFinite).
#include "common.cuh"
#include "gemv.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kKRecord = 304;     // per activation block in shared memory: codes[256] | sums[16] | scale | pad
constexpr int kKWarps = 8;        // one row per warp in the batch kernel

__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t *p)
{
    // A 4-byte read at any 2-byte-aligned address (Q6_K blocks sit at 210-byte steps).
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    if ((a & 3) == 0) return w[0];
    return __funnelshift_r(w[0], w[1], 8 * (uint32_t)(a & 3));
}

__device__ __forceinline__ float h2f(const uint8_t *p) { return half_bits_to_float((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

// Q4KCodec.GetScaleMin (Q4KCodec.cs:24-37).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *sc, int &s, int &m)
{
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// The centred 6-bit code of Q6_K weight (half, l, k) (Q6KCodec.cs:38-46).
__device__ __forceinline__ int q6k_code(const uint8_t *b, int half, int l, int k)
{
    const uint8_t *lql = b + half * 64, *lqh = b + 128 + half * 32;
    const int nib = k == 0 ? (lql[l] & 0xF) : k == 1 ? (lql[l + 32] & 0xF) : k == 2 ? (lql[l] >> 4) : (lql[l + 32] >> 4);
    return (nib | (((lqh[l] >> (2 * k)) & 3) << 4)) - 32;
}

__device__ __forceinline__ int dp4a_us(uint32_t a_u8, uint32_t b_s8, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8), "r"(b_s8), "r"(c));
    return d;
}

// ---------------------------------------------------------------------------------------- Q8_K
// Q8KCodec.QuantizeBlock for the 256 values x[0..255] by one warp (8 values per lane): the magnitude
// maximum with the first index among equals, inverse = -127 / max, codes = min(127, nearest(inverse * x))
// with the 1.5 * 2^23 rounding of NearestInteger, group sums of 16, scale = 1 / inverse.
__device__ void q8k_quantize_warp(const float *x, uint8_t *rec, int lane)
{
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[lane * 8 + i];
    float mag = 0.0f, mx = 0.0f;
    int idx = 1 << 30;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > mag) {
            mag = a;
            mx = v[i];
            idx = lane * 8 + i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float om = __shfl_xor_sync(0xFFFFFFFFu, mag, o);
        const float ox = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
        if (om > mag || (om == mag && oi < idx)) {
            mag = om;
            mx = ox;
            idx = oi;
        }
    }
    int8_t *codes = reinterpret_cast<int8_t *>(rec);
    int16_t *sums = reinterpret_cast<int16_t *>(rec + 256);
    float *scale = reinterpret_cast<float *>(rec + 288);
    if (mag == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) codes[lane * 8 + i] = 0;
        if (lane < 16) sums[lane] = 0;
        if (lane == 0) *scale = 0.0f;
        return;
    }
    const float inverse = __fdiv_rn(-127.0f, mx);
    int part = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float shifted = fadd(fmul(inverse, v[i]), 12582912.0f);
        const int c = min(127, (int)(__float_as_uint(shifted) & 0x007FFFFFu) - 0x00400000);
        codes[lane * 8 + i] = (int8_t)c;
        part += (int8_t)c;
    }
    part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
    if ((lane & 1) == 0) sums[lane >> 1] = (int16_t)part;
    if (lane == 0) *scale = __fdiv_rn(1.0f, inverse);
}

// ---------------------------------------------------------------------------------------- batch order
struct KBatchArgs {
    const uint8_t *payload;
    int rows, cols;
    const float *x;
    float *y;
    int epilogue;
    const float *bias;
    float *residual;
    int use_pdl;
    int stage;                 // 1: each warp copies its row into shared memory first (coalesced)
    int stage_stride;          // bytes of shared memory per warp's row copy (a multiple of 16, with slack)
};

// Half `h` of one (row, block) product: the exact integer sums of sub-blocks 4h..4h+3 (Q4_K) or groups
// 8h..8h+7 (Q6_K), which two lanes add together before one of them forms the FP32 term (k_term); integer
// sums do not depend on their order, so the term is the reference's bit for bit.  `rec` = the Q8_K record.
template <int FMT>
__device__ __forceinline__ void k_block_half(const uint8_t *blk, const uint8_t *rec, int h, int &isum, int &mins)
{
    const uint32_t *codes = reinterpret_cast<const uint32_t *>(rec);
    const int16_t *sums = reinterpret_cast<const int16_t *>(rec + 256);
    isum = 0;
    mins = 0;
    if (FMT == SATORI_Q4_K) {
        // Words 0..3: d, dmin and the 12 scale bytes; then this half's 64 code bytes (words 4 + 16h ..).
        const uint4 *b4 = reinterpret_cast<const uint4 *>(blk);
        uint32_t hw[4], qs[16];
        {
            const uint4 t = b4[0];
            hw[0] = t.x, hw[1] = t.y, hw[2] = t.z, hw[3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 t = b4[1 + 4 * h + k];
            qs[4 * k] = t.x, qs[4 * k + 1] = t.y, qs[4 * k + 2] = t.z, qs[4 * k + 3] = t.w;
        }
        // Scale byte n of the 12 (bytes 4 + n of the block), picked by shifts and selects (no local array:
        // the half h is a runtime value).
        auto sb = [&](int n) -> int {
            const uint32_t wd = n < 4 ? hw[1] : (n < 8 ? hw[2] : hw[3]);
            return (int)((wd >> (8 * (n & 3))) & 0xFFu);
        };
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int sub = 4 * h + s;
            int sc, mn;
            if (h == 0) {                       // Q4KCodec.GetScaleMin (Q4KCodec.cs:24-37), j < 4
                sc = sb(s) & 63;
                mn = sb(s + 4) & 63;
            } else {                            // j = 4 + s
                sc = (sb(s + 8) & 0xF) | ((sb(s) >> 6) << 4);
                mn = (sb(s + 8) >> 4) | ((sb(s + 4) >> 6) << 4);
            }
            int acc = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t q = qs[(s >> 1) * 8 + k];              // qs bytes (sub/2)*32 + 4k
                const uint32_t nib = (s & 1) ? (q >> 4) & 0x0F0F0F0Fu : q & 0x0F0F0F0Fu;
                acc = dp4a_us(nib, codes[sub * 8 + k], acc);
            }
            isum += sc * acc;
            mins += mn * ((int)sums[2 * sub] + (int)sums[2 * sub + 1]);
        }
    } else {
        // This half's low bits (words 16h ..), high bits (words 32 + 8h ..) and 8 scales (bytes 192 + 8h).
        uint32_t ql[16], qh[8], sw[2];
#pragma unroll
        for (int j = 0; j < 16; ++j) ql[j] = ld_u32_any(blk + 4 * (16 * h + j));
#pragma unroll
        for (int j = 0; j < 8; ++j) qh[j] = ld_u32_any(blk + 4 * (32 + 8 * h + j));
        sw[0] = ld_u32_any(blk + 192 + 8 * h);
        sw[1] = ld_u32_any(blk + 196 + 8 * h);
        const uint32_t *hcodes = codes + 32 * h;
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {                         // group g = 8h + gg = sub-block g
            const int k = gg >> 1, l0 = (gg & 1) * 16;
            int acc = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int l = l0 + 4 * i;
                const uint32_t qlw = ql[((k & 1) * 32 + l) >> 2];
                const uint32_t qhw = qh[l >> 2];
                const uint32_t nib = k < 2 ? qlw & 0x0F0F0F0Fu : (qlw >> 4) & 0x0F0F0F0Fu;
                const uint32_t q = nib | (((qhw >> (2 * k)) & 0x03030303u) << 4);
                acc = dp4a_us(q, hcodes[(32 * k + l) >> 2], acc);
            }
            const int scale = (int)(int8_t)((sw[gg >> 2] >> (8 * (gg & 3))) & 0xFFu);
            isum += scale * (acc - 32 * (int)sums[8 * h + gg]);
        }
    }
}

// The FP32 term of a block from its whole integer sums (the reference's combine order).
template <int FMT>
__device__ __forceinline__ float k_term(const uint8_t *blk, float as, int isum, int mins)
{
    if (FMT == SATORI_Q4_K) {
        const float d = h2f(blk), dmin = h2f(blk + 2);
        const float da = fmul(d, as), ma = fmul(dmin, as);
        return __fsub_rn(fmul(da, __int2float_rn(isum)), fmul(ma, __int2float_rn(mins)));
    }
    return fmul(fmul(as, h2f(blk + 208)), __int2float_rn(isum));
}

template <int FMT>
__global__ void __launch_bounds__(kKWarps * 32) kq_batch_kernel(const KBatchArgs a)
{
    extern __shared__ __align__(16) uint8_t kq_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.cols / 256;
    constexpr int BB = FMT == SATORI_Q4_K ? 144 : 210;
    const int row = blockIdx.x * kKWarps + warp;
    const uint8_t *rowp = a.payload + (size_t)min(row, a.rows - 1) * nb * BB;
    // The weights do not depend on the previous kernel: each warp's row starts moving into shared memory
    // (16-byte asynchronous copies, coalesced; a lane reading its own block would make every warp load
    // touch 32 lines) before the programmatic-launch wait, and lands while x is quantized.
    uint8_t *staged = kq_smem + (size_t)nb * kKRecord + (size_t)warp * a.stage_stride;
    if (a.stage && row < a.rows) {
        for (int i = lane; i < nb * BB / 16; i += 32)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(staged + 16 * i)),
                         "l"(rowp + 16 * i)
                         : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (a.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    for (int b = warp; b < nb; b += kKWarps) q8k_quantize_warp(a.x + b * 256, kq_smem + b * kKRecord, lane);
    if (a.stage) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (row >= a.rows) return;
    if (a.stage) rowp = staged;
    // Lanes 2j and 2j+1 share block j of each pass of 16 (one half each), so a 16-block row uses the
    // whole warp; the even lane holds the block's term.
    constexpr int kMaxPerLane = 8;                               // up to 128 blocks (32768 columns)
    float t[kMaxPerLane];
    bool live[kMaxPerLane];
    const int h = lane & 1;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        live[i] = false;
        t[i] = 0.0f;
        if (16 * i < nb) {                                       // warp-uniform: the shuffles see every lane
            const int b = (lane >> 1) + 16 * i;
            const int bc = min(b, nb - 1);                       // lanes past the row repeat its last block
            const uint8_t *blk = rowp + (size_t)bc * BB, *rec = kq_smem + bc * kKRecord;
            int isum, mins;
            k_block_half<FMT>(blk, rec, h, isum, mins);
            isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 1);
            mins += __shfl_xor_sync(0xFFFFFFFFu, mins, 1);
            const float as = *reinterpret_cast<const float *>(rec + 288);
            if (b < nb && as != 0.0f) {                          // an all-zero activation block adds nothing
                t[i] = k_term<FMT>(blk, as, isum, mins);
                live[i] = true;
            }
        }
    }
    // acc[row] += term, block by block (skipped blocks add nothing): block 16i + j is t[i] of lane 2j.
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
        if (16 * i >= nb) break;
        for (int j = 0; j < 16 && 16 * i + j < nb; ++j) {
            const float v = __shfl_sync(0xFFFFFFFFu, t[i], 2 * j);
            const bool on = __shfl_sync(0xFFFFFFFFu, live[i], 2 * j);
            if (on) acc = fadd(acc, v);
        }
    }
    if (lane == 0) {
        if (a.epilogue == kEpiBias) acc = fadd(acc, a.bias[row]);
        if (a.epilogue == kEpiResidual) {
            acc = fadd(a.residual[row], acc);
            a.residual[row] = acc;
        }
        a.y[row] = acc;
    }
}

// ---------------------------------------------------------------------------------------- float orders
template <int FMT, bool EXECUTE>
__global__ void kq_float_kernel(const uint8_t *payload, int rows, int cols, const float *x, float *y)
{
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const int nb = cols / 256;
    constexpr int BB = FMT == SATORI_Q4_K ? 144 : 210;
    float total = 0.0f;
    for (int blk = 0; blk < nb; ++blk) {
        const uint8_t *b = payload + ((size_t)row * nb + blk) * BB;
        const float *xb = x + blk * 256;
        // ExecuteScalar adds each block's DotBlock, which sums its own groups from zero; the execute order
        // adds every group's horizontal sum straight into the row total.
        float block_total = 0.0f;
        if (FMT == SATORI_Q4_K) {
            const float d = h2f(b), dmin = h2f(b + 2);
            for (int g = 0; g < 4; ++g) {
                const uint8_t *q = b + 16 + g * 32;
                int s0, n0, s1, n1;
                q4k_scale_min(2 * g, b + 4, s0, n0);
                q4k_scale_min(2 * g + 1, b + 4, s1, n1);
                const float dl = fmul(d, (float)s0), ml = fmul(dmin, (float)n0);
                const float dh = fmul(d, (float)s1), mh = fmul(dmin, (float)n1);
                if (!EXECUTE) {
                    // Q4KCodec.DotBlock (Q4KCodec.cs:40-66).
                    float lo = 0.0f, hi = 0.0f;
                    for (int l = 0; l < 32; ++l) {
                        lo = fadd(lo, fmul(__fsub_rn(fmul(dl, (float)(q[l] & 0xF)), ml), xb[g * 64 + l]));
                        hi = fadd(hi, fmul(__fsub_rn(fmul(dh, (float)(q[l] >> 4)), mh), xb[g * 64 + 32 + l]));
                    }
                    block_total = fadd(block_total, fadd(lo, hi));
                } else {
                    // QuantizedKAvx2Kernel.ExecuteQ4K (QuantizedKAvx2Kernel.cs:225-269).
                    float acc[8];
                    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
                    for (int j = 0; j < 32; j += 8)
                        for (int i = 0; i < 8; ++i) {
                            const float lw = __fsub_rn(fmul((float)(q[j + i] & 0xF), dl), ml);
                            const float hw = __fsub_rn(fmul((float)(q[j + i] >> 4), dh), mh);
                            acc[i] = fadd(acc[i], fmul(lw, xb[g * 64 + j + i]));
                            acc[i] = fadd(acc[i], fmul(hw, xb[g * 64 + 32 + j + i]));
                        }
                    total = fadd(total, hsum8(acc));
                }
            }
        } else {
            const float d = h2f(b + 208);
            const int8_t *scales = reinterpret_cast<const int8_t *>(b + 192);
            for (int half = 0; half < 2; ++half) {
                if (!EXECUTE) {
                    // Q6KCodec.DotBlock (Q6KCodec.cs:14-44): ((d * scale) * q) * x, left to right.
                    for (int l = 0; l < 32; ++l) {
                        const int sub = l / 16;
                        for (int k = 0; k < 4; ++k)
                            block_total = fadd(block_total, fmul(fmul(fmul(d, (float)scales[half * 8 + sub + 2 * k]),
                                                                      (float)q6k_code(b, half, l, k)),
                                                                 xb[half * 128 + l + 32 * k]));
                    }
                } else {
                    // QuantizedKAvx2Kernel.ExecuteQ6K (QuantizedKAvx2Kernel.cs:271-316).
                    for (int l = 0; l < 32; l += 8) {
                        const int sub = l / 16;
                        float acc[8];
                        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
                        for (int k = 0; k < 4; ++k) {
                            const float sk = fmul(d, (float)scales[half * 8 + sub + 2 * k]);
                            for (int i = 0; i < 8; ++i)
                                acc[i] = fadd(acc[i], fmul(fmul((float)q6k_code(b, half, l + i, k), sk),
                                                           xb[half * 128 + l + i + 32 * k]));
                        }
                        total = fadd(total, hsum8(acc));
                    }
                }
            }
        }
        if (!EXECUTE) total = fadd(total, block_total);
    }
    y[row] = total;
}

// ---------------------------------------------------------------------------------------- decode / validate
__global__ void kq_decode_row_kernel(const uint8_t *payload, int cols, int format, const int *row_dev, int row_host,
                                     float *out)
{
    const int row = row_dev ? *row_dev : row_host;
    const int nb = cols / 256;
    const int BB = format == SATORI_Q4_K ? 144 : 210;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < cols; e += gridDim.x * blockDim.x) {
        const uint8_t *b = payload + ((size_t)row * nb + e / 256) * BB;
        const int i = e % 256;
        float w;
        if (format == SATORI_Q4_K) {
            // Q4KCodec.DecodeBlock (Q4KCodec.cs:70-91).
            const int g = i / 64, hiq = (i % 64) >= 32, l = i % 32;
            int s, m;
            q4k_scale_min(2 * g + hiq, b + 4, s, m);
            const uint8_t q = b[16 + g * 32 + l];
            const float dd = fmul(h2f(b), (float)s), mm = fmul(h2f(b + 2), (float)m);
            w = __fsub_rn(fmul(dd, (float)(hiq ? q >> 4 : q & 0xF)), mm);
        } else {
            // Q6KCodec.DecodeBlock (Q6KCodec.cs:58-85).
            const int half = i / 128, r = i % 128, k = r / 32, l = r % 32;
            const int8_t sc = reinterpret_cast<const int8_t *>(b + 192)[half * 8 + l / 16 + 2 * k];
            w = fmul(fmul(h2f(b + 208), (float)sc), (float)q6k_code(b, half, l, k));
        }
        out[e] = w;
    }
}

__global__ void kq_validate_kernel(const uint8_t *payload, long long nblocks, int format, int *status)
{
    const int BB = format == SATORI_Q4_K ? 144 : 210;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nblocks;
         k += (long long)gridDim.x * blockDim.x) {
        const uint8_t *b = payload + k * BB;
        auto finite = [](const uint8_t *p) { return ((p[0] | (p[1] << 8)) & 0x7C00) != 0x7C00; };
        const bool ok = format == SATORI_Q4_K ? finite(b) && finite(b + 2) : finite(b + 208);
        if (!ok) atomicMax(status, (int)SATORI_ERR_INVALID_DATA);
    }
}

}  // namespace

bool is_kquant(int format) { return format == SATORI_Q4_K || format == SATORI_Q6_K; }

cudaError_t launch_kq_gemv(const GemvArgs &a, cudaStream_t stream)
{
    if (!is_kquant(a.format) || a.cols % 256 != 0 || a.cols > 32768) return cudaErrorInvalidValue;
    if (a.order == SATORI_ORDER_BATCH) {
        if (a.positions != 1) return cudaErrorInvalidValue;
        KBatchArgs k = {a.payload, a.rows, a.cols, a.x, a.y, a.epilogue, a.bias, a.residual, a.use_pdl, 0, 0};
        const int nb = a.cols / 256, bb = a.format == SATORI_Q4_K ? 144 : 210;
        size_t smem = (size_t)nb * kKRecord;
        // Rows are staged through shared memory when each row starts on a 16-byte boundary and the copies fit.
        // Each copy is followed by 16 bytes of slack: a Q6_K term reads its 210-byte block as 53 words, and
        // for a block at an odd 2-byte offset the last word reaches up to 6 bytes past the block (in global
        // memory the payload's padding covers the same reads).
        const size_t row_bytes = (size_t)nb * bb, stride = row_bytes + 16;
        if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(a.payload) & 15) == 0 &&
            smem + kKWarps * stride <= 96 * 1024) {
            k.stage = 1;
            k.stage_stride = (int)stride;
            smem += kKWarps * stride;
        }
        auto kern = a.format == SATORI_Q4_K ? kq_batch_kernel<SATORI_Q4_K> : kq_batch_kernel<SATORI_Q6_K>;
        const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(kern), smem);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((a.rows + kKWarps - 1) / kKWarps);
        cfg.blockDim = dim3(kKWarps * 32);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = a.use_pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, kern, k);
    }
    if (a.positions != 1 || a.epilogue != kEpiNone) return cudaErrorInvalidValue;
    const dim3 grid((a.rows + 127) / 128), block(128);
    const bool ex = a.order == SATORI_ORDER_EXECUTE;
    if (a.format == SATORI_Q4_K) {
        if (ex) kq_float_kernel<SATORI_Q4_K, true><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, a.x, a.y);
        else kq_float_kernel<SATORI_Q4_K, false><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, a.x, a.y);
    } else {
        if (ex) kq_float_kernel<SATORI_Q6_K, true><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, a.x, a.y);
        else kq_float_kernel<SATORI_Q6_K, false><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, a.x, a.y);
    }
    return cudaGetLastError();
}

cudaError_t launch_kq_decode_row(const uint8_t *payload, int cols, int format, const int *row_dev, int row_host,
                                 float *out, cudaStream_t stream)
{
    kq_decode_row_kernel<<<std::min(64, (cols + 255) / 256), 256, 0, stream>>>(payload, cols, format, row_dev,
                                                                              row_host, out);
    return cudaGetLastError();
}

cudaError_t launch_kq_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                               cudaStream_t stream)
{
    kq_validate_kernel<<<592, 256, 0, stream>>>(payload, (long long)rows * (cols / 256), format, status_dev);
    return cudaGetLastError();
}

}  // namespace satori
