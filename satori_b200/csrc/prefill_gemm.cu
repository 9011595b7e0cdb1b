// prefill_gemm.cu -- the batched projection of a prefill chunk on the 5th-generation tensor cores:
// Y[p][r] = sum_k W[r][k] * X[p][k] for up to 128 positions, W a GGUF Q8_0 / Q4_0 payload.
//
// DenseSession.Forward runs a chunk of positions through DenseForward.LayerBatch
// (src/Satori.Core/Model/DenseSession.cs:136-181, DenseForward.cs:178-262), whose projections are
// QuantizedMatVec.ExecuteBatch over all the chunk's positions (QuantizedMatVec.cs:221-365).  With many
// positions per weight this is a GEMM, and it belongs on tcgen05.  The tensor cores do not add in the
// reference's order, so this path is not bit-exact; it is accurate to FP32 level instead, because every
// operand is exact and every product exact:
//  * a weight w = d * q (fp16 scale times a 4- or 8-bit code) has at most 15 (Q4_0) or 19 (Q8_0)
//    significant bits, so it is exactly w1 + w2 (+ w3) with bf16 parts w_i (8 bits each, FP32's range);
//  * an activation x is x1 + x2 + x3 with bf16 parts, to within 2^-27 |x|;
//  * the cross products w_i * x_j with weight above 2^-24 go through kind::f16 MMAs (bf16 x bf16 ->
//    exact FP32 product) into one FP32 accumulator in tensor memory: 5 MMAs per K step for Q4_0, 6 for
//    Q8_0.
// The result differs from the reference's FP32 order by FP32 rounding of the sum (~K * 2^-24 of
// sum |w x|), which the prefill tests bound.
//
// One CTA computes a 128-row x N-position tile (N = positions rounded up to 16, at most 128):
//  * warps 0-3 (one warpgroup; thread t = row t of the tile) stage their row's Q8_0/Q4_0 bytes four
//    64-column steps ahead with cp.async, decode w exactly (byte-permute + FP32x2 FMA), split it with
//    packed bf16x2 conversions and store the parts in the canonical K-major layout (8-row x 16-byte core
//    matrices, no swizzle); after the last K step they read the accumulator back with tcgen05.ld (warp w
//    owns TMEM lanes 32w..32w+31) and write Y;
//  * warp 4 allocates the tensor memory, streams the pre-split activation tiles with 1-D bulk copies,
//    and one elected thread issues the MMAs and commits them to an mbarrier that frees the stage.
// Two stages; every wait is bounded, and on an expired wait the CTA still drains its MMAs and frees
// its tensor memory before returning.
//
// When the row tiles alone cannot fill the SMs (a 3584-row projection is 28 tiles) the K range is split
// across CTAs (blockIdx.y); each split writes its raw FP32 tile, and a second kernel adds the splits in
// split order and applies the epilogue, so the result does not depend on scheduling.
//
// Epilogues (the decode step's, applied per (position, row)): none, + bias (DenseForward.cs:124-129),
// residual += acc (DenseForward.cs:148,160), and SwiGlu of interleaved gate/up rows (DenseForward.cs:151-153).
#include "common.cuh"
#include "gemv.cuh"
#include "qblock.cuh"

#include <cuda_bf16.h>

#include <algorithm>

namespace satori {

namespace {

constexpr int kTcM = 128;            // tile rows (MMA M)
constexpr int kTcK = 64;             // columns per stage (4 MMA K steps of 16)
constexpr int kTcStages = 2;
constexpr int kTcXParts = 3;
constexpr int kTcThreads = 160;      // warps 0-3 decode + epilogue, warp 4 control
constexpr int kTcHeader = 256;
constexpr int kTcMaxPositions = 128;
constexpr int kTcRaw = 4;                 // K steps of raw weight bytes staged ahead per decode thread
constexpr uint32_t kTcApart = kTcM * kTcK * 2;   // 16 KB per bf16 weight part

struct TcOut {
    int rows, positions;
    int epilogue;                    // kEpiNone / kEpiBias / kEpiResidual / kEpiSwiGlu
    float *y;                        // y[p * ldy + r] (SwiGlu: y[p * ldy + r / 2]); may be null for residual
    int ldy;
    const float *bias;               // [rows]
    float *residual;                 // residual[p * ldr + r]
    int ldr;
};

struct TcArgs {
    const uint8_t *payload;
    int rows, cols, nkt;             // nkt = cols / 64
    int ksplit;                      // K ranges (blockIdx.y); > 1: raw tiles go to `partial`
    const uint8_t *xs;               // pre-split activations: [nkt][3][n16 * 64] bf16, core layout
    int n16;
    float *partial;                  // [ksplit][positions][rows]
    TcOut out;
    unsigned *err;
};

// The epilogue for one (position, row): `acc` is row r's sum, `acc_next` row r+1's (SwiGlu, r even).
__device__ __forceinline__ void tc_store(const TcOut &o, int p, int r, float acc, float acc_next)
{
    switch (o.epilogue) {
    case kEpiBias: o.y[(size_t)p * o.ldy + r] = fadd(acc, o.bias[r]); break;
    case kEpiResidual: {
        float *res = o.residual + (size_t)p * o.ldr + r;
        const float v = fadd(*res, acc);
        *res = v;
        if (o.y) o.y[(size_t)p * o.ldy + r] = v;
        break;
    }
    case kEpiSwiGlu:
        if ((r & 1) == 0) o.y[(size_t)p * o.ldy + r / 2] = swiglu_value(acc, acc_next);
        break;
    default: o.y[(size_t)p * o.ldy + r] = acc;
    }
}

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    // Shared-memory matrix descriptor, K-major without swizzle: start, leading (K) and stride (M/N) byte
    // offsets in 16-byte units, descriptor version 1, layout type 0.
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate ? 1u : 0u) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t bf16_bits(float v) { return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float bf16_value(uint32_t bits) { return __uint_as_float(bits << 16); }
// Both halves of a float pair rounded to bf16 (x in the low half), and their values back as floats.
__device__ __forceinline__ uint32_t bf16x2_bits(float2 v)
{
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t *>(&b);
}
__device__ __forceinline__ float2 bf16x2_value(uint32_t bits)
{
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xFFFF0000u));
}

template <int FMT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const TcArgs a)
{
    constexpr int NA = FMT == 0 ? 3 : 2;                    // bf16 parts of a weight
    constexpr int BB = FMT == 0 ? 34 : 18;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    uint64_t *full_b = reinterpret_cast<uint64_t *>(smem);          // activation tile landed
    uint64_t *a_ready = full_b + kTcStages;                          // 128 decode threads wrote the weights
    uint64_t *consumed = a_ready + kTcStages;                        // the stage's MMAs completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(consumed + kTcStages);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const uint32_t bpart = (uint32_t)a.n16 * kTcK * 2;               // bytes per activation part
    const uint32_t stage_bytes = NA * kTcApart + kTcXParts * bpart;
    uint8_t *stage0 = smem + kTcHeader;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * kTcM;
    // This CTA's K steps [k0, k0 + nk).
    const int k0 = (int)(((long long)a.nkt * blockIdx.y) / a.ksplit);
    const int nk = (int)(((long long)a.nkt * (blockIdx.y + 1)) / a.ksplit) - k0;
    const uint8_t *xs = a.xs + (size_t)k0 * kTcXParts * bpart;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full_b[s], 1);
            mbar_init(&a_ready[s], kTcM);
            mbar_init(&consumed[s], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" :: "r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            auto load_b = [&](int kt) {
                const int s = kt % kTcStages;
                uint8_t *dst = stage0 + (size_t)s * stage_bytes + NA * kTcApart;
                mbar_expect_tx(&full_b[s], kTcXParts * bpart);
                bulk_g2s(dst, xs + (size_t)kt * kTcXParts * bpart, kTcXParts * bpart, &full_b[s]);
            };
            for (int kt = 0; kt < min(kTcStages, nk); ++kt) load_b(kt);
            // Instruction descriptor: FP32 accumulator, bf16 A and B, both K-major, N = n16, M = 128.
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.n16 >> 3) << 17) |
                                   ((uint32_t)(kTcM >> 4) << 24);
            const int pairs = NA == 3 ? 6 : 5;
            const int pa[6] = {0, 0, 0, 1, 1, 2}, pb[6] = {0, 1, 2, 0, 1, 0};
            int last = -1;
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % kTcStages;
                const uint32_t par = (uint32_t)((kt / kTcStages) & 1);
                if (!mbar_wait_bounded(&full_b[s], par) || !mbar_wait_bounded(&a_ready[s], par)) goto fail;
                tc_fence_after();
                {
                    const uint32_t abase = smem_u32(stage0 + (size_t)s * stage_bytes);
                    const uint32_t bbase = abase + NA * kTcApart;
                    const uint32_t npg = (uint32_t)a.n16 / 8;
#pragma unroll
                    for (int ks = 0; ks < kTcK / 16; ++ks)
                        for (int q = 0; q < pairs; ++q) {
                            const uint64_t da = tc_desc(abase + pa[q] * kTcApart + ks * 4096u, 2048u, 128u);
                            const uint64_t db = tc_desc(bbase + pb[q] * bpart + ks * 2u * npg * 128u, npg * 128u, 128u);
                            tc_mma(tmem, da, db, idesc, kt > 0 || ks > 0 || q > 0);
                        }
                }
                tc_commit(&consumed[s]);
                last = kt;
                if (kt >= 1 && kt + 1 < nk) {
                    // Step kt is queued behind step kt-1: once kt-1's MMAs are done, its stage takes step
                    // kt+1's activations.
                    if (!mbar_wait_bounded(&consumed[(kt - 1) % kTcStages], (uint32_t)(((kt - 1) / kTcStages) & 1)))
                        goto fail;
                    load_b(kt + 1);
                }
            }
            goto done;
        fail:
            atomicOr(a.err, kDevErrTimeout);
            *abort_flag = 1;
        done:
            // The issued MMAs finish before the tensor memory can be freed.
            if (last >= 0) mbar_wait_bounded(&consumed[last % kTcStages], (uint32_t)((last / kTcStages) & 1));
        }
        __syncwarp();
    } else {
        // Decode: thread t owns tile row t.
        const int r = tid;
        const int grow = row0 + r;
        const bool live = grow < a.rows;
        const uint8_t *rowp = a.payload + (size_t)min(grow, a.rows - 1) * (a.cols / 32) * BB + (size_t)k0 * 2 * BB;
        // This thread's row bytes of each K step (two blocks: 36 (Q4_0) or 68 (Q8_0) bytes, 4-byte aligned)
        // are staged kTcRaw steps ahead by asynchronous copies into its own slots of the raw ring; only
        // this thread reads them, so its own wait_group is the only synchronisation they need.
        constexpr int NWD = BB * 2 / 4;
        uint32_t *raw = reinterpret_cast<uint32_t *>(stage0 + (size_t)kTcStages * stage_bytes) + r * NWD;
        auto stage_raw = [&](int kt) {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(rowp + (size_t)kt * 2 * BB);
            uint32_t *dst = raw + (size_t)(kt % kTcRaw) * kTcM * NWD;
#pragma unroll
            for (int i = 0; i < NWD; ++i)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst + i)), "l"(src + i)
                             : "memory");
        };
#pragma unroll
        for (int i = 0; i < kTcRaw; ++i) {
            if (i < nk) stage_raw(i);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        for (int kt = 0; kt < nk && !*abort_flag; ++kt) {
            const int s = kt % kTcStages;
            if (kt >= kTcStages &&
                !mbar_wait_bounded(&consumed[s], (uint32_t)(((kt - kTcStages) / kTcStages) & 1))) {
                atomicOr(a.err, kDevErrTimeout);
                *abort_flag = 1;
                break;
            }
            // Groups committed so far: kTcRaw + kt; step kt's is complete once at most kTcRaw - 1 pend.
            asm volatile("cp.async.wait_group %0;" ::"n"(kTcRaw - 1) : "memory");
            uint32_t wd[NWD];
            const uint32_t *mine = raw + (size_t)(kt % kTcRaw) * kTcM * NWD;
#pragma unroll
            for (int i = 0; i < NWD; ++i) wd[i] = live ? mine[i] : 0u;
            // Exact decode (QuantizedRow.DecodeQ8Block / DecodeQ4Block): a byte-permute puts each code byte
            // (the biased int8, or a masked nibble) under the 2^23 exponent and one FP32x2 FMA turns the pair
            // into d * code exactly (the scale constants are exact: d has at most 11 significant bits).
            float2 S[2][2], C[2][2];
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                const int pos = blk * BB;                                    // byte of the block's scale
                const float d = half_bits_to_float((wd[pos >> 2] >> (8 * (pos & 3))) & 0xFFFFu);
                if (FMT == 0) {
                    const float sc = fmul(d, 0.00390625f), cc = fmul(d, -32896.0f);      // 2^-8, -(2^15 + 128)
                    S[blk][0] = S[blk][1] = make_float2(sc, sc);
                    C[blk][0] = C[blk][1] = make_float2(cc, cc);
                } else {
                    const float sl = fmul(d, 0.00390625f), cl = fmul(d, -32776.0f);      // low nibble in place
                    const float sh = fmul(d, 0.000244140625f), ch = fmul(d, -2056.0f);   // high nibble in place
                    S[blk][0] = make_float2(sl, sl);
                    C[blk][0] = make_float2(cl, cl);
                    S[blk][1] = make_float2(sh, sh);
                    C[blk][1] = make_float2(ch, ch);
                }
            }
            const float2 minus1 = make_float2(-1.0f, -1.0f);
            uint8_t *abase = stage0 + (size_t)s * stage_bytes;
#pragma unroll
            for (int kc = 0; kc < kTcK / 8; ++kc) {
                uint32_t part[NA][4];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    // Weights k, k+1 of this step: block k / 32, codes j, j+1 (j even, so the two code
                    // bytes share a word).
                    const int k = kc * 8 + e, blk = k >> 5, j = k & 31;
                    float2 W;
                    if (FMT == 0) {
                        const int pb = blk * BB + 2 + j;
                        const uint32_t u = wd[pb >> 2] ^ 0x80808080u;        // biased: code + 128
                        W = __ffma2_rn(code_pair(u, pb & 3, (pb & 3) + 1), S[blk][0], C[blk][0]);
                    } else {
                        const int hi = j >= 16, pb = blk * BB + 2 + (j & 15);
                        const uint32_t u = wd[pb >> 2] & (hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
                        W = __ffma2_rn(code_pair(u, pb & 3, (pb & 3) + 1), S[blk][hi], C[blk][hi]);
                    }
                    // Exact bf16 parts: each residual w - part is exact in FP32 (fma with -1).
                    const uint32_t p0 = bf16x2_bits(W);
                    const float2 r1 = __ffma2_rn(bf16x2_value(p0), minus1, W);
                    const uint32_t p1 = bf16x2_bits(r1);
                    part[0][e / 2] = p0;
                    part[1][e / 2] = p1;
                    if (NA == 3) part[2][e / 2] = bf16x2_bits(__ffma2_rn(bf16x2_value(p1), minus1, r1));
                }
                // Core matrix (row group r/8, K chunk kc): 8 rows x 16 bytes; chunks of a row group are
                // 2048 bytes apart (the K direction), row groups 128 bytes apart.
                const uint32_t off = (uint32_t)(kc * 16 + (r >> 3)) * 128u + (uint32_t)(r & 7) * 16u;
#pragma unroll
                for (int p = 0; p < NA; ++p)
                    *reinterpret_cast<uint4 *>(abase + p * kTcApart + off) =
                        make_uint4(part[p][0], part[p][1], part[p][2], part[p][3]);
            }
            fence_proxy_async();          // the tensor core reads these stores through the async proxy
            mbar_arrive(&a_ready[s]);
            // wd has been consumed, so step kt's slots are free for step kt + kTcRaw.
            if (kt + kTcRaw < nk) stage_raw(kt + kTcRaw);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        asm volatile("cp.async.wait_all;" ::: "memory");     // no copy lands after the CTA winds down
        // Epilogue: wait for the last step's MMAs, then TMEM lanes 32w..32w+31 hold rows of this warp.
        const int lastkt = nk - 1;
        bool ok = !*abort_flag &&
                  mbar_wait_bounded(&consumed[lastkt % kTcStages], (uint32_t)((lastkt / kTcStages) & 1));
        ok = __all_sync(0xFFFFFFFFu, ok);     // tcgen05.ld and the shuffles below take the whole warp
        tc_fence_after();
        if (ok) {
            for (int c0 = 0; c0 < a.n16; c0 += 32) {
                uint32_t v[32];
                const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                             "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                             "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
                               "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
                               "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
                               "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
                               "=r"(v[31])
                             : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int np = a.out.positions;
                if (a.ksplit > 1) {
                    float *part = a.partial + (size_t)blockIdx.y * np * a.rows;
                    if (live) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (c0 + j < np) part[(size_t)(c0 + j) * a.rows + grow] = __uint_as_float(v[j]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float acc = __uint_as_float(v[j]);
                        const float nxt = __shfl_down_sync(0xFFFFFFFFu, acc, 1);   // row r+1 (SwiGlu pairs)
                        if (live && c0 + j < np) tc_store(a.out, c0 + j, grow, acc, nxt);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" :: "r"(tmem));
}

// Activations [positions][cols] FP32 -> three bf16 parts per value, laid out per 64-column step in the
// canonical K-major core-matrix order the MMA reads (positions padded with zeros to n16).
__global__ void tc_split_kernel(const float *x, int positions, int cols, int n16, uint8_t *xs)
{
    const int npg = n16 / 8;
    const size_t per_part = (size_t)n16 * kTcK * 2;
    const size_t total = (size_t)n16 * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int p = (int)(i / cols), k = (int)(i % cols);
        const float v = p < positions ? x[(size_t)p * cols + k] : 0.0f;
        const uint32_t x1 = bf16_bits(v);
        const float r1 = __fsub_rn(v, bf16_value(x1));
        const uint32_t x2 = bf16_bits(r1);
        const uint32_t x3 = bf16_bits(__fsub_rn(r1, bf16_value(x2)));
        const int kt = k / kTcK, kk = k % kTcK, kc = kk / 8;
        const size_t off = (size_t)kt * kTcXParts * per_part + (size_t)(kc * npg + p / 8) * 128 + (p % 8) * 16 +
                           (kk % 8) * 2;
        *reinterpret_cast<uint16_t *>(xs + off) = (uint16_t)x1;
        *reinterpret_cast<uint16_t *>(xs + off + per_part) = (uint16_t)x2;
        *reinterpret_cast<uint16_t *>(xs + off + 2 * per_part) = (uint16_t)x3;
    }
}

// Split-K: adds the splits' raw tiles in split order, then the epilogue.  One thread per (position,
// row) -- per row pair for SwiGlu.
__global__ void tc_reduce_kernel(const float *partial, int ksplit, TcOut o)
{
    const int step = o.epilogue == kEpiSwiGlu ? 2 : 1;
    const size_t per = (size_t)o.positions * o.rows;
    const size_t n = per / step;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t e = i * step;
        const int p = (int)(e / o.rows), r = (int)(e % o.rows);
        float acc = partial[e], nxt = step == 2 ? partial[e + 1] : 0.0f;
        for (int s = 1; s < ksplit; ++s) {
            acc = fadd(acc, partial[s * per + e]);
            if (step == 2) nxt = fadd(nxt, partial[s * per + e + 1]);
        }
        tc_store(o, p, r, acc, nxt);
    }
}

int tc_ksplit(int rows, int cols, int sm_count)
{
    const int tiles = (rows + kTcM - 1) / kTcM, nkt = cols / kTcK;
    int ks = std::max(1, sm_count / tiles);
    ks = std::min(ks, std::max(1, nkt / 8));   // at least 8 K steps per split
    return std::min(ks, 16);
}

}  // namespace

bool tc_gemm_takes(int rows, int cols, int format, int positions, int epilogue)
{
    return (format == SATORI_Q8_0 || format == SATORI_Q4_0) && rows > 0 && cols > 0 && cols % kTcK == 0 &&
           positions >= 1 && positions <= kTcMaxPositions && (epilogue != kEpiSwiGlu || rows % 2 == 0);
}

size_t tc_scratch_bytes(int rows, int cols, int positions, int sm_count)
{
    const int n16 = (std::min(positions, kTcMaxPositions) + 15) / 16 * 16;
    const size_t xs = ((size_t)n16 * cols * 2 * kTcXParts + 255) / 256 * 256;
    const int ks = tc_ksplit(rows, cols, sm_count);
    return xs + (ks > 1 ? (size_t)ks * positions * rows * 4 : 0);
}

cudaError_t launch_tc_gemm(const TcGemm &g, int sm_count, cudaStream_t stream)
{
    if (!tc_gemm_takes(g.rows, g.cols, g.format, g.positions, g.epilogue) || !g.x || !g.scratch ||
        g.scratch_bytes < tc_scratch_bytes(g.rows, g.cols, g.positions, sm_count))
        return cudaErrorInvalidValue;
    if ((g.epilogue == kEpiResidual && !g.residual) || (g.epilogue != kEpiResidual && !g.y) ||
        (g.epilogue == kEpiBias && !g.bias))
        return cudaErrorInvalidValue;
    const int n16 = (g.positions + 15) / 16 * 16;
    const size_t elems = (size_t)n16 * g.cols;
    uint8_t *xs = g.scratch;
    const size_t xs_bytes = ((size_t)n16 * g.cols * 2 * kTcXParts + 255) / 256 * 256;
    tc_split_kernel<<<(unsigned)std::min<size_t>(4 * (size_t)sm_count, (elems + 255) / 256), 256, 0, stream>>>(
        g.x, g.positions, g.cols, n16, xs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    TcArgs a;
    a.payload = g.payload;
    a.rows = g.rows;
    a.cols = g.cols;
    a.nkt = g.cols / kTcK;
    a.ksplit = tc_ksplit(g.rows, g.cols, sm_count);
    a.xs = xs;
    a.n16 = n16;
    a.partial = reinterpret_cast<float *>(g.scratch + xs_bytes);
    a.out.rows = g.rows;
    a.out.positions = g.positions;
    a.out.epilogue = g.epilogue;
    a.out.y = g.y;
    a.out.ldy = g.ldy > 0 ? g.ldy : (g.epilogue == kEpiSwiGlu ? g.rows / 2 : g.rows);
    a.out.bias = g.bias;
    a.out.residual = g.residual;
    a.out.ldr = g.ldr > 0 ? g.ldr : g.rows;
    a.err = g.err;
    const int na = g.format == SATORI_Q8_0 ? 3 : 2;
    const int bb = g.format == SATORI_Q8_0 ? 34 : 18;
    const size_t smem = 128 + kTcHeader + (size_t)kTcStages * (na * kTcApart + kTcXParts * (size_t)n16 * kTcK * 2) +
                        (size_t)kTcRaw * kTcM * 2 * bb;
    auto kern = g.format == SATORI_Q8_0 ? tc_gemm_kernel<0> : tc_gemm_kernel<1>;
    e = opt_in_smem(reinterpret_cast<const void *>(kern), smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3((g.rows + kTcM - 1) / kTcM, a.ksplit), kTcThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess || a.ksplit == 1) return e;
    const size_t n = (size_t)g.positions * g.rows / (g.epilogue == kEpiSwiGlu ? 2 : 1);
    tc_reduce_kernel<<<(unsigned)std::min<size_t>(4 * (size_t)sm_count, (n + 255) / 256), 256, 0, stream>>>(
        a.partial, a.ksplit, a.out);
    return cudaGetLastError();
}

}  // namespace satori
