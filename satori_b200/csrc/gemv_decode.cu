// gemv_decode.cu -- decode-order MatVec of one position for GGUF Q8_0 / Q4_0, sm_100a.
//
// QuantizedMatVec.ExecuteBatchFloat -> ExecuteBatchRows -> Dot (QuantizedMatVec.cs:221-365) with a
// single position is what every decode projection runs.  Per row it is a left-to-right FP32 sum over
// blocks of one term per block; a term is eight FMA lanes over the block's 32 dequantized weights
// (QuantizedRow.DecodeQ8Block / DecodeQ4Block: scale * code) closed by the SSE horizontal sum
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)).  Terms are independent, so the compute warps produce them
// in parallel and a control warp adds them per row in block order: bit-identical to the reference.
//
// Requirements (checked by plan_gemv_decode; other shapes take the general kernel in gemv.cu):
// cols % 256 == 0, so every row is a whole number of 16-byte units and 8-block groups.
//
// Data movement and layout:
//  * The CTA owns `rc` consecutive rows (a multiple of 8).  They are streamed in column chunks of 16
//    blocks: one 2-D TMA tile load (rc rows x 16 blocks of bytes, unicast) per chunk into a ring of
//    shared-memory slots.  Rows past the matrix end read as zeros.  Weights cross HBM exactly once,
//    in their GGUF layout.  The activation vector stays resident in shared memory for the whole CTA,
//    128 floats (4 blocks) per 528-byte group: the 16-byte pad puts the four groups a warp reads in
//    distinct bank quads, and the 8 lanes that share a group read the same address (broadcast).
//  * Warp task = 8 rows x 16 blocks x one half of each 4-block group.  Lane (r = lane / 4, p = lane % 4)
//    takes blocks 4p + 2h and 4p + 2h + 1 of row r.  A 4-block group is 136 (Q8_0) or 72 (Q4_0) bytes,
//    8-byte aligned, read with 64-bit shared loads; with the tile's row pitch (544 / 288 bytes) the 32
//    lanes hit 32 distinct banks.  Inside a group the blocks sit at fixed byte phases, so every byte
//    select is a constant.
//  * A weight slot is released as soon as its tasks have loaded their words into registers (mbarrier
//    `empty`), so the next chunk's copy starts while the terms are still being computed.
//  * Terms go to a separate ring of tables D[block][row] (row pitch rc + 2 floats: conflict-free for
//    the lanes writing and for the control warp reading one row per lane).
//  * One control warp keeps both rings moving without blocking: it re-arms each weight slot once its
//    chunk is consumed and adds each chunk's terms, in block order, into its row sums.
#include <cuda.h>

#include "common.cuh"
#include "gemv.cuh"
#include "qblock.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kComputeWarps = 8;
constexpr int kDecThreads = (kComputeWarps + 1) * 32;
constexpr int kChunkBlocks = 16;     // blocks per column chunk (one stage)
constexpr int kTaskRows = 8;         // rows per warp task
constexpr int kMaxRows = 128;        // rows per CTA (control warp: 4 rows per lane)
constexpr int kMaxStages = 8;
constexpr uint32_t kStageTarget = 40960;   // largest stage (bytes of weights) a plan uses
constexpr int kTermSlots = 3;              // ring of term tables
constexpr int kHeaderBytes = 256;          // mbarriers, flags, slot tags
constexpr size_t kSmemBudget = 110 * 1024; // two CTAs per SM when the shape allows

struct DecGeo {
    int rows, bpr, rc, nchunks, stages;
    uint32_t x_bytes, d_bytes;
    const float *x;
    float *y;
    int epilogue;
    const float *bias;
    float *residual;
    unsigned *err;
    int use_pdl;
};

// Shared-memory byte offset of the 16-byte x chunk q of block B in the resident activation table:
// blocks are 128 bytes, chunk q stored at slot q ^ ((B >> 1) & 7) so that the 8 blocks of one phase
// a warp reads (B = 2e + phase) sit in 8 distinct bank quads.
__host__ __device__ __forceinline__ uint32_t x_chunk_offset(int B, int q)
{
    return 128u * (uint32_t)B + 16u * (uint32_t)(q ^ ((B >> 1) & 7));
}

// Bounded wait until a shared counter reaches `target` (written by the control warp).
__device__ __forceinline__ bool wait_counter(volatile int *counter, int target)
{
    if (*counter >= target) return true;
    const long long start = clock64();
    while (*counter < target) {
        if (clock64() - start > kWaitBudgetCycles) return false;
        __nanosleep(32);
    }
    return true;
}

// One warp task: rows 8*rg .. 8*rg+7 x the 8 blocks of phase PH (even blocks: PH = 0, odd: PH = 2) of
// a chunk.  Lane (r = lane / 8, e = lane % 8) keeps the activations of block b = 2e + PH/2 in registers
// and computes rows r and r + 4.  Returns after the weights are read (the caller releases the slot)
// through `terms`.
template <int FMT, int PH>
struct PhaseTask {
    static constexpr int NW = FMT == 0 ? 9 : 5;   // words holding one block (from its aligned start)

    // Words of the lane's two rows, from the weight slot at shared address `ws`.
    __device__ __forceinline__ static void load(uint32_t ws, int rg, int lane, uint32_t (&w)[2][9])
    {
        constexpr int PITCH = kChunkBlocks * blk_bytes(FMT);
        const int r = lane >> 3, e = lane & 7;
        const int b = 2 * e + (PH ? 1 : 0);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const uint32_t a = ws + (uint32_t)((rg * kTaskRows + r + 4 * m) * PITCH + b * blk_bytes(FMT) - PH);
#pragma unroll
            for (int k = 0; k < NW; ++k) w[m][k] = lds32(a + 4u * k);
        }
    }

    __device__ __forceinline__ static void activations(uint32_t xs, int k, int lane, float4 (&xv)[8])
    {
        const int B = k * kChunkBlocks + 2 * (lane & 7) + (PH ? 1 : 0);
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[q] = lds128f(xs + x_chunk_offset(B, q));
    }
};

template <int FMT>
__global__ void __launch_bounds__(kDecThreads, 2) gemv_decode_kernel(const __grid_constant__ CUtensorMap tmap, DecGeo g)
{
    constexpr int PITCH = kChunkBlocks * blk_bytes(FMT);   // bytes of one row in a weight slot
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // Carve from a 128-byte aligned base (TMA destinations); the plan adds the slack.
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = g.stages, SD = kTermSlots, rc = g.rc, nchunks = g.nchunks;
    const int row0 = blockIdx.x * rc;
    const int tpc = 2 * (rc / kTaskRows);          // tasks per chunk
    const int dpitch = rc + 2;                       // D row pitch (floats)
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);     // [kMaxStages] weights landed
    uint64_t *empty = full + kMaxStages;                     // [kMaxStages] weights consumed
    uint64_t *dfull = empty + kMaxStages;                    // [kTermSlots] terms written
    volatile int *abort_flag = reinterpret_cast<volatile int *>(dfull + kTermSlots);
    volatile int *folded = abort_flag + 1;          // chunks added into the row sums so far
    // issued[s] = the latest chunk put in flight into weight slot s.  A compute warp may skip some of
    // a slot's chunks (its tasks need not touch every chunk) and a parity wait only tells the current
    // phase from the one before it, so a warp first checks that its chunk is the one in flight.
    volatile int *issued = folded + 1;
    uint8_t *xs = smem + kHeaderBytes;
    float *D = reinterpret_cast<float *>(xs + g.x_bytes);
    uint8_t *wslot0 = reinterpret_cast<uint8_t *>(D) + g.d_bytes;
    const uint32_t w_bytes = (uint32_t)rc * PITCH;

    if (tid == 0) {
        *abort_flag = 0;
        *folded = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], tpc);
            issued[s] = s;
        }
        for (int s = 0; s < SD; ++s) mbar_init(&dfull[s], tpc);
        fence_mbar_init();
    }
    __syncthreads();

    const bool control = warp == kComputeWarps;
    auto issue_weights = [&](int k) {
        const int s = k % S;
        mbar_expect_tx(&full[s], w_bytes);
        tma_load_2d(wslot0 + (size_t)s * w_bytes, &tmap, k * (PITCH / 4), row0, &full[s]);
    };
    // Weights never depend on the previous kernel: start streaming them before the PDL wait; the
    // activations are read once the previous kernel is complete.
    const int first = min(S, nchunks);
    if (control && lane == 0) {
        prefetch_tensormap(&tmap);
        for (int k = 0; k < first; ++k) issue_weights(k);
    }
    if (g.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    {
        const float4 *x4 = reinterpret_cast<const float4 *>(g.x);
        const int n4 = g.bpr * 8;
        for (int i = tid; i < n4; i += kDecThreads)
            *reinterpret_cast<float4 *>(xs + x_chunk_offset(i >> 3, i & 7)) = x4[i];
    }
    __syncthreads();

    const uint32_t xs_u = smem_u32(xs), w_u = smem_u32(wslot0);
    if (!control) {
        // Task t = warp, warp + kComputeWarps, ...: chunk k = t / tpc, rem = t % tpc, slot s = k % S,
        // stepped incrementally (kComputeWarps <= tpc is not assumed).
        int k = 0, rem = warp, s = 0;
        while (rem >= tpc) {
            rem -= tpc;
            ++k;
            if (++s == S) s = 0;
        }
        for (; k < nchunks;) {
            const int rg = rem >> 1, ph = rem & 1;
            bool ok = !*abort_flag;
            if (ok) ok = wait_counter(issued + s, k) && mbar_wait_bounded(&full[s], (uint32_t)((k / S) & 1));
            if (!ok) {
                atomicOr(g.err, kDevErrTimeout);
                *abort_flag = 1;
                break;
            }
            const uint32_t ws = w_u + (uint32_t)s * w_bytes;
            uint32_t w[2][9];
            float4 xv[8];
            if (ph == 0) {
                PhaseTask<FMT, 0>::load(ws, rg, lane, w);
                PhaseTask<FMT, 0>::activations(xs_u, k, lane, xv);
            } else {
                PhaseTask<FMT, 2>::load(ws, rg, lane, w);
                PhaseTask<FMT, 2>::activations(xs_u, k, lane, xv);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);       // the slot may be refilled now
            float t0, t1;
            if (ph == 0) {
                t0 = block_term<FMT, 0>(w[0], xv);
                t1 = block_term<FMT, 0>(w[1], xv);
            } else {
                t0 = block_term<FMT, 2>(w[0], xv);
                t1 = block_term<FMT, 2>(w[1], xv);
            }
            // Term slot k % SD is free once chunk k - SD has been added in.
            if (!wait_counter(folded, k - SD + 1)) {
                atomicOr(g.err, kDevErrTimeout);
                *abort_flag = 1;
                break;
            }
            const int row = rg * kTaskRows + (lane >> 3), b = 2 * (lane & 7) + ph;
            float *dcol = D + ((size_t)(k % SD) * kChunkBlocks + b) * dpitch;
            dcol[row] = t0;
            dcol[row + 4] = t1;
            __syncwarp();
            if (lane == 0) mbar_arrive(&dfull[k % SD]);
            rem += kComputeWarps;
            while (rem >= tpc) {
                rem -= tpc;
                ++k;
                if (++s == S) s = 0;
            }
        }
    } else {
        float acc[kMaxRows / 32];
#pragma unroll
        for (int i = 0; i < kMaxRows / 32; ++i) acc[i] = 0.0f;
        int ka = 0;                                   // chunks whose slot has been re-armed
        int kf = 0;                                   // chunks added into the row sums
        const int rearm = max(0, nchunks - S);
        long long idle_since = clock64();
        while (kf < nchunks && !*abort_flag) {
            bool progress = false;
            if (ka < rearm) {
                const bool ready = __shfl_sync(0xFFFFFFFFu, lane == 0 ? (int)mbar_test(&empty[ka % S], (uint32_t)((ka / S) & 1)) : 0, 0);
                if (ready) {
                    if (lane == 0) {
                        issued[ka % S] = ka + S;
                        issue_weights(ka + S);
                    }
                    ++ka;
                    progress = true;
                }
            }
            const bool done = __shfl_sync(0xFFFFFFFFu, lane == 0 ? (int)mbar_test(&dfull[kf % SD], (uint32_t)((kf / SD) & 1)) : 0, 0);
            if (done) {
                const int nb = min(kChunkBlocks + 0, g.bpr - kf * kChunkBlocks);
                const float *dtab = D + (size_t)(kf % SD) * kChunkBlocks * dpitch;
#pragma unroll
                for (int i = 0; i < kMaxRows / 32; ++i) {
                    const int row = lane + 32 * i;
                    if (row < rc) {
                        float v[kChunkBlocks];
#pragma unroll
                        for (int j = 0; j < kChunkBlocks; ++j) v[j] = dtab[j * dpitch + row];
#pragma unroll
                        for (int j = 0; j < kChunkBlocks; ++j)
                            if (j < nb) acc[i] = fadd(acc[i], v[j]);
                    }
                }
                __syncwarp();
                ++kf;
                if (lane == 0) *folded = kf;
                progress = true;
            }
            if (progress) {
                idle_since = clock64();
            } else if (clock64() - idle_since <= kWaitBudgetCycles) {
                __nanosleep(64);                      // leave the issue slots to the compute warps
            } else {
                if (lane == 0) {
                    atomicOr(g.err, kDevErrTimeout);
                    *abort_flag = 1;
                }
                __syncwarp();
            }
        }
        if (*abort_flag) {
            // Let the copies already issued land before the CTA's shared memory goes away.
            if (lane == 0) {
                const int last = ka + S - 1 < nchunks - 1 ? ka + S - 1 : nchunks - 1;
                for (int k = max(0, last - S + 1); k <= last; ++k) mbar_wait_bounded(&full[k % S], (uint32_t)((k / S) & 1));
            }
        } else {
#pragma unroll
            for (int i = 0; i < kMaxRows / 32; ++i) {
                const int row = lane + 32 * i, grow = row0 + row;
                if (row < rc && grow < g.rows) {
                    float v = acc[i];
                    if (g.epilogue == kEpiBias) v = fadd(v, g.bias[grow]);
                    if (g.epilogue == kEpiResidual) {
                        v = fadd(g.residual[grow], v);
                        g.residual[grow] = v;
                    }
                    g.y[grow] = v;
                }
            }
        }
    }
}

// cuTensorMapEncodeTiled is resolved through the runtime so the library needs no link-time driver symbol.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

template <int FMT>
cudaError_t launch_decode(const CUtensorMap &map, const DecGeo &g, const DecodePlan &plan, cudaStream_t stream)
{
    auto kern = gemv_decode_kernel<FMT>;
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(kern), plan.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, map, g);
}

}  // namespace

namespace {
struct DecSizes {
    size_t x, d, w;
};
DecSizes dec_sizes(int format, int bpr, int rc)
{
    const int nchunks = (bpr + kChunkBlocks - 1) / kChunkBlocks;
    DecSizes z;
    z.x = (size_t)nchunks * kChunkBlocks * 128;    // resident activations, 128 bytes per block
    z.d = (((size_t)kTermSlots * kChunkBlocks * (rc + 2) * 4) + 127) & ~(size_t)127;
    z.w = (size_t)rc * kChunkBlocks * blk_bytes(format);
    return z;
}
}  // namespace

DecodePlan plan_gemv_decode(const GemvArgs &a, int sm_count, size_t smem_limit)
{
    DecodePlan p = {};
    if ((a.format != 0 && a.format != 1) || a.order != SATORI_ORDER_BATCH || a.positions != 1) return p;
    if (a.cols <= 0 || a.cols % 256 != 0 || a.rows <= 0 || a.epilogue == kEpiSwiGlu) return p;
    if ((reinterpret_cast<uintptr_t>(a.payload) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return p;
    if (!encode_fn()) return p;
    const int pitch = kChunkBlocks * blk_bytes(a.format);
    const int bpr = a.cols / 32;
    const int nchunks = (bpr + kChunkBlocks - 1) / kChunkBlocks;
    // Rows per CTA: one wave over the SMs, in whole 8-row tasks, stage at most kStageTarget bytes.
    const int per_sm = (a.rows + sm_count - 1) / std::max(sm_count, 1);
    int rc = (per_sm + kTaskRows - 1) / kTaskRows * kTaskRows;
    const int rc_cap = std::min(kMaxRows, (int)(kStageTarget / pitch) / kTaskRows * kTaskRows);
    rc = std::max(kTaskRows, std::min(rc, rc_cap));
    const DecSizes z = dec_sizes(a.format, bpr, rc);
    const size_t fixed = 128 + kHeaderBytes + z.x + z.d;
    // Two CTAs per SM (the next kernel's prologue overlaps this one) when three stages fit in half the
    // SM; otherwise one CTA with as many stages as the SM holds.
    const size_t budget = fixed + 3 * z.w <= kSmemBudget ? kSmemBudget : smem_limit;
    if (budget < fixed + 2 * z.w) return p;
    int stages = (int)std::min<size_t>(kMaxStages, (budget - fixed) / z.w);
    stages = std::min(stages, std::max(nchunks, 2));
    p.ok = 1;
    p.kind = 2;
    p.rc = rc;
    p.grid = (a.rows + rc - 1) / rc;
    p.stages = stages;
    p.nchunks = nchunks;
    p.smem = fixed + stages * z.w;
    return p;
}

cudaError_t launch_gemv_decode(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream)
{
    EncodeTiledFn enc = encode_fn();
    if (!plan.ok || !enc) return cudaErrorInvalidValue;
    const int bb = blk_bytes(a.format);
    const int bpr = a.cols / 32;
    const cuuint64_t row_bytes = (cuuint64_t)bpr * bb;
    // The payload as a 2-D array of 32-bit words: [rows][row_bytes / 4].
    CUtensorMap map;
    const cuuint64_t dims[2] = {row_bytes / 4, (cuuint64_t)a.rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(kChunkBlocks * bb / 4), (cuuint32_t)plan.rc};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(a.payload), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    DecGeo g;
    g.rows = a.rows;
    g.bpr = bpr;
    g.rc = plan.rc;
    g.nchunks = plan.nchunks;
    g.stages = plan.stages;
    {
        const DecSizes z = dec_sizes(a.format, bpr, plan.rc);
        g.x_bytes = (uint32_t)z.x;
        g.d_bytes = (uint32_t)z.d;
    }
    g.x = a.x;
    g.y = a.y;
    g.epilogue = a.epilogue;
    g.bias = a.bias;
    g.residual = a.residual;
    g.err = a.err;
    g.use_pdl = a.use_pdl;
    return a.format == 0 ? launch_decode<0>(map, g, plan, stream) : launch_decode<1>(map, g, plan, stream);
}

}  // namespace satori
