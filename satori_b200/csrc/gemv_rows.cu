// gemv_rows.cu -- decode-order MatVec of one position, GGUF Q8_0 / Q4_0, rows up to 8192 columns.
//
// Same arithmetic as gemv_decode.cu (QuantizedMatVec.ExecuteBatchFloat -> ExecuteBatchRows -> Dot,
// QuantizedMatVec.cs:221-365, one position): per row a left-to-right FP32 sum over blocks of one
// block term each (qblock.cuh), bit-identical to the reference.
//
// Layout and data movement (cols % 256 == 0 and cols <= 8192):
//  * One wave: CTA c owns a contiguous range of `rc` rows, i.e. one contiguous byte range of the GGUF
//    payload.  It is streamed front to back in stages of `rs` whole rows, one 1-D bulk copy each (TMA
//    unicast), into a ring of shared-memory slots.  Weights cross HBM exactly once.
//  * Each lane of the compute warps owns one block column for the whole kernel: warp w takes blocks of
//    one phase (even or odd block index -- the block's byte offset mod 4 is then fixed, so every byte
//    select is a constant) and 32 consecutive blocks of that phase; its 32 activations are loaded once,
//    into registers.  With 4-byte word loads the 32 lanes read 32 distinct banks (block strides of 17 /
//    9 words are odd).  When a row needs fewer warps than there are, the warps split the stage's rows.
//  * A lane loads the next row's words before computing the current one; the slot is released once
//    every warp has loaded its last row, then the lanes finish their terms into a per-slot table
//    D[row][phase][column] (conflict-free writes and reads).
//  * One control warp re-arms consumed slots, and adds each finished stage's terms in block order (one
//    lane per row) and writes the rows' outputs with the epilogue.
#include "common.cuh"
#include "gemv.cuh"
#include "qblock.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kRowsWarps = 8;                          // compute warps (warps 1 .. 8)
constexpr int kRowsThreads = (kRowsWarps + 2) * 32;    // + fold warp (0) + producer warp (9)
constexpr int kFoldRows = 32;                          // rows per fold batch (one fold lane per row)
constexpr int kFoldSlots = 2;                          // term tables (fold batches in flight)
constexpr int kRowsMaxStages = 8;
constexpr int kRowsMaxStageRows = 32;                  // one control lane per row of a stage
constexpr int kRowsHeader = 256;
constexpr size_t kRowsStageTarget = 20 * 1024;         // bytes of weights per stage
constexpr size_t kRowsBudget = 110 * 1024;             // two CTAs per SM: the next kernel starts early

struct RowsGeo {
    const uint8_t *payload;
    int rows, bpr, rc, rs, stages, nstages;
    int wpp;              // warps per phase for one row
    int rl;               // rows processed in parallel (warp sets)
    int dpitch;           // D row pitch in floats (odd)
    uint32_t row_bytes, slot_bytes, d_bytes;      // d_bytes: one fold batch's term table
    const float *x;
    float *y;
    int epilogue;
    const float *bias;
    float *residual;
    unsigned *err;
    int use_pdl;
};

// Bounded wait until a shared counter reaches `target` (written by the control warp).
__device__ __forceinline__ bool rows_wait_counter(volatile int *counter, int target)
{
    if (*counter >= target) return true;
    const long long start = clock64();
    while (*counter < target) {
        if (clock64() - start > kWaitBudgetCycles) return false;
        __nanosleep(32);
    }
    return true;
}

template <int FMT, int PH>
__device__ __forceinline__ void rows_load(uint32_t a, uint32_t (&w)[9])
{
    constexpr int NW = FMT == 0 ? 9 : 5;
#pragma unroll
    for (int k = 0; k < NW; ++k) w[k] = lds32(a + 4u * k);
}

// Shared-memory header: full[kRowsMaxStages] | empty[kRowsMaxStages] | dfull[kFoldSlots] | flags.
struct RowsHeader {
    uint64_t *full, *empty, *dfull;
    volatile int *abort_flag, *folded;   // folded = fold batches whose rows are written out
    __device__ explicit RowsHeader(uint8_t *smem)
    {
        full = reinterpret_cast<uint64_t *>(smem);
        empty = full + kRowsMaxStages;
        dfull = empty + kRowsMaxStages;
        abort_flag = reinterpret_cast<volatile int *>(dfull + kFoldSlots);
        folded = abort_flag + 1;
    }
};

// The compute-warp side for one phase (PH = byte offset of the lane's blocks inside their first word).
template <int FMT, int PH>
__device__ __forceinline__ bool rows_compute(const RowsGeo &g, uint8_t *smem, int warp, int lane)
{
    constexpr int BB = blk_bytes(FMT);
    const RowsHeader h(smem);
    const uint32_t slot0 = smem_u32(smem + kRowsHeader);
    float *dtab0 = reinterpret_cast<float *>(smem + kRowsHeader + (size_t)g.stages * g.slot_bytes);

    const int half = g.bpr >> 1;                       // blocks of one phase in a row
    const int cw = warp % g.wpp;                       // column warp within the phase
    const int set = warp / (2 * g.wpp);                // row set
    const int e = cw * 32 + lane;                      // column of this lane within the phase
    const bool valid = e < half && set < g.rl;
    const int ec = min(e, half - 1);
    const int b = 2 * ec + (PH ? 1 : 0);               // block index in the row
    // Byte offset of the word holding the block's first byte, inside a row.
    const uint32_t wofs = (uint32_t)(b * BB - PH);

    float4 xv[8];
    {
        const float4 *xb = reinterpret_cast<const float4 *>(g.x) + (size_t)b * 8;
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[q] = xb[q];
    }

    const int row0 = blockIdx.x * g.rc;
    const int nrows_cta = min(g.rc, g.rows - row0);
    const int nst = (nrows_cta + g.rs - 1) / g.rs;      // stages of this CTA
    for (int i = 0; i < nst; ++i) {
        const int s = i % g.stages;
        if (*h.abort_flag) return false;
        if (!mbar_wait_bounded(&h.full[s], (uint32_t)((i / g.stages) & 1))) return false;
        const int nrows = min(g.rs, nrows_cta - i * g.rs);
        const uint32_t base = slot0 + (uint32_t)s * g.slot_bytes + wofs;
        // Rows of this stage belong to fold batch fb (rs divides kFoldRows); its table is free once
        // batch fb - kFoldSlots has been written out.
        const int fb = (i * g.rs) / kFoldRows, r0 = (i * g.rs) % kFoldRows;
        float *dtab = dtab0 + (size_t)(fb % kFoldSlots) * kFoldRows * g.dpitch;
        bool dready = fb < kFoldSlots;
        // This warp's rows of the stage: set, set + rl, ...; taken two at a time so that the two block
        // terms' dependency chains interleave.
        const int j0 = set < g.rl ? set : nrows;       // warps beyond the row sets only take part in the barriers
        const int nmine = j0 < nrows ? (nrows - j0 + g.rl - 1) / g.rl : 0;
        if (nmine == 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&h.empty[s]);
        }
        for (int m = 0; m < nmine; m += 2) {
            const int ja = j0 + m * g.rl, jb = ja + g.rl;
            const bool two = m + 1 < nmine;
            uint32_t wa[9], wb[9];
            rows_load<FMT, PH>(base + (uint32_t)ja * g.row_bytes, wa);
            if (two) rows_load<FMT, PH>(base + (uint32_t)jb * g.row_bytes, wb);
            if (m + 2 >= nmine) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&h.empty[s]);  // this warp is done reading the slot
            }
            float ta, tb = 0.0f;
            if (two) {
                ta = block_term<FMT, PH>(wa, xv);
                tb = block_term<FMT, PH>(wb, xv);
            } else {
                ta = block_term<FMT, PH>(wa, xv);
            }
            if (!dready) {
                if (!rows_wait_counter(h.folded, fb - kFoldSlots + 1)) return false;
                dready = true;
            }
            if (valid) {
                dtab[(r0 + ja) * g.dpitch + (PH ? half : 0) + e] = ta;
                if (two) dtab[(r0 + jb) * g.dpitch + (PH ? half : 0) + e] = tb;
            }
        }
        // Last stage of the fold batch (or of the CTA): this warp's terms of the batch are written.
        if (r0 + g.rs >= kFoldRows || i == nst - 1) {
            // Every warp, with rows in the batch or not, arrives only once batch fb - kFoldSlots has been
            // added in: dfull[fb % kFoldSlots] is then in batch fb's phase, never in an earlier batch's.
            if (!dready && !rows_wait_counter(h.folded, fb - kFoldSlots + 1)) return false;
            __syncwarp();
            if (lane == 0) mbar_arrive(&h.dfull[fb % kFoldSlots]);
        }
    }
    return true;
}

template <int FMT>
__global__ void __launch_bounds__(kRowsThreads, 2) gemv_rows_kernel(const RowsGeo g)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const RowsHeader h(smem);
    uint8_t *slot0 = smem + kRowsHeader;
    const int S = g.stages;
    const int row0 = blockIdx.x * g.rc;
    const int nrows_cta = min(g.rc, g.rows - row0);
    const int nst = (nrows_cta + g.rs - 1) / g.rs;      // stages of this CTA
    const int nfb = (nrows_cta + kFoldRows - 1) / kFoldRows;   // fold batches of this CTA

    if (tid == 0) {
        *h.abort_flag = 0;
        *h.folded = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&h.full[s], 1);
            mbar_init(&h.empty[s], kRowsWarps);
        }
        for (int s = 0; s < kFoldSlots; ++s) mbar_init(&h.dfull[s], kRowsWarps);
        fence_mbar_init();
    }
    __syncthreads();

    const bool producer = warp == kRowsWarps + 1;
    auto issue = [&](int i) {
        const int s = i % S;
        const int nrows = min(g.rs, nrows_cta - i * g.rs);
        const uint32_t bytes = (uint32_t)nrows * g.row_bytes;
        mbar_expect_tx(&h.full[s], bytes);
        bulk_g2s(slot0 + (size_t)s * g.slot_bytes,
                 g.payload + ((size_t)row0 + (size_t)i * g.rs) * g.row_bytes, bytes, &h.full[s]);
    };
    // Weights never depend on the previous kernel: start streaming them before the PDL wait.
    const int first = min(S, nst);
    if (producer && lane == 0)
        for (int i = 0; i < first; ++i) issue(i);
    if (g.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    if (producer) {
        // Re-arm each slot once every compute warp has read its words.
        if (lane == 0) {
            int i = 0;
            for (; i + S < nst; ++i) {
                if (*h.abort_flag || !mbar_wait_bounded(&h.empty[i % S], (uint32_t)((i / S) & 1))) {
                    atomicOr(g.err, kDevErrTimeout);
                    *h.abort_flag = 1;
                    break;
                }
                issue(i + S);
            }
            if (*h.abort_flag) {
                // Let the copies already issued land before the CTA's shared memory goes away.
                const int last = min(i + S, nst) - 1;
                for (int k = max(0, last - S + 1); k <= last; ++k)
                    mbar_wait_bounded(&h.full[k % S], (uint32_t)((k / S) & 1));
            }
        }
        return;
    }

    if (warp != 0) {
        const int cwarp = warp - 1;
        const int ph = (cwarp / g.wpp) & 1;
        const bool ok = ph == 0 ? rows_compute<FMT, 0>(g, smem, cwarp, lane) : rows_compute<FMT, 2>(g, smem, cwarp, lane);
        if (!ok) {
            if (lane == 0) atomicOr(g.err, kDevErrTimeout);
            *h.abort_flag = 1;
        }
        return;
    }

    // Fold warp (warp 0, the oldest of its scheduler, so its dependent adds are not starved): one lane
    // per row of a batch adds the row's block terms left to right (QuantizedMatVec.cs:300-365) and
    // writes the row's output with the epilogue.
    const int half = g.bpr >> 1;
    const float *dtab0 = reinterpret_cast<const float *>(slot0 + (size_t)S * g.slot_bytes);
    for (int fb = 0; fb < nfb; ++fb) {
        if (*h.abort_flag) break;
        if (!mbar_wait_bounded(&h.dfull[fb % kFoldSlots], (uint32_t)((fb / kFoldSlots) & 1))) {
            if (lane == 0) atomicOr(g.err, kDevErrTimeout);
            *h.abort_flag = 1;
            break;
        }
        const int nrows = min(kFoldRows, nrows_cta - fb * kFoldRows);
        if (lane < nrows) {
            // Block 2c is even[c], block 2c + 1 is odd[c].
            const float *even = dtab0 + ((size_t)(fb % kFoldSlots) * kFoldRows + lane) * g.dpitch, *odd = even + half;
            float acc = 0.0f;
            int c = 0;
#pragma unroll 2
            for (; c + 8 <= half; c += 8) {
                float v[16];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    v[2 * q] = even[c + q];
                    v[2 * q + 1] = odd[c + q];
                }
#pragma unroll
                for (int q = 0; q < 16; ++q) acc = fadd(acc, v[q]);
            }
            if (c < half) {                    // half is a multiple of 4
                float v[8];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v[2 * q] = even[c + q];
                    v[2 * q + 1] = odd[c + q];
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) acc = fadd(acc, v[q]);
            }
            const int grow = row0 + fb * kFoldRows + lane;
            if (g.epilogue == kEpiBias) acc = fadd(acc, g.bias[grow]);
            if (g.epilogue == kEpiResidual) {
                acc = fadd(g.residual[grow], acc);
                g.residual[grow] = acc;
            }
            g.y[grow] = acc;
        }
        __syncwarp();
        if (lane == 0) *h.folded = fb + 1;
    }
}

template <int FMT>
cudaError_t launch_rows(const RowsGeo &g, const DecodePlan &plan, cudaStream_t stream)
{
    auto kern = gemv_rows_kernel<FMT>;
    static size_t configured = 48 * 1024;
    if (plan.smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
        if (e != cudaSuccess) return e;
        configured = plan.smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kRowsThreads);
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

DecodePlan plan_gemv_rows(const GemvArgs &a, int sm_count, size_t smem_limit)
{
    DecodePlan p = {};
    if ((a.format != 0 && a.format != 1) || a.order != SATORI_ORDER_BATCH || a.positions != 1) return p;
    if (a.cols <= 0 || a.cols % 256 != 0 || a.rows <= 0) return p;
    if ((reinterpret_cast<uintptr_t>(a.payload) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return p;
    const int bpr = a.cols / 32, half = bpr / 2;
    const int wpp = (half + 31) / 32;                  // warps per phase for one row
    if (2 * wpp > kRowsWarps) return p;               // more than 8192 columns: chunked kernel
    const size_t row_bytes = (size_t)bpr * blk_bytes(a.format);
    // Rows per stage: a power of two (so that a stage never straddles a fold batch), ~kRowsStageTarget bytes.
    int rs = 1;
    while (rs * 2 <= kRowsMaxStageRows && (size_t)rs * 2 * row_bytes <= kRowsStageTarget) rs *= 2;
    // Two CTAs per SM: twice the copies in flight and twice the compute warps of one CTA.
    const int grid0 = std::min(a.rows, 2 * sm_count);
    const int rc = (a.rows + grid0 - 1) / grid0;
    const int dpitch = bpr + 1;
    const size_t slot = (row_bytes * rs + 127) & ~(size_t)127;
    const size_t dtab = (((size_t)kFoldSlots * kFoldRows * dpitch * 4) + 127) & ~(size_t)127;
    const int nstages = (rc + rs - 1) / rs;
    const size_t fixed = 128 + kRowsHeader + dtab;
    const size_t budget = std::min(smem_limit, kRowsBudget);
    if (budget < fixed + slot) return p;
    int stages = (int)std::min<size_t>(kRowsMaxStages, (budget - fixed) / slot);
    stages = std::min(stages, std::max(nstages, 1));
    if (stages < 1 || (stages < 2 && nstages > 1)) return p;
    p.ok = 1;
    p.kind = 1;
    p.rc = rc;
    p.grid = (a.rows + rc - 1) / rc;
    p.stages = stages;
    p.nchunks = nstages;
    p.rs = rs;
    p.smem = fixed + stages * slot;
    return p;
}

cudaError_t launch_gemv_rows(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream)
{
    if (!plan.ok || plan.kind != 1) return cudaErrorInvalidValue;
    const int bpr = a.cols / 32;
    RowsGeo g;
    g.payload = a.payload;
    g.rows = a.rows;
    g.bpr = bpr;
    g.rc = plan.rc;
    g.rs = plan.rs;
    g.stages = plan.stages;
    g.nstages = plan.nchunks;
    g.wpp = ((bpr / 2) + 31) / 32;
    g.rl = kRowsWarps / (2 * g.wpp);
    g.dpitch = bpr + 1;
    g.row_bytes = (uint32_t)((size_t)bpr * blk_bytes(a.format));
    g.slot_bytes = (uint32_t)((((size_t)g.row_bytes * g.rs) + 127) & ~(size_t)127);
    g.d_bytes = (uint32_t)((size_t)kFoldRows * g.dpitch * 4);
    g.x = a.x;
    g.y = a.y;
    g.epilogue = a.epilogue;
    g.bias = a.bias;
    g.residual = a.residual;
    g.err = a.err;
    g.use_pdl = a.use_pdl;
    return a.format == 0 ? launch_rows<0>(g, plan, stream) : launch_rows<1>(g, plan, stream);
}

}  // namespace satori
