// gemv_rows.cu -- decode-order MatVec of one position, GGUF Q8_0 / Q4_0, rows up to 24576 columns.
//
// Same arithmetic as gemv_decode.cu (QuantizedMatVec.ExecuteBatchFloat -> ExecuteBatchRows -> Dot,
// QuantizedMatVec.cs:221-365, one position): per row a left-to-right FP32 sum over blocks of one
// block term each (qblock.cuh), bit-identical to the reference.
//
// Shapes of the same kernel (cols % 256 == 0):
//  * up to 8192 columns: 8 compute warps, one block column per lane, two CTAs per SM;
//  * up to 20480 columns: 12, 16 or 20 compute warps (as many as cover a row), one block column per
//    lane, one CTA per SM;
//  * up to 24576 columns: 12 compute warps, two block columns per lane, one CTA per SM.
//
// Layout and data movement:
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

constexpr int kFoldSlots = 2;                          // term tables (fold batches in flight)
constexpr int kRowsMaxStages = 16;
constexpr int kRowsMaxStageRows = 32;                  // one control lane per row of a stage
constexpr int kRowsHeader = 384;
constexpr size_t kRowsStageTarget = 40 * 1024;         // bytes of weights per stage (narrow shape)
constexpr size_t kRowsStageTargetWide = 32 * 1024;     // wide shapes: at least two rows of 10 KB
constexpr size_t kRowsBudget = 110 * 1024;             // two CTAs per SM: the next kernel starts early
constexpr size_t kRowsBudgetWide = 200 * 1024;         // one CTA per SM
constexpr size_t kRowsFoldBudget = 40 * 1024;          // term tables of the wide shapes

constexpr int rows_threads(int cw) { return (cw + 2) * 32; }   // + fold warp (0) + producer warp (cw + 1)

struct RowsGeo {
    const uint8_t *payload;
    int rows, bpr, rc, rs, stages, nstages;
    int wpp;              // warps per phase for one row
    int rl;               // rows processed in parallel (warp sets)
    int fold_rows;        // rows per fold batch (one fold lane per row; a multiple of rs)
    int dpitch;           // D row pitch in floats (odd)
    uint32_t row_bytes, slot_bytes, d_bytes;      // d_bytes: one fold batch's term table
    int d_floats;                                  // d_bytes / 4
    const float *x;
    float *y;
    int epilogue;
    const float *bias;
    float *residual;
    unsigned *err;
    int use_pdl;
    const float *norm_w;  // non-null: RmsNorm x (TransformerOps.RmsNorm) before the products
    float norm_eps;
    XPush xp;             // sharded step: the epilogue's output also goes to every peer (xchg.cuh)
    XWait xw;             // sharded step: x holds peers' slices; wait for their signals before reading it
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

// The words of one block: plain shared-memory loads, so the compiler schedules them (they stay after
// the stage's mbarrier wait, which is a compiler memory barrier).
template <int FMT, int PH>
__device__ __forceinline__ void rows_load(const uint8_t *a, uint32_t (&w)[9])
{
    constexpr int NW = FMT == 0 ? 9 : 5;
    const uint32_t *p = reinterpret_cast<const uint32_t *>(a);
#pragma unroll
    for (int k = 0; k < NW; ++k) w[k] = p[k];
}

// Shared-memory header: full[kRowsMaxStages] | empty[kRowsMaxStages] | dfull[kFoldSlots] | flags.
struct RowsHeader {
    uint64_t *full, *empty, *dfull;
    volatile int *abort_flag, *folded;   // folded = fold batches whose rows are written out
    double *red;                         // the RmsNorm's eight warp sums
    __device__ explicit RowsHeader(uint8_t *smem)
    {
        full = reinterpret_cast<uint64_t *>(smem);
        empty = full + kRowsMaxStages;
        dfull = empty + kRowsMaxStages;
        abort_flag = reinterpret_cast<volatile int *>(dfull + kFoldSlots);
        folded = abort_flag + 1;
        red = reinterpret_cast<double *>(dfull + kFoldSlots + 1);
    }
};
static_assert((2 * kRowsMaxStages + kFoldSlots + 1 + 8) * 8 <= kRowsHeader, "rows header");

// The compute-warp side for one phase (PH = byte offset of the lane's blocks inside their first word).
// A lane owns NB block columns of its phase: e_k = (k * wpp + column warp) * 32 + lane.
template <int FMT, int PH, int NB, int CW>
__device__ __forceinline__ bool rows_compute(const RowsGeo &g, uint8_t *smem, int warp, int lane)
{
    constexpr int BB = blk_bytes(FMT);
    const RowsHeader h(smem);
    const uint8_t *slot0 = smem + kRowsHeader;
    float *dtab0 = reinterpret_cast<float *>(smem + kRowsHeader + (size_t)g.stages * g.slot_bytes);

    const int half = g.bpr >> 1;                       // blocks of one phase in a row
    const int cw = warp % g.wpp;                       // column warp within the phase
    const int set = warp / (2 * g.wpp);                // row set
    int e[NB];                                         // columns of this lane within the phase
    bool valid[NB];
    uint32_t wofs[NB];                                 // byte offset of the word holding the block's first byte
    float4 xv[NB][8];
    const double scale = g.norm_w ? rms_scale(h.red, g.bpr * 32, g.norm_eps) : 0.0;
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        e[k] = (k * g.wpp + cw) * 32 + lane;
        valid[k] = e[k] < half && set < g.rl;
        const int b = 2 * min(e[k], half - 1) + (PH ? 1 : 0);   // block index in the row
        wofs[k] = (uint32_t)(b * BB - PH);
        const float4 *xb = reinterpret_cast<const float4 *>(g.x) + (size_t)b * 8;
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[k][q] = xb[q];
        if (g.norm_w) {
            const float4 *wb = reinterpret_cast<const float4 *>(g.norm_w) + (size_t)b * 8;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 w4 = wb[q];
                xv[k][q] = make_float4(rms_apply(xv[k][q].x, scale, w4.x), rms_apply(xv[k][q].y, scale, w4.y),
                                       rms_apply(xv[k][q].z, scale, w4.z), rms_apply(xv[k][q].w, scale, w4.w));
            }
        }
    }

    int dcol[NB];                                      // the lane's columns in a term-table row
#pragma unroll
    for (int k = 0; k < NB; ++k) dcol[k] = (PH ? half : 0) + e[k];

    const int row0 = blockIdx.x * g.rc;
    const int nrows_cta = min(g.rc, g.rows - row0);
    const int nst = (nrows_cta + g.rs - 1) / g.rs;      // stages of this CTA
    // This warp's rows of a stage: set, set + rl, ...; warps beyond the row sets only take part in the
    // barriers.  Every stage but the last is full (rs rows).
    const int j0 = set < g.rl ? set : g.rs;
    const int nfull = j0 < g.rs ? (g.rs - j0 + g.rl - 1) / g.rl : 0;
    // Ring position and fold batch advance by counting: no division in the stage loop.
    int s = 0, fb = 0, r0 = 0;
    uint32_t par = 0;
    for (int i = 0; i < nst; ++i) {
        if (*h.abort_flag) return false;
        if (!mbar_wait_bounded(&h.full[s], par)) return false;
        const bool last = i == nst - 1;
        const int nrows = last ? nrows_cta - i * g.rs : g.rs;
        const uint8_t *base = slot0 + (size_t)s * g.slot_bytes;
        // Rows of this stage belong to fold batch fb (rs divides fold_rows); its table is free once
        // batch fb - kFoldSlots has been written out.
        float *dtab = dtab0 + (fb & (kFoldSlots - 1)) * g.d_floats + r0 * g.dpitch;
        bool dready = fb < kFoldSlots;
        const int nmine = !last ? nfull : (j0 < nrows ? (nrows - j0 + g.rl - 1) / g.rl : 0);
        if (nmine == 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&h.empty[s]);
        }
        // One block column per lane: two rows at a time; several columns: one row at a time.
        constexpr int RP = NB == 1 ? 2 : 1;
        for (int m = 0; m < nmine; m += RP) {
            const int ja = j0 + m * g.rl, jb = ja + g.rl;
            const bool two = RP == 2 && m + 1 < nmine;
            uint32_t w[RP][NB][9];
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                rows_load<FMT, PH>(base + (size_t)ja * g.row_bytes + wofs[k], w[0][k]);
                if (RP == 2 && two) rows_load<FMT, PH>(base + (size_t)jb * g.row_bytes + wofs[k], w[RP - 1][k]);
            }
            if (m + RP >= nmine) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&h.empty[s]);  // this warp is done reading the slot
            }
            float t[RP][NB];
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                t[0][k] = block_term<FMT, PH>(w[0][k], xv[k]);
                if (RP == 2) t[RP - 1][k] = two ? block_term<FMT, PH>(w[RP - 1][k], xv[k]) : 0.0f;
            }
            if (!dready) {
                if (!rows_wait_counter(h.folded, fb - kFoldSlots + 1)) return false;
                dready = true;
            }
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                if (!valid[k]) continue;
                dtab[ja * g.dpitch + dcol[k]] = t[0][k];
                if (RP == 2 && two) dtab[jb * g.dpitch + dcol[k]] = t[RP - 1][k];
            }
        }
        // Last stage of the fold batch (or of the CTA): this warp's terms of the batch are written.
        if (r0 + g.rs >= g.fold_rows || last) {
            // Every warp, with rows in the batch or not, arrives only once batch fb - kFoldSlots has been
            // added in: dfull[fb % kFoldSlots] is then in batch fb's phase, never in an earlier batch's.
            if (!dready && !rows_wait_counter(h.folded, fb - kFoldSlots + 1)) return false;
            __syncwarp();
            if (lane == 0) mbar_arrive(&h.dfull[fb & (kFoldSlots - 1)]);
        }
        if (++s == g.stages) {
            s = 0;
            par ^= 1u;
        }
        r0 += g.rs;
        if (r0 == g.fold_rows) {
            r0 = 0;
            ++fb;
        }
    }
    return true;
}

template <int FMT, int CW, int NB>
__global__ void __launch_bounds__(rows_threads(CW), CW == 8 ? 2 : 1) gemv_rows_kernel(const RowsGeo g)
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
    const int nfb = (nrows_cta + g.fold_rows - 1) / g.fold_rows;   // fold batches of this CTA

    if (tid == 0) {
        *h.abort_flag = 0;
        *h.folded = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&h.full[s], 1);
            mbar_init(&h.empty[s], CW);
        }
        for (int s = 0; s < kFoldSlots; ++s) mbar_init(&h.dfull[s], CW);
        fence_mbar_init();
    }
    __syncthreads();

    const bool producer = warp == CW + 1;
    auto issue = [&](int i, int s) {   // stage i into ring slot s
        const int nrows = min(g.rs, nrows_cta - i * g.rs);
        const uint32_t bytes = (uint32_t)nrows * g.row_bytes;
        mbar_expect_tx(&h.full[s], bytes);
        bulk_g2s(slot0 + (size_t)s * g.slot_bytes,
                 g.payload + ((size_t)row0 + (size_t)i * g.rs) * g.row_bytes, bytes, &h.full[s]);
    };
    // Weights never depend on the previous kernel: start streaming them before the PDL wait.
    const int first = min(S, nst);
    if (producer && lane == 0)
        for (int i = 0; i < first; ++i) issue(i, i);
    if (g.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    if (g.xw.world) {
        // Sharded step: x holds slices the peers store; wait for all of them before anyone reads it (the
        // acquire load of the peers' flags, then the barrier, orders every thread's later loads of x).
        if (tid == 0) xwait_peers(g.xw, g.err);
        __syncthreads();
    }
    if (g.norm_w) {
        // The RmsNorm scale of x: warps 0..7 form the fixed-order sum, every thread reads it back.
        if (tid < 256) rms_partial(g.x, g.bpr * 32, tid, h.red);
        __syncthreads();
    }

    if (producer) {
        // Re-arm each slot once every compute warp has read its words.
        if (lane == 0) {
            int i = 0, si = 0;
            uint32_t par = 0;
            for (; i + S < nst; ++i) {
                if (*h.abort_flag || !mbar_wait_bounded(&h.empty[si], par)) {
                    atomicOr(g.err, kDevErrTimeout);
                    *h.abort_flag = 1;
                    break;
                }
                issue(i + S, si);
                if (++si == S) {
                    si = 0;
                    par ^= 1u;
                }
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
        const bool ok = ph == 0 ? rows_compute<FMT, 0, NB, CW>(g, smem, cwarp, lane)
                                : rows_compute<FMT, 2, NB, CW>(g, smem, cwarp, lane);
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
        const int nrows = min(g.fold_rows, nrows_cta - fb * g.fold_rows);
        if (lane < nrows) {
            // Block 2c is even[c], block 2c + 1 is odd[c].
            const float *even = dtab0 + ((size_t)(fb % kFoldSlots) * g.fold_rows + lane) * g.dpitch, *odd = even + half;
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
            const int grow = row0 + fb * g.fold_rows + lane;
            if (g.epilogue == kEpiSwiGlu) {
                // Rows 2i and 2i + 1 are gate row i and up row i; batches and CTAs start on even rows.
                const float up = __shfl_down_sync(nrows == 32 ? 0xFFFFFFFFu : (1u << nrows) - 1u, acc, 1);
                if ((lane & 1) == 0) {
                    const float a = swiglu_value(acc, up);
                    g.y[grow >> 1] = a;
                    if (g.xp.world) xpush_value(g.xp, grow >> 1, a);
                }
            } else {
                if (g.epilogue == kEpiBias) acc = fadd(acc, g.bias[grow]);
                if (g.epilogue == kEpiResidual) {
                    acc = fadd(g.residual[grow], acc);
                    g.residual[grow] = acc;
                }
                g.y[grow] = acc;
                // The gathered buffer is the residual stream for a residual epilogue, else y.
                if (g.xp.world) xpush_value(g.xp, grow, acc);
            }
        }
        __syncwarp();
        if (lane == 0) *h.folded = fb + 1;
    }
    if (g.xp.world) {
        __threadfence_system();   // this lane's peer stores, before the CTA counts as done
        __syncwarp();
        if (lane == 0) xpush_finish(g.xp);
    }
}

template <int FMT, int CW, int NB>
cudaError_t launch_rows(const RowsGeo &g, const DecodePlan &plan, cudaStream_t stream)
{
    auto kern = gemv_rows_kernel<FMT, CW, NB>;
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(kern), plan.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(rows_threads(CW));
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
    // Shape: compute warps and block columns per lane (see the top of the file).
    int cw, nb = 1;
    if (half <= 4 * 32)
        cw = 8;
    else if (half <= 6 * 32)
        cw = 12;
    else if (half <= 8 * 32)
        cw = 16;
    else if (half <= 10 * 32)
        cw = 20;
    else if (half <= 2 * 6 * 32)
        cw = 12, nb = 2;
    else
        return p;                                      // wider rows: chunked kernel
    const bool wide = cw != 8;
    const size_t row_bytes = (size_t)bpr * blk_bytes(a.format);
    // Rows per stage: a power of two (so that a stage never straddles a fold batch), ~kRowsStageTarget bytes.
    int rs = 1;
    const size_t target = wide ? kRowsStageTargetWide : kRowsStageTarget;
    while (rs * 2 <= kRowsMaxStageRows && (size_t)rs * 2 * row_bytes <= target) rs *= 2;
    const int dpitch = bpr + 1;
    // Rows per fold batch: 32 (one per fold lane) unless the two term tables would not fit their budget.
    int fold = 32;
    while (wide && fold > rs && (size_t)kFoldSlots * fold * dpitch * 4 > kRowsFoldBudget) fold /= 2;
    // Two CTAs per SM for the narrow shape: twice the copies in flight and twice the compute warps.
    const int grid0 = std::min(a.rows, (wide ? 1 : 2) * sm_count);
    int rc = (a.rows + grid0 - 1) / grid0;
    if (a.epilogue == kEpiSwiGlu) {
        if (a.rows % 2) return p;
        rc += rc & 1;                                  // a gate/up row pair never straddles two CTAs
    }
    const size_t slot = (row_bytes * rs + 127) & ~(size_t)127;
    const size_t dtab = (((size_t)kFoldSlots * fold * dpitch * 4) + 127) & ~(size_t)127;
    const int nstages = (rc + rs - 1) / rs;
    const size_t fixed = 128 + kRowsHeader + dtab;
    const size_t budget = std::min(smem_limit, wide ? kRowsBudgetWide : kRowsBudget);
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
    p.cw = cw;
    p.nb = nb;
    p.fold = fold;
    p.smem = fixed + stages * slot;
    return p;
}

bool gemv_rows_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit)
{
    GemvArgs a = {};
    a.rows = rows;
    a.cols = cols;
    a.format = format;
    a.order = SATORI_ORDER_BATCH;
    a.positions = 1;
    a.epilogue = epilogue;
    // Device allocations and the session's vectors are 256-byte aligned; stand-ins with that alignment.
    a.payload = reinterpret_cast<const uint8_t *>(uintptr_t(256));
    a.x = reinterpret_cast<const float *>(uintptr_t(256));
    return plan_gemv_rows(a, sm_count, smem_limit).ok != 0;
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
    // Narrow shape: as few warps per phase as cover the row, the others take further rows; wide shapes:
    // every warp on the same row.
    g.wpp = plan.cw == 8 ? ((bpr / 2) + 31) / 32 : plan.cw / 2;
    static_assert(kRowsMaxStageRows <= 32, "one control lane per stage row");
    g.rl = plan.cw / (2 * g.wpp);
    g.fold_rows = plan.fold;
    g.dpitch = bpr + 1;
    g.row_bytes = (uint32_t)((size_t)bpr * blk_bytes(a.format));
    g.slot_bytes = (uint32_t)((((size_t)g.row_bytes * g.rs) + 127) & ~(size_t)127);
    g.d_bytes = (uint32_t)((size_t)plan.fold * g.dpitch * 4);
    g.d_floats = (int)(g.d_bytes / 4);
    g.x = a.x;
    g.y = a.y;
    g.epilogue = a.epilogue;
    g.bias = a.bias;
    g.residual = a.residual;
    g.err = a.err;
    g.use_pdl = a.use_pdl;
    g.norm_w = a.norm_w;
    g.norm_eps = a.norm_eps;
    g.xp = a.xp;
    g.xw = a.xw;
    const bool q8 = a.format == 0;
    if (plan.nb == 2) return q8 ? launch_rows<0, 12, 2>(g, plan, stream) : launch_rows<1, 12, 2>(g, plan, stream);
    switch (plan.cw) {
    case 8: return q8 ? launch_rows<0, 8, 1>(g, plan, stream) : launch_rows<1, 8, 1>(g, plan, stream);
    case 12: return q8 ? launch_rows<0, 12, 1>(g, plan, stream) : launch_rows<1, 12, 1>(g, plan, stream);
    case 16: return q8 ? launch_rows<0, 16, 1>(g, plan, stream) : launch_rows<1, 16, 1>(g, plan, stream);
    default: return q8 ? launch_rows<0, 20, 1>(g, plan, stream) : launch_rows<1, 20, 1>(g, plan, stream);
    }
}

}  // namespace satori
