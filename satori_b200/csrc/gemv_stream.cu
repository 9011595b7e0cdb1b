// gemv_stream.cu -- decode-order MatVec of one position, GGUF Q8_0 / Q4_0, for the row widths of the
// decode configurations (1536, 3584, 4096, 8960 and 18944 columns), with the row width a compile-time
// constant.
//
// Arithmetic: QuantizedMatVec.ExecuteBatchFloat -> ExecuteBatchRows -> Dot (QuantizedMatVec.cs:221-365)
// for one position: per row a left-to-right FP32 sum over the row's blocks of one block term each
// (qblock.cuh), bit-identical to the reference, exactly like gemv_rows.cu.
//
// What the fixed width buys: every shared-memory offset inside a stage (row r of a stage, word k of a
// block, row r of a term table) is an immediate, every loop over rows and blocks is unrolled, and the
// stage loop carries only a ring position, a batch position and two mbarrier waits.  A block term then
// costs the term's own instructions plus a handful.
//
// Data movement and roles (one wave of CTAs, each owning a contiguous range of rows, i.e. one
// contiguous byte range of the payload):
//  * producer warp: streams the CTA's rows in stages of R whole rows, one 1-D bulk copy (TMA unicast)
//    per stage, into a ring of S slots; the first S stages are requested before the programmatic-launch
//    wait (weights never depend on the previous kernel), later ones as slots are released;
//  * compute warps: lane (warp, lane) owns one block column of one phase (even or odd block index, so
//    the block's byte offset mod 4 is a constant) and keeps that block's 32 activations in registers
//    for the whole kernel; per stage it loads its words of RPW rows, releases the slot, computes RPW
//    block terms and stores them into a term table D[row][even blocks | odd blocks];
//  * fold warp: per fold batch (FR rows, one lane per row) adds a row's terms in block order and writes
//    the row's output through the epilogue (bias, residual add, or SwiGLU of an interleaved gate/up
//    row pair), and optionally stores it into every peer's copy (sharded step).
// Hand-offs are mbarriers in both directions: full/empty per ring slot, dfull/dfree per term table.
// Every wait is bounded; an expired wait records kDevErrTimeout and the CTA winds down.
#include "common.cuh"
#include "gemv.cuh"
#include "qblock.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kStMaxStages = 12;
constexpr int kStHeader = 512;
constexpr int kStTables = 2;                      // term tables (fold batches in flight)

// Compile-time geometry of one instantiation.
template <int FMT, int NB, int CW, int RPW>
struct StGeo {
    static constexpr int BB = blk_bytes(FMT);
    static constexpr int RB = NB * BB;                       // row bytes (a multiple of 16)
    static constexpr int HALF = NB / 2;                      // blocks of one phase
    static constexpr int WPP = (HALF + 31) / 32;             // warps per phase of one row
    static constexpr int WPR = 2 * WPP;                      // warps per row
    static constexpr int RL = CW / WPR;                      // rows in parallel (row sets)
    static constexpr int R = RL * RPW;                       // rows per stage
    static constexpr int SLOT = ((R * RB + 16) + 127) / 128 * 128;   // slot stride (reads may run 2 bytes past)
    static constexpr int PITCH = NB + 4;                     // term-table row (floats): 16-byte rows, no conflicts
    static constexpr int NW = FMT == 0 ? 9 : 5;              // words a block term reads
    static_assert(NB % 8 == 0 && CW % WPR == 0 && RL >= 1, "geometry");
    static_assert(R <= 32, "one fold lane per row of a stage");
};

struct StreamArgs {
    const uint8_t *payload;
    int rows, rc, stages, fold_stages;   // rows per CTA, ring slots, stages per fold batch
    const float *x;
    float *y;
    int epilogue;
    const float *bias;
    float *residual;
    unsigned *err;
    int use_pdl;
    const float *norm_w;
    float norm_eps;
    XPush xp;
    XWait xw;
    const uint8_t *next;      // head of the next MatVec's weights, prefetched into L2 in the tail
    uint32_t next_chunk;      // bytes of it per CTA (a multiple of 16)
    size_t next_bytes;
};

struct StHeader {
    uint64_t *full, *empty, *dfull, *dfree, *xready;
    double *red;
    volatile int *abort_flag;
    __device__ explicit StHeader(uint8_t *smem)
    {
        full = reinterpret_cast<uint64_t *>(smem);
        empty = full + kStMaxStages;
        dfull = empty + kStMaxStages;
        dfree = dfull + kStTables;
        xready = dfree + kStTables;
        red = reinterpret_cast<double *>(xready + 1);
        abort_flag = reinterpret_cast<volatile int *>(red + 8);
    }
};
static_assert((2 * kStMaxStages + 2 * kStTables + 1 + 8) * 8 + 4 <= kStHeader, "stream header");

__device__ __forceinline__ bool st_wait(uint64_t *bar, uint32_t parity, const StHeader &h, unsigned *err)
{
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicOr(err, kDevErrTimeout);
    *h.abort_flag = 1;
    return false;
}

// The fused RmsNorm of x exists for the hidden widths only (the inputs of q/k/v and gate/up); the wide
// variants (ffn widths, inputs of ffn_down) leave it out and keep their registers for the block terms.
template <int NB>
__device__ __forceinline__ bool st_norm(const StreamArgs &a)
{
    return NB <= 128 && a.norm_w != nullptr;
}

// Where the compute warps stage x (and the norm weights): the last slots of the ring, which receive no
// weights before every lane holds its activations.  Chunk q of block k sits at chunk q ^ ((k >> 1) & 7)
// of the block, so the eight lanes of a shared-memory wavefront (blocks two apart) read distinct banks.
template <int FMT, int NB, int CW, int RPW>
__device__ __forceinline__ float4 *st_staged_x(const StreamArgs &a, const uint8_t *ring)
{
    using G = StGeo<FMT, NB, CW, RPW>;
    const int xslots = (NB * 128 * (st_norm<NB>(a) ? 2 : 1) + G::SLOT - 1) / G::SLOT;
    return reinterpret_cast<float4 *>(const_cast<uint8_t *>(ring) + (size_t)(a.stages - xslots) * G::SLOT);
}

__device__ __forceinline__ int st_swz(int chunk)
{
    const int k = chunk >> 3;
    return k * 8 + ((chunk & 7) ^ ((k >> 1) & 7));
}

// The compute warps copy x (and the norm weights) into the staging area with coalesced 16-byte loads:
// a lane loading its own block directly would make every warp load touch 32 lines.
template <int FMT, int NB, int CW, int RPW>
__device__ __forceinline__ void st_stage_x(const StreamArgs &a, const uint8_t *ring, int ct)
{
    float4 *xs = st_staged_x<FMT, NB, CW, RPW>(a, ring);
    constexpr int NCH = NB * 8;
    for (int i = ct; i < NCH; i += CW * 32) {
        const int dst = st_swz(i);
        xs[dst] = reinterpret_cast<const float4 *>(a.x)[i];
        if (st_norm<NB>(a)) xs[NCH + dst] = reinterpret_cast<const float4 *>(a.norm_w)[i];
    }
}

// rms_partial's sum (the same 256 strided partials and tree, so the same bits) over the staged copy of x.
__device__ __forceinline__ void rms_partial_staged(const float4 *xs, int n, int tid, double *red)
{
    const float *f = reinterpret_cast<const float *>(xs);
    double sum = 0;
    for (int i = tid; i < n; i += 256) {
        const float v = f[st_swz(i >> 2) * 4 + (i & 3)];
        sum = __dadd_rn(sum, __dmul_rn((double)v, (double)v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xFFFFFFFFu, sum, o));
    if ((tid & 31) == 0) red[tid >> 5] = sum;
}

// Compute warp `cw` (0-based) for phase PH.
template <int FMT, int NB, int CW, int RPW, int PH>
__device__ __forceinline__ void st_compute(const StreamArgs &a, uint8_t *smem, int cw, int lane, int nrows_cta,
                                           int table_floats)
{
    using G = StGeo<FMT, NB, CW, RPW>;
    const StHeader h(smem);
    float *dtab = reinterpret_cast<float *>(smem + kStHeader);
    const uint8_t *ring = smem + kStHeader + (size_t)table_floats * 4;

    const int set = cw / G::WPR;
    const int e = (cw % G::WPP) * 32 + lane;                 // column within the phase
    const bool valid = e < G::HALF;
    const int b = 2 * min(e, G::HALF - 1) + (PH ? 1 : 0);    // block index in the row (odd blocks: PH = 2)
    float4 xv[8];
    {
        // x (and the norm weights) were staged into the ring by the compute warps (st_stage_x); each lane
        // reads its block's 32 values from there.
        constexpr int NCH = NB * 8;
        const float4 *xs = st_staged_x<FMT, NB, CW, RPW>(a, ring);
        asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");   // the compute warps only
        const double scale = st_norm<NB>(a) ? rms_scale(h.red, NB * 32, a.norm_eps) : 0.0;
        const int sw = (b >> 1) & 7;
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[q] = xs[b * 8 + (q ^ sw)];
        if (st_norm<NB>(a)) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 w4 = xs[NCH + b * 8 + (q ^ sw)];
                xv[q] = make_float4(rms_apply(xv[q].x, scale, w4.x), rms_apply(xv[q].y, scale, w4.y),
                                    rms_apply(xv[q].z, scale, w4.z), rms_apply(xv[q].w, scale, w4.w));
            }
        }
    }
    // Release the weight copies only once this warp's activations are in registers: the copies overwrite
    // the staged activations, and issued earlier they would also delay the activation loads behind the
    // ring fill.  (Adding the 32 values makes every load complete before the arrival.)
    {
        float all = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) all += (xv[q].x + xv[q].y) + (xv[q].z + xv[q].w);
        asm volatile("" ::"f"(all));
        __syncwarp();
        if (lane == 0) mbar_arrive(h.xready);
    }
    // This lane's word of row 0 (row set `set`) in slot 0, and its term-table column.
    const uint8_t *lrow = ring + set * G::RB + (b * G::BB - PH);
    float *lcol = dtab + set * G::PITCH + (PH ? G::HALF : 0) + e;

    const int nst = (nrows_cta + G::R - 1) / G::R;
    const int FRS = a.fold_stages;
    int s = 0, si = 0, fb = 0;
    uint32_t par = 0;
    for (int i = 0; i < nst; ++i) {
        if (*h.abort_flag) return;
        if (!st_wait(&h.full[s], par, h, a.err)) return;
        const uint8_t *base = lrow + (size_t)s * G::SLOT;
        uint32_t w[RPW][9];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(base + r * G::RL * G::RB);
#pragma unroll
            for (int k = 0; k < G::NW; ++k) w[r][k] = p[k];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&h.empty[s]);             // this warp has read the slot
        float t[RPW];
#pragma unroll
        for (int r = 0; r < RPW; ++r) t[r] = block_term<FMT, PH>(w[r], xv);
        const int k = fb & 1;
        if (si == 0 && fb >= kStTables) {
            // Table k is free once the fold warp has written out batch fb - 2.
            if (!st_wait(&h.dfree[k], (uint32_t)(((fb >> 1) - 1) & 1), h, a.err)) return;
        }
        const int nrows = min(G::R, nrows_cta - i * G::R);
        float *dst = lcol + (size_t)k * (table_floats / kStTables) + si * G::R * G::PITCH;
        if (valid) {
#pragma unroll
            for (int r = 0; r < RPW; ++r)
                if (set + r * G::RL < nrows) dst[r * G::RL * G::PITCH] = t[r];
        }
        if (++si == FRS || i == nst - 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&h.dfull[k]);         // this warp's terms of batch fb are in
            si = 0;
            ++fb;
        }
        if (++s == a.stages) {
            s = 0;
            par ^= 1u;
        }
    }
}

template <int FMT, int NB, int CW, int RPW, int MINB>
__global__ void __launch_bounds__((CW + 2) * 32, MINB) gemv_stream_kernel(const StreamArgs a)
{
    using G = StGeo<FMT, NB, CW, RPW>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const StHeader h(smem);
    const int FR = a.fold_stages * G::R;                     // rows per fold batch
    const int table_floats = kStTables * FR * G::PITCH;
    uint8_t *ring = smem + kStHeader + (size_t)table_floats * 4;
    const int row0 = blockIdx.x * a.rc;
    const int nrows_cta = max(0, min(a.rc, a.rows - row0));
    const int nst = (nrows_cta + G::R - 1) / G::R;
    const int S = a.stages;

    if (tid == 0) {
        *h.abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&h.full[s], 1);
            mbar_init(&h.empty[s], CW);
        }
        for (int k = 0; k < kStTables; ++k) {
            mbar_init(&h.dfull[k], CW);
            mbar_init(&h.dfree[k], 1);
        }
        mbar_init(h.xready, CW);
        fence_mbar_init();
    }
    __syncthreads();

    const bool producer = warp == CW + 1;
    auto issue = [&](int i, int s) {
        const uint32_t bytes = (uint32_t)(min(G::R, nrows_cta - i * G::R) * G::RB);
        mbar_expect_tx(&h.full[s], bytes);
        bulk_g2s(ring + (size_t)s * G::SLOT, a.payload + ((size_t)row0 + (size_t)i * G::R) * G::RB, bytes,
                 &h.full[s]);
    };
    // Weights never depend on the previous kernel: the stages whose slots lie below the activation
    // staging area (the last slots of the ring) are requested before the programmatic-launch wait; the
    // rest follow once every lane holds its activations.
    const int xslots = (NB * 128 * (st_norm<NB>(a) ? 2 : 1) + G::SLOT - 1) / G::SLOT;
    const int early = max(0, min(nst, S - xslots));
    if (producer && lane == 0)
        for (int i = 0; i < early; ++i) issue(i, i);
    if (a.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    if (a.xw.world) {
        if (tid == 0) xwait_peers(a.xw, a.err);
        __syncthreads();
    }
    if (warp >= 1 && warp <= CW) st_stage_x<FMT, NB, CW, RPW>(a, ring, tid - 32);
    if (st_norm<NB>(a)) {
        // The norm's sum of squares reads the staged copy (one pass over global memory instead of two).
        __syncthreads();
        if (tid < 256) rms_partial_staged(st_staged_x<FMT, NB, CW, RPW>(a, ring), NB * 32, tid, h.red);
        __syncthreads();
    }

    if (producer) {
        if (lane != 0) return;
        if (!st_wait(h.xready, 0, h, a.err)) {
            for (int k = 0; k < early; ++k) mbar_wait_bounded(&h.full[k], 0);   // copies land before exit
            return;
        }
        for (int i = early; i < min(S, nst); ++i) issue(i, i);
        int i = S, s = 0;
        uint32_t par = 0;
        for (; i < nst; ++i) {
            if (*h.abort_flag || !st_wait(&h.empty[s], par, h, a.err)) break;
            issue(i, s);
            if (++s == S) {
                s = 0;
                par ^= 1u;
            }
        }
        if (*h.abort_flag) {
            // Copies already issued land before the CTA's shared memory goes away.
            const int last = min(i, nst) - 1;
            for (int k = max(0, last - S + 1); k <= last; ++k) mbar_wait_bounded(&h.full[k % S], (uint32_t)((k / S) & 1));
            return;
        }
        // Once this CTA's last stage has landed, DRAM has room: start the next MatVec's weights (this CTA's
        // share of their head) on their way into L2.
        if (a.next && nst > 0 && mbar_wait_bounded(&h.full[(nst - 1) % S], (uint32_t)(((nst - 1) / S) & 1))) {
            const size_t begin = (size_t)blockIdx.x * a.next_chunk;
            if (begin < a.next_bytes) {
                const size_t end = min(a.next_bytes, begin + a.next_chunk);
                for (size_t o = begin; o < end; o += 65536)
                    bulk_prefetch_l2(a.next + o, (uint32_t)min((size_t)65536, end - o));
            }
        }
        return;
    }

    if (warp != 0) {
        const int cw = warp - 1;
        if (((cw % G::WPR) / G::WPP) == 0)
            st_compute<FMT, NB, CW, RPW, 0>(a, smem, cw, lane, nrows_cta, table_floats);
        else
            st_compute<FMT, NB, CW, RPW, 2>(a, smem, cw, lane, nrows_cta, table_floats);
        return;
    }

    // Fold warp: lane r adds row r of the batch, blocks in order 0, 1, 2, ... (even[c], odd[c]).
    const float *dtab = reinterpret_cast<const float *>(smem + kStHeader);
    const int nfb = (nst + a.fold_stages - 1) / a.fold_stages;
    for (int fb = 0; fb < nfb; ++fb) {
        if (*h.abort_flag) break;
        const int k = fb & 1;
        if (!st_wait(&h.dfull[k], (uint32_t)((fb >> 1) & 1), h, a.err)) break;
        const int nrows = min(FR, nrows_cta - fb * FR);
        if (lane < nrows) {
            const float *row = dtab + (size_t)k * FR * G::PITCH + lane * G::PITCH;
            float acc = 0.0f;
#pragma unroll 4
            for (int c = 0; c < G::HALF; c += 4) {
                const float4 ev = *reinterpret_cast<const float4 *>(row + c);
                const float4 od = *reinterpret_cast<const float4 *>(row + G::HALF + c);
                acc = fadd(acc, ev.x);
                acc = fadd(acc, od.x);
                acc = fadd(acc, ev.y);
                acc = fadd(acc, od.y);
                acc = fadd(acc, ev.z);
                acc = fadd(acc, od.z);
                acc = fadd(acc, ev.w);
                acc = fadd(acc, od.w);
            }
            const int grow = row0 + fb * FR + lane;
            if (a.epilogue == kEpiSwiGlu) {
                // Rows 2i and 2i + 1 are gate row i and up row i; batches and CTAs start on even rows.
                const float up = __shfl_down_sync(nrows == 32 ? 0xFFFFFFFFu : (1u << nrows) - 1u, acc, 1);
                if ((lane & 1) == 0) {
                    const float v = swiglu_value(acc, up);
                    a.y[grow >> 1] = v;
                    if (a.xp.world) xpush_value(a.xp, grow >> 1, v);
                }
            } else {
                if (a.epilogue == kEpiBias) acc = fadd(acc, a.bias[grow]);
                if (a.epilogue == kEpiResidual) {
                    acc = fadd(a.residual[grow], acc);
                    a.residual[grow] = acc;
                }
                a.y[grow] = acc;
                if (a.xp.world) xpush_value(a.xp, grow, acc);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&h.dfree[k]);
    }
    if (a.xp.world) {
        __threadfence_system();
        __syncwarp();
        if (lane == 0) xpush_finish(a.xp);
    }
}

// One instantiation: its kernel and its launch-time constants.
struct StVariant {
    int fmt, nb, cw, rpw, minb;
    int rows_per_stage, slot, pitch;
    void (*kernel)(const StreamArgs);
};

template <int FMT, int NB, int CW, int RPW, int MINB>
constexpr StVariant st_variant()
{
    using G = StGeo<FMT, NB, CW, RPW>;
    return StVariant{FMT, NB, CW, RPW, MINB, G::R, G::SLOT, G::PITCH, gemv_stream_kernel<FMT, NB, CW, RPW, MINB>};
}

// The decode configurations' row widths: 1536 / 8960 (1.5B shape), 3584 / 18944 (7B shape), 4096
// (the MatVec benchmark).
const StVariant kVariants[] = {
    st_variant<0, 48, 8, 4, 2>(),   st_variant<1, 48, 8, 4, 2>(),
    st_variant<0, 112, 8, 4, 2>(),  st_variant<1, 112, 8, 4, 2>(),
    st_variant<0, 128, 8, 4, 2>(),  st_variant<1, 128, 8, 4, 2>(),
    st_variant<0, 280, 20, 2, 1>(), st_variant<1, 280, 20, 2, 1>(),
    st_variant<0, 592, 20, 2, 1>(), st_variant<1, 592, 20, 2, 1>(),
};

const StVariant *find_variant(int fmt, int nb)
{
    for (const StVariant &v : kVariants)
        if (v.fmt == fmt && v.nb == nb) return &v;
    return nullptr;
}

}  // namespace

DecodePlan plan_gemv_stream(const GemvArgs &a, int sm_count, size_t smem_limit)
{
    DecodePlan p = {};
    if ((a.format != 0 && a.format != 1) || a.order != SATORI_ORDER_BATCH || a.positions != 1) return p;
    if (a.cols <= 0 || a.cols % 256 != 0 || a.rows <= 0) return p;
    if ((reinterpret_cast<uintptr_t>(a.payload) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return p;
    const StVariant *v = find_variant(a.format, a.cols / 32);
    if (!v) return p;
    if (a.epilogue == kEpiSwiGlu && (a.rows % 2 || v->rows_per_stage % 2)) return p;
    const size_t budget = std::min(smem_limit, v->minb == 2 ? (size_t)113 * 1024 : (size_t)220 * 1024);
    // Rows per fold batch: up to 32 (one fold lane each), whole stages, two tables within ~40 KB.
    int fold_stages = 32 / v->rows_per_stage;
    while (fold_stages > 1 && (size_t)kStTables * fold_stages * v->rows_per_stage * v->pitch * 4 > 40 * 1024)
        --fold_stages;
    const size_t tables = (size_t)kStTables * fold_stages * v->rows_per_stage * v->pitch * 4;
    const size_t fixed = 128 + kStHeader + tables;
    if (budget < fixed + 2 * (size_t)v->slot) return p;
    const int grid0 = std::max(1, std::min(a.rows / std::max(1, v->rows_per_stage / 2), v->minb * sm_count));
    int rc = (a.rows + grid0 - 1) / grid0;
    if (a.epilogue == kEpiSwiGlu) rc += rc & 1;              // a gate/up row pair stays in one CTA
    const int nst = (rc + v->rows_per_stage - 1) / v->rows_per_stage;
    int stages = (int)std::min<size_t>(kStMaxStages, (budget - fixed) / v->slot);
    stages = std::max(1, std::min(stages, nst));
    // The ring first holds the staged activations (and norm weights): at least that much of it is needed.
    if (a.norm_w && v->nb > 128) return p;                  // no fused norm in the wide variants
    const size_t staged = (size_t)v->nb * 128 * (a.norm_w ? 2 : 1);
    while ((size_t)stages * v->slot < staged && stages < kStMaxStages && fixed + (size_t)(stages + 1) * v->slot <= budget)
        ++stages;
    if ((size_t)stages * v->slot < staged) return p;
    p.ok = 1;
    p.kind = 3;
    p.rc = rc;
    p.grid = (a.rows + rc - 1) / rc;
    p.stages = stages;
    p.nchunks = nst;
    p.rs = v->rows_per_stage;
    p.cw = v->cw;
    p.fold = fold_stages;
    p.smem = fixed + (size_t)stages * v->slot;
    return p;
}

bool gemv_stream_takes(int rows, int cols, int format, int epilogue, int sm_count, size_t smem_limit)
{
    GemvArgs a = {};
    a.rows = rows;
    a.cols = cols;
    a.format = format;
    a.order = SATORI_ORDER_BATCH;
    a.positions = 1;
    a.epilogue = epilogue;
    a.payload = reinterpret_cast<const uint8_t *>(uintptr_t(256));
    a.x = reinterpret_cast<const float *>(uintptr_t(256));
    return plan_gemv_stream(a, sm_count, smem_limit).ok != 0;
}

cudaError_t launch_gemv_stream(const GemvArgs &a, const DecodePlan &plan, cudaStream_t stream)
{
    if (!plan.ok || plan.kind != 3) return cudaErrorInvalidValue;
    const StVariant *v = find_variant(a.format, a.cols / 32);
    if (!v) return cudaErrorInvalidValue;
    StreamArgs g;
    g.payload = a.payload;
    g.rows = a.rows;
    g.rc = plan.rc;
    g.stages = plan.stages;
    g.fold_stages = plan.fold;
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
    g.next = nullptr;
    g.next_chunk = 0;
    g.next_bytes = 0;
    if (a.next_payload && a.next_bytes >= 16) {
        // At most 32 MB of the next weights (a fraction of L2), split evenly over the CTAs.
        g.next = a.next_payload;
        g.next_bytes = std::min(a.next_bytes, (size_t)32 << 20) & ~(size_t)15;
        const size_t chunk = (g.next_bytes + plan.grid - 1) / plan.grid;
        g.next_chunk = (uint32_t)((chunk + 15) & ~(size_t)15);
    }
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(v->kernel), plan.smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3((v->cw + 2) * 32);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, v->kernel, g);
}

}  // namespace satori
