// gemv_ternary.cu -- ternary MatVec in the AVX2 order, for Ternary2 (2-bit codes) and the ternary bitplane
// layout (STB1: a positive and a negative bit plane per block), streamed row by row.
//
// Arithmetic (Ternary2Avx2Kernel.Execute, src/Satori.Core/Ternary2Avx2Kernel.cs:10-56, and
// TernaryBitplaneAvx2Kernel.Execute, src/Satori.Core/TernaryBitplaneAvx2Kernel.cs:18-52, which compute the
// same thing from the two layouts): per block, eight FP32 lanes; lane l adds weight l, l+8, l+16, ... of
// the block as +x, -x or +0 in that order; then the fixed horizontal sum ((a0+a4)+(a2+a6)) +
// ((a1+a5)+(a3+a7)); the row's total adds partial * scale block by block.  A lane's running sum starts at
// +0 and, in round-to-nearest, can never become -0, so adding +0 for a zero code is the identity and is
// skipped: every add that happens is the reference's add, bit for bit.
//
// Mapping: eight GPU lanes stand for the eight AVX2 lanes of one block column and keep that column's
// activations in registers (x[b*BS + l + 8k]); a lane may own NBC block columns, and computes them in
// several rows of each stage (four independent add chains, two for the widest variants).  Rows stream
// through a shared-memory ring (1-D bulk copies of whole rows, as in gemv_stream.cu); the eight lanes of
// a column finish all their block sums together in one transposed butterfly, and a fold warp adds each
// row's block terms in block order.
// Rows whose width is not a multiple of the block size (a partial last block has a scalar tail) and the
// scalar order use the general kernel in gemv.cu (Ternary2) or tb_rowwise_kernel below (bitplanes).
#include "common.cuh"
#include "gemv.cuh"

#include <algorithm>

namespace satori {

namespace {

constexpr int kTnCW = 8;               // compute warps
// Rows each lane computes per stage: four independent block sums, or two when the lane already holds
// 32 activations across four block columns (more would spill).
__host__ __device__ constexpr int tn_rows_per_lane(int nbc) { return nbc >= 4 ? 2 : 4; }
constexpr int kTnMaxStages = 12;
constexpr int kTnHeader = 512;
constexpr int kTnTables = 2;

struct TnArgs {
    const uint8_t *payload;
    int rows, nblk, rc, stages, rl, rows_per_stage, fold_rows, pitch;
    uint32_t row_bytes, slot;
    int lpr;                           // lanes per row
    const float *x;
    float *y;
    unsigned *err;
    int use_pdl;
};

struct TnHeader {
    uint64_t *full, *empty, *dfull, *dfree;
    volatile int *abort_flag;
    __device__ explicit TnHeader(uint8_t *smem)
    {
        full = reinterpret_cast<uint64_t *>(smem);
        empty = full + kTnMaxStages;
        dfull = empty + kTnMaxStages;
        dfree = dfull + kTnTables;
        abort_flag = reinterpret_cast<volatile int *>(dfree + kTnTables);
    }
};

__device__ __forceinline__ bool tn_wait(uint64_t *bar, uint32_t parity, const TnHeader &h, unsigned *err)
{
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicOr(err, kDevErrTimeout);
    *h.abort_flag = 1;
    return false;
}

// The fixed horizontal sum of one block's eight lane partials by three shuffles (the sum is valid in every
// lane of the column).
__device__ __forceinline__ float tn_hsum(float a)
{
    const float s1 = fadd(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));     // a_l + a_(l+4)
    const float s2 = fadd(s1, __shfl_xor_sync(0xFFFFFFFFu, s1, 2));   // (a0+a4) + (a2+a6) | (a1+a5) + (a3+a7)
    return fadd(s2, __shfl_xor_sync(0xFFFFFFFFu, s2, 1));
}

// One lane's share of one block: the running sum of its lane of the eight, and with HSUM the block's
// horizontal sum (otherwise tn_reduce forms it).  LAYOUT 0 = Ternary2 codes, 1 = bitplanes.
template <int BS, int LAYOUT, bool HSUM>
__device__ __forceinline__ float tn_block(const uint8_t *blk, const float (&xr)[BS / 8], uint32_t m_lo, uint32_t m_hi)
{
    const uint32_t *w = reinterpret_cast<const uint32_t *>(blk + 4);
    float a = 0.0f;
    if (LAYOUT == 0) {
        // Group k's eight codes are bits 16*(k&1) .. +15 of word k/2; this lane's code is bits 2l, 2l+1.
#pragma unroll
        for (int m = 0; m < BS / 16; ++m) {
            const uint32_t word = w[m];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float xv = xr[2 * m + h];
                if (word & (m_lo << (16 * h))) a = fadd(a, xv);
                if (word & (m_hi << (16 * h))) a = fadd(a, -xv);
            }
        }
    } else {
        // Group k's P and N bits are byte k of each plane; this lane's bit is l of that byte.
        constexpr int PW = BS / 32;
#pragma unroll
        for (int m = 0; m < PW; ++m) {
            const uint32_t p = w[m], n = w[PW + m];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float xv = xr[4 * m + q];
                if (p & (m_lo << (8 * q))) a = fadd(a, xv);
                if (n & (m_lo << (8 * q))) a = fadd(a, -xv);
            }
        }
    }
    (void)m_hi;
    return HSUM ? tn_hsum(a) : a;
}

// Whether a variant interleaves its rows' add chains in one loop (tn_blocks) or computes the rows one after
// another (tn_block) and leaves the overlap to the compiler.  Measured at 4096^2 on a B200: interleaving
// takes the Ternary2 128-block, one-column kernel from 8.7 to 6.3 us, and slows the other variants by 2-5 %.
template <int BS, int NBC, int LAYOUT>
__host__ __device__ constexpr bool tn_interleave_rows()
{
    return LAYOUT == 0 && BS == 128 && NBC == 1;
}

// Whether a variant finishes its lane's block sums together in one transposed butterfly (tn_reduce) or
// each by its own three shuffles (tn_hsum).  Measured at 4096^2 on a B200: the butterfly takes the 64-block
// kernel from 7.1 to 6.5 us and the 256-block kernel from 6.1 to 5.8 us, but slows the 128-block,
// one-column kernels (Ternary2 and STB1) from 6.4 to 8.0 us.
template <int BS, int NBC>
__host__ __device__ constexpr bool tn_transposed_sum()
{
    return !(BS == 128 && NBC == 1);
}

// One lane's share of the same block column in RPL rows: per row, the running sum of its lane of the
// eight, and with HSUM the block's horizontal sum.  The rows' add chains are interleaved weight by weight
// so that they overlap; each row's chain is still added in the reference's order.  LAYOUT 0 = Ternary2
// codes, 1 = bitplanes.
template <int BS, int LAYOUT, int RPL, bool HSUM>
__device__ __forceinline__ void tn_blocks(const uint8_t *const (&blk)[RPL], const float (&xr)[BS / 8], uint32_t m_lo,
                                          uint32_t m_hi, float (&t)[RPL])
{
    float a[RPL];
#pragma unroll
    for (int r = 0; r < RPL; ++r) a[r] = 0.0f;
    if (LAYOUT == 0) {
        // Group k's eight codes are bits 16*(k&1) .. +15 of word k/2; this lane's code is bits 2l, 2l+1.
#pragma unroll
        for (int m = 0; m < BS / 16; ++m) {
            uint32_t word[RPL];
#pragma unroll
            for (int r = 0; r < RPL; ++r) word[r] = reinterpret_cast<const uint32_t *>(blk[r] + 4)[m];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float xv = xr[2 * m + h];
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    if (word[r] & (m_lo << (16 * h))) a[r] = fadd(a[r], xv);
                    if (word[r] & (m_hi << (16 * h))) a[r] = fadd(a[r], -xv);
                }
            }
        }
    } else {
        // Group k's P and N bits are byte k of each plane; this lane's bit is l of that byte.
        constexpr int PW = BS / 32;
#pragma unroll
        for (int m = 0; m < PW; ++m) {
            uint32_t p[RPL], n[RPL];
#pragma unroll
            for (int r = 0; r < RPL; ++r) {
                p[r] = reinterpret_cast<const uint32_t *>(blk[r] + 4)[m];
                n[r] = reinterpret_cast<const uint32_t *>(blk[r] + 4)[PW + m];
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float xv = xr[4 * m + q];
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    if (p[r] & (m_lo << (8 * q))) a[r] = fadd(a[r], xv);
                    if (n[r] & (m_lo << (8 * q))) a[r] = fadd(a[r], -xv);
                }
            }
        }
    }
    (void)m_hi;
    if constexpr (HSUM) {
        float s1[RPL], s2[RPL];
#pragma unroll
        for (int r = 0; r < RPL; ++r) s1[r] = fadd(a[r], __shfl_xor_sync(0xFFFFFFFFu, a[r], 4));
#pragma unroll
        for (int r = 0; r < RPL; ++r) s2[r] = fadd(s1[r], __shfl_xor_sync(0xFFFFFFFFu, s1[r], 2));
#pragma unroll
        for (int r = 0; r < RPL; ++r) t[r] = fadd(s2[r], __shfl_xor_sync(0xFFFFFFFFu, s2[r], 1));
    } else {
#pragma unroll
        for (int r = 0; r < RPL; ++r) t[r] = a[r];
    }
}

// The fixed horizontal sum ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) of V lane partials at once, V = 8 or 4,
// over the eight lanes of a block column (avx = lane & 7), as a transposed butterfly: at each step a lane
// keeps half of its values and sends the other half to its partner, so every value still meets the same
// partners in the same tree and only its operand order can differ, which addition ignores.  V = 8: lane
// avx ends with value avx.  V = 4: lanes 2k and 2k+1 both end with value k.
template <int V>
__device__ __forceinline__ float tn_reduce(const float (&v)[V], int avx)
{
    static_assert(V == 8 || V == 4, "four or eight values per lane");
    const bool b2 = avx & 4, b1 = avx & 2, b0 = avx & 1;
    constexpr int H1 = V / 2, H2 = V / 4;
    float u[H1];
#pragma unroll
    for (int i = 0; i < H1; ++i) {   // a_l + a_(l+4): the low lanes keep values [0, H1), the high lanes the rest
        const float send = b2 ? v[i] : v[i + H1], keep = b2 ? v[i + H1] : v[i];
        u[i] = fadd(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 4));
    }
    float w[H2];
#pragma unroll
    for (int i = 0; i < H2; ++i) {   // (a0+a4) + (a2+a6) on even lanes, (a1+a5) + (a3+a7) on odd lanes
        const float send = b1 ? u[i] : u[i + H2], keep = b1 ? u[i + H2] : u[i];
        w[i] = fadd(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 2));
    }
    if constexpr (V == 8) {
        const float send = b0 ? w[0] : w[1], keep = b0 ? w[1] : w[0];
        return fadd(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 1));
    } else {
        return fadd(w[0], __shfl_xor_sync(0xFFFFFFFFu, w[0], 1));
    }
}

template <int BS, int NBC, int LAYOUT>
__global__ void __launch_bounds__((kTnCW + 2) * 32, 2) gemv_ternary_kernel(const TnArgs a)
{
    constexpr int BB = 4 + BS / 4;
    constexpr int RPL = tn_rows_per_lane(NBC);
    constexpr bool kTransposed = tn_transposed_sum<BS, NBC>();
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const TnHeader h(smem);
    float *dtab = reinterpret_cast<float *>(smem + kTnHeader);
    const int table_floats = a.fold_rows * a.pitch;
    uint8_t *ring = smem + kTnHeader + (size_t)kTnTables * table_floats * 4;
    const int row0 = blockIdx.x * a.rc;
    const int nrows_cta = max(0, min(a.rc, a.rows - row0));
    const int R = a.rows_per_stage;
    const int nst = (nrows_cta + R - 1) / R;
    const int S = a.stages;
    const int fold_stages = a.fold_rows / R;

    if (tid == 0) {
        *h.abort_flag = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&h.full[s], 1);
            mbar_init(&h.empty[s], kTnCW);
        }
        for (int k = 0; k < kTnTables; ++k) {
            mbar_init(&h.dfull[k], kTnCW);
            mbar_init(&h.dfree[k], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const bool producer = warp == kTnCW + 1;
    auto issue = [&](int i, int s) {
        const uint32_t bytes = (uint32_t)min(R, nrows_cta - i * R) * a.row_bytes;
        mbar_expect_tx(&h.full[s], bytes);
        bulk_g2s(ring + (size_t)s * a.slot, a.payload + ((size_t)row0 + (size_t)i * R) * a.row_bytes, bytes, &h.full[s]);
    };
    if (producer && lane == 0)
        for (int i = 0; i < min(S, nst); ++i) issue(i, i);
    if (a.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }

    if (producer) {
        if (lane != 0) return;
        int i = S, s = 0;
        uint32_t par = 0;
        for (; i < nst; ++i) {
            if (*h.abort_flag || !tn_wait(&h.empty[s], par, h, a.err)) break;
            issue(i, s);
            if (++s == S) {
                s = 0;
                par ^= 1u;
            }
        }
        if (*h.abort_flag) {
            const int last = min(i, nst) - 1;
            for (int k = max(0, last - S + 1); k <= last; ++k) mbar_wait_bounded(&h.full[k % S], (uint32_t)((k / S) & 1));
        }
        return;
    }

    if (warp != 0) {
        const int g = (warp - 1) * 32 + lane;
        const int set = g / a.lpr, within = g - set * a.lpr;
        const int col = within >> 3, avx = within & 7;
        const bool active = set < a.rl;
        // Activations of this lane's AVX2 lane in its NBC block columns.
        float xr[NBC][BS / 8];
#pragma unroll
        for (int j = 0; j < NBC; ++j) {
            const int b = min(col * NBC + j, a.nblk - 1);
#pragma unroll
            for (int k = 0; k < BS / 8; ++k) xr[j][k] = a.x[b * BS + avx + 8 * k];
        }
        const uint32_t m_lo = LAYOUT == 0 ? 1u << (2 * avx) : 1u << avx, m_hi = 2u << (2 * avx);
        int s = 0, si = 0, fb = 0;
        uint32_t par = 0;
        for (int i = 0; i < nst; ++i) {
            if (*h.abort_flag) return;
            if (!tn_wait(&h.full[s], par, h, a.err)) return;
            const int nrows = min(R, nrows_cta - i * R);
            float t[RPL][NBC];
            if constexpr (tn_interleave_rows<BS, NBC, LAYOUT>()) {
#pragma unroll
                for (int j = 0; j < NBC; ++j) {
                    const uint8_t *blk[RPL];
#pragma unroll
                    for (int r = 0; r < RPL; ++r) {
                        const int row = min(set, a.rl - 1) + r * a.rl;
                        blk[r] = ring + (size_t)s * a.slot + (size_t)min(row, R - 1) * a.row_bytes +
                                 (size_t)min(col * NBC + j, a.nblk - 1) * BB;
                    }
                    float tj[RPL];
                    tn_blocks<BS, LAYOUT, RPL, !kTransposed>(blk, xr[j], m_lo, m_hi, tj);
#pragma unroll
                    for (int r = 0; r < RPL; ++r) t[r][j] = tj[r];
                }
            } else {
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    const int row = min(set, a.rl - 1) + r * a.rl;
                    const uint8_t *base = ring + (size_t)s * a.slot + (size_t)min(row, R - 1) * a.row_bytes;
#pragma unroll
                    for (int j = 0; j < NBC; ++j)
                        t[r][j] = tn_block<BS, LAYOUT, !kTransposed>(base + (size_t)min(col * NBC + j, a.nblk - 1) * BB,
                                                                     xr[j], m_lo, m_hi);
                }
            }
            const int k = fb & 1;   // fold table of this stage
            if constexpr (kTransposed) {
                // This lane finishes value vi = (row r, column j) of the V = RPL * NBC block sums of its column.
                constexpr int V = RPL * NBC;
                const int vi = V == 8 ? avx : avx >> 1, vr = vi / NBC, vj = vi - vr * NBC;
                const float scale = *reinterpret_cast<const float *>(
                    ring + (size_t)s * a.slot + (size_t)min(min(set, a.rl - 1) + vr * a.rl, R - 1) * a.row_bytes +
                    (size_t)min(col * NBC + vj, a.nblk - 1) * BB);
                // The blocks' words and the scale are read: release the slot, then finish the terms.
                __syncwarp();
                if (lane == 0) mbar_arrive(&h.empty[s]);
                float v[V];
#pragma unroll
                for (int r = 0; r < RPL; ++r)
#pragma unroll
                    for (int j = 0; j < NBC; ++j) v[r * NBC + j] = t[r][j];
                const float term = fmul(tn_reduce<V>(v, avx), scale);
                if (si == 0 && fb >= kTnTables) {
                    if (!tn_wait(&h.dfree[k], (uint32_t)(((fb >> 1) - 1) & 1), h, a.err)) return;
                }
                float *dst = dtab + (size_t)k * table_floats + (size_t)si * R * a.pitch;
                if (active && (V == 8 || (avx & 1) == 0)) {
                    const int row = set + vr * a.rl;
                    if (row < nrows && col * NBC + vj < a.nblk) dst[row * a.pitch + col * NBC + vj] = term;
                }
            } else {
                // Scales and the blocks' words are read: release the slot, then finish the terms.
                float scale[RPL][NBC];
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    const int row = min(min(set, a.rl - 1) + r * a.rl, R - 1);
                    const uint8_t *base = ring + (size_t)s * a.slot + (size_t)row * a.row_bytes;
#pragma unroll
                    for (int j = 0; j < NBC; ++j)
                        scale[r][j] =
                            *reinterpret_cast<const float *>(base + (size_t)min(col * NBC + j, a.nblk - 1) * BB);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&h.empty[s]);
                if (si == 0 && fb >= kTnTables) {
                    if (!tn_wait(&h.dfree[k], (uint32_t)(((fb >> 1) - 1) & 1), h, a.err)) return;
                }
                float *dst = dtab + (size_t)k * table_floats + (size_t)si * R * a.pitch;
                if (active && avx == 0) {
#pragma unroll
                    for (int r = 0; r < RPL; ++r) {
                        const int row = set + r * a.rl;
                        if (row < nrows) {
#pragma unroll
                            for (int j = 0; j < NBC; ++j)
                                if (col * NBC + j < a.nblk)
                                    dst[row * a.pitch + col * NBC + j] = fmul(t[r][j], scale[r][j]);
                        }
                    }
                }
            }
            if (++si == fold_stages || i == nst - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&h.dfull[k]);
                si = 0;
                ++fb;
            }
            if (++s == S) {
                s = 0;
                par ^= 1u;
            }
        }
        return;
    }

    // Fold warp: lane r adds row r's block terms in block order (total += partial * scale).
    const int nfb = (nst + fold_stages - 1) / fold_stages;
    for (int fb = 0; fb < nfb; ++fb) {
        if (*h.abort_flag) break;
        const int k = fb & 1;
        if (!tn_wait(&h.dfull[k], (uint32_t)((fb >> 1) & 1), h, a.err)) break;
        const int nrows = min(a.fold_rows, nrows_cta - fb * a.fold_rows);
        if (lane < nrows) {
            const float *row = dtab + (size_t)k * table_floats + (size_t)lane * a.pitch;
            float acc = 0.0f;
            for (int b = 0; b < a.nblk; ++b) acc = fadd(acc, row[b]);
            a.y[row0 + fb * a.fold_rows + lane] = acc;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&h.dfree[k]);
    }
}

// ---------------------------------------------------------------------------------------- bitplane fallbacks
// One thread per row: TernaryBitplaneMatVec.ExecuteScalar (ORDER_SCALAR) or TernaryBitplaneAvx2Kernel with
// its scalar tail (ORDER_EXECUTE), for any width.
template <bool EXECUTE>
__global__ void tb_rowwise_kernel(const uint8_t *payload, int rows, int cols, int bs, const float *x, float *y)
{
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const int bpr = (cols + bs - 1) / bs, bb = 4 + bs / 4, plane = bs / 8;
    float total = 0.0f;
    for (int b = 0; b < bpr; ++b) {
        const uint8_t *blk = payload + ((size_t)row * bpr + b) * bb;
        const int column = b * bs, count = min(bs, cols - column);
        float partial = 0.0f;
        int i = 0;
        if (EXECUTE) {
            float acc[8];
            for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
            for (; i <= count - 8; i += 8)
                for (int l = 0; l < 8; ++l) {
                    const bool p = (blk[4 + i / 8] >> l) & 1, n = (blk[4 + plane + i / 8] >> l) & 1;
                    const float v = x[column + i + l];
                    acc[l] = fadd(acc[l], p || n ? (n ? -v : v) : 0.0f);
                }
            partial = hsum8(acc);
        }
        for (; i < count; ++i) {
            const int mask = 1 << (i % 8);
            if (blk[4 + i / 8] & mask) partial = fadd(partial, x[column + i]);
            else if (blk[4 + plane + i / 8] & mask) partial = __fsub_rn(partial, x[column + i]);
        }
        total = fadd(total, fmul(__uint_as_float(*reinterpret_cast<const uint32_t *>(blk)), partial));
    }
    y[row] = total;
}

__global__ void tb_decode_row_kernel(const uint8_t *payload, int cols, int bs, const int *row_dev, int row_host,
                                     float *out)
{
    const int row = row_dev ? *row_dev : row_host;
    const int bpr = (cols + bs - 1) / bs, bb = 4 + bs / 4, plane = bs / 8;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < cols; e += gridDim.x * blockDim.x) {
        const uint8_t *blk = payload + ((size_t)row * bpr + e / bs) * bb;
        const int i = e % bs;
        const float scale = __uint_as_float(*reinterpret_cast<const uint32_t *>(blk));
        const bool p = (blk[4 + i / 8] >> (i % 8)) & 1, n = (blk[4 + plane + i / 8] >> (i % 8)) & 1;
        out[e] = p ? scale : n ? -scale : 0.0f;   // the reconstructed weight scale * (P - N)
    }
}

// TernaryBitplaneMatrix.Validate (src/Satori.Core/TernaryBitplaneMatrix.cs:66-87).
__global__ void tb_validate_kernel(const uint8_t *payload, int rows, int cols, int bs, int *status)
{
    const int bpr = (cols + bs - 1) / bs, bb = 4 + bs / 4, plane = bs / 8;
    const long long n = (long long)rows * bpr;
    for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < n; k += (long long)gridDim.x * blockDim.x) {
        const uint8_t *blk = payload + k * bb;
        const uint32_t sb = *reinterpret_cast<const uint32_t *>(blk);
        const float scale = __uint_as_float(sb);
        bool bad = (sb & 0x7F800000u) == 0x7F800000u || scale < 0.0f || sb == 0x80000000u;
        const int count = min(bs, cols - (int)(k % bpr) * bs);
        for (int i = 0; i < plane && !bad; ++i) {
            const int p = blk[4 + i], q = blk[4 + plane + i];
            const int valid = max(0, min(8, count - i * 8));
            const int padding = ~((1 << valid) - 1);
            if ((p & q) != 0 || ((p | q) & padding) != 0 || (scale == 0.0f && (p | q) != 0)) bad = true;
        }
        if (bad) atomicMax(status, (int)SATORI_ERR_ARGUMENT);
    }
}

struct TnVariant {
    int bs, nbc, layout;
    void (*kernel)(const TnArgs);
};

template <int BS, int NBC, int LAYOUT>
constexpr TnVariant tn_variant()
{
    return TnVariant{BS, NBC, LAYOUT, gemv_ternary_kernel<BS, NBC, LAYOUT>};
}

const TnVariant kTnVariants[] = {
    tn_variant<64, 1, 0>(),  tn_variant<64, 2, 0>(),  tn_variant<64, 4, 0>(),  tn_variant<128, 1, 0>(),
    tn_variant<128, 2, 0>(), tn_variant<256, 1, 0>(), tn_variant<64, 1, 1>(),  tn_variant<64, 2, 1>(),
    tn_variant<64, 4, 1>(),  tn_variant<128, 1, 1>(), tn_variant<128, 2, 1>(), tn_variant<256, 1, 1>(),
};

}  // namespace

bool is_bitplane(int format) { return format == SATORI_TB_64 || format == SATORI_TB_128 || format == SATORI_TB_256; }

int ternary_block_size(int format) { return is_bitplane(format) ? format - 1000 : format; }

cudaError_t launch_ternary_stream(const GemvArgs &a, int sm_count, size_t smem_limit, cudaStream_t stream, bool *taken)
{
    *taken = false;
    const int bs = ternary_block_size(a.format);
    const int layout = is_bitplane(a.format) ? 1 : 0;
    if (a.order != SATORI_ORDER_EXECUTE || a.positions != 1 || a.epilogue != kEpiNone) return cudaSuccess;
    if (a.cols % bs != 0 || (reinterpret_cast<uintptr_t>(a.payload) & 15)) return cudaSuccess;
    const int nblk = a.cols / bs, bb = 4 + bs / 4;
    const size_t row_bytes = (size_t)nblk * bb;
    if (row_bytes % 16) return cudaSuccess;
    int nbc = 1;
    while (nblk > 32 * nbc && nbc * bs / 8 < 32) nbc *= 2;
    if (nblk > 32 * nbc || nblk % nbc) return cudaSuccess;
    const TnVariant *v = nullptr;
    for (const TnVariant &c : kTnVariants)
        if (c.bs == bs && c.nbc == nbc && c.layout == layout) v = &c;
    if (!v) return cudaSuccess;
    const int lpr = nblk / nbc * 8;
    const int rl = kTnCW * 32 / lpr;
    if (rl < 1) return cudaSuccess;
    const int R = rl * tn_rows_per_lane(nbc);
    const int pitch = nblk + 1;
    int fold_rows = std::max(R, (32 / R) * R);
    while (fold_rows > R && (size_t)kTnTables * fold_rows * pitch * 4 > 32 * 1024) fold_rows -= R;
    if (fold_rows > 32) return cudaSuccess;
    const size_t slot = ((size_t)R * row_bytes + 16 + 127) & ~(size_t)127;
    const size_t fixed = 128 + kTnHeader + (size_t)kTnTables * fold_rows * pitch * 4;
    const size_t budget = std::min(smem_limit, (size_t)113 * 1024);
    if (budget < fixed + slot) return cudaSuccess;
    const int grid0 = std::min((a.rows + R - 1) / R, 2 * sm_count);
    const int rc = (a.rows + grid0 - 1) / grid0;
    const int nst = (rc + R - 1) / R;
    const int stages = std::max(1, std::min({(int)((budget - fixed) / slot), kTnMaxStages, nst}));
    TnArgs t;
    t.payload = a.payload;
    t.rows = a.rows;
    t.nblk = nblk;
    t.rc = rc;
    t.stages = stages;
    t.rl = rl;
    t.rows_per_stage = R;
    t.fold_rows = fold_rows;
    t.pitch = pitch;
    t.row_bytes = (uint32_t)row_bytes;
    t.slot = (uint32_t)slot;
    t.lpr = lpr;
    t.x = a.x;
    t.y = a.y;
    t.err = a.err;
    t.use_pdl = a.use_pdl;
    const size_t smem = fixed + stages * slot;
    cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(v->kernel), smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.rows + rc - 1) / rc);
    cfg.blockDim = dim3((kTnCW + 2) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.use_pdl ? 1 : 0;
    *taken = true;
    return cudaLaunchKernelEx(&cfg, v->kernel, t);
}

cudaError_t launch_bitplane_rowwise(const GemvArgs &a, cudaStream_t stream)
{
    const int bs = ternary_block_size(a.format);
    const dim3 grid((a.rows + 127) / 128), block(128);
    if (a.order == SATORI_ORDER_EXECUTE)
        tb_rowwise_kernel<true><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, bs, a.x, a.y);
    else
        tb_rowwise_kernel<false><<<grid, block, 0, stream>>>(a.payload, a.rows, a.cols, bs, a.x, a.y);
    return cudaGetLastError();
}

cudaError_t launch_bitplane_decode_row(const uint8_t *payload, int cols, int format, const int *row_dev, int row_host,
                                       float *out, cudaStream_t stream)
{
    tb_decode_row_kernel<<<std::min(64, (cols + 255) / 256), 256, 0, stream>>>(payload, cols, ternary_block_size(format),
                                                                              row_dev, row_host, out);
    return cudaGetLastError();
}

cudaError_t launch_bitplane_validate(const uint8_t *payload, int rows, int cols, int format, int *status_dev,
                                     cudaStream_t stream)
{
    tb_validate_kernel<<<592, 256, 0, stream>>>(payload, rows, cols, ternary_block_size(format), status_dev);
    return cudaGetLastError();
}

}  // namespace satori
