// attention.cu -- decode grouped-query attention for sm_100a.
//
// Restates TransformerOps.GroupedAttention (src/Satori.Core/TransformerOps.cs:140-179): query
// head h attends to KV head h / (q_heads / kv_heads) over the causal prefix; softmax of
// (q . k) / sqrt(head_dim), weighted sum of v.  The reference works in FP64; this kernel works in
// FP32 with split-K flash decoding, which stays within the stated 1e-5 relative + 1e-6 absolute
// of the FP64 result for finite scores.  Where FP32 scores overflow (|q . k| beyond FP32 range --
// the reference's own FLT_MAX test), the merge kernel recomputes that head in FP64 on the device.
//
// Work decomposition: one CTA per (sequence split, KV head, group of up to 8 query heads).  The
// CTA's four warps walk 32-token blocks of the split; each lane owns 4 contiguous dims of the
// 128-wide head, so a token's K or V row is one coalesced 512-byte warp load and every K/V byte
// is read from HBM once for all query heads of its group.  Per token the 8 head partial dots are
// reduced across the warp with a transposed butterfly (9 shuffles instead of 40).  Online softmax
// state (m, l, acc) is kept per warp, merged per CTA into one partial record, and the records of
// all splits are merged by a second kernel.
#include <cuda.h>

#include "attention.cuh"
#include "common.cuh"

#include <algorithm>
#include <cmath>

namespace satori {

namespace {

constexpr int kWarps = 4;
constexpr int kTokBlock = 32;

struct AttnParams {
    const float *q, *keys, *values;
    int q_heads, kv_heads, head_dim, group, ngroups;
    int kv_stride;   // floats between consecutive tokens' K (or V) rows
    int tokens;
    const int *tokens_dev;
    int nsplit;
    float scale;
    float *scratch;        // split records [nsplit][q_heads][head_dim + 2]
    float *out;
    unsigned *err;
    int use_pdl;
    // Prefill chunk: position z of the batch (blockIdx.z of the partial kernels, blockIdx.y of the merge)
    // reads q + z * q_pstride, attends to tokens + z tokens and writes out + z * out_pstride.
    int batch;
    long long q_pstride, out_pstride;
};

// The parameters of batch position z.
__device__ __forceinline__ AttnParams attn_at(const AttnParams &in, int z)
{
    AttnParams p = in;
    if (z > 0) {
        p.q += z * in.q_pstride;
        p.out += z * in.out_pstride;
        p.scratch += (long long)z * in.nsplit * in.q_heads * (in.head_dim + 2);
        p.tokens += z;
    }
    return p;
}

// Sum across the warp of N values per lane, N a power of two <= 8.  On return v[0] holds, in
// every lane, the total of head (lane / (32 / N)); all lanes of a head hold identical bits.
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[8], int lane)
{
    int off = 16;
#pragma unroll
    for (int n = N; n > 1; n >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
        }
    }
#pragma unroll
    for (; off >= 1; off >>= 1) v[0] = v[0] + __shfl_xor_sync(0xFFFFFFFFu, v[0], off);
    return v[0];
}

template <int DPL, bool VEC4>
__device__ __forceinline__ void load_row(const float *row, int lane, int hd, float (&r)[DPL])
{
    if (VEC4) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(row) + lane);
        r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            r[i] = d < hd ? __ldg(row + d) : 0.0f;
        }
    }
}

template <int DPL, bool VEC4>
__device__ __forceinline__ int dim_of(int lane, int i) { return VEC4 ? 4 * lane + i : lane + 32 * i; }

template <int DPL, bool VEC4, int GMAX>
__global__ void __launch_bounds__(kWarps * 32) attn_partial_kernel(const AttnParams pin)
{
    const AttnParams p = attn_at(pin, blockIdx.z);
    constexpr int R = 32 / GMAX;  // lanes per head after the transposed reduction
    __shared__ float P[kWarps][GMAX][kTokBlock];
    __shared__ float wm[kWarps][GMAX], wl[kWarps][GMAX];
    __shared__ float wacc[kWarps][GMAX][DPL * 32];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.ngroups, grp = blockIdx.y % p.ngroups;
    const int h0 = kvh * p.group + grp * GMAX;
    const int gc = min(GMAX, p.group - grp * GMAX);
    const int hd = p.head_dim;
    const int kvw = p.kv_stride;
    const int hl = lane / R;

    if (p.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const int T = p.tokens_dev ? *p.tokens_dev : p.tokens;
    const int t0 = (int)(((long long)T * split) / p.nsplit);
    const int t1 = (int)(((long long)T * (split + 1)) / p.nsplit);

    float qr[GMAX][DPL];
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = dim_of<DPL, VEC4>(lane, i);
            qr[h][i] = (h < gc && d < hd) ? p.q[(h0 + h) * hd + d] : 0.0f;
        }
    float acc[GMAX][DPL];
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[h][i] = 0.0f;
    float m_my = -INFINITY, l_my = 0.0f;

    const float *kbase = p.keys + (long long)kvh * hd;
    const float *vbase = p.values + (long long)kvh * hd;

    for (int tb = t0 + warp * kTokBlock; tb < t1; tb += kWarps * kTokBlock) {
        const int nt = min(kTokBlock, t1 - tb);
        float sc[kTokBlock];
#pragma unroll
        for (int j = 0; j < kTokBlock; ++j) {
            if (j < nt) {
                float kr[DPL];
                load_row<DPL, VEC4>(kbase + (long long)(tb + j) * kvw, lane, hd, kr);
                float v[8];
#pragma unroll
                for (int h = 0; h < 8; ++h) v[h] = 0.0f;
#pragma unroll
                for (int h = 0; h < GMAX; ++h) {
                    float s = 0.0f;
#pragma unroll
                    for (int i = 0; i < DPL; ++i) s = fmaf(qr[h][i], kr[i], s);
                    v[h] = s;
                }
                sc[j] = transpose_reduce<GMAX>(v, lane) * p.scale;
            } else {
                sc[j] = -INFINITY;
            }
        }
        float mb = sc[0];
#pragma unroll
        for (int j = 1; j < kTokBlock; ++j) mb = fmaxf(mb, sc[j]);
        const float m_new = fmaxf(m_my, mb);
        const float alpha = m_my == -INFINITY ? 0.0f : expf(m_my - m_new);
        float lsum = 0.0f;
#pragma unroll
        for (int j = 0; j < kTokBlock; ++j) {
            const float pj = j < nt ? expf(sc[j] - m_new) : 0.0f;
            lsum += pj;
            if ((j % R) == (lane % R)) P[warp][hl][j] = pj;
        }
        l_my = l_my * alpha + lsum;
        m_my = m_new;
        float alpha_h[GMAX];
#pragma unroll
        for (int h = 0; h < GMAX; ++h) alpha_h[h] = __shfl_sync(0xFFFFFFFFu, alpha, h * R);
#pragma unroll
        for (int h = 0; h < GMAX; ++h)
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[h][i] *= alpha_h[h];
        __syncwarp();
        for (int j = 0; j < nt; ++j) {
            float vr[DPL];
            load_row<DPL, VEC4>(vbase + (long long)(tb + j) * kvw, lane, hd, vr);
#pragma unroll
            for (int h = 0; h < GMAX; ++h) {
                const float pj = P[warp][h][j];
#pragma unroll
                for (int i = 0; i < DPL; ++i) acc[h][i] = fmaf(pj, vr[i], acc[h][i]);
            }
        }
        __syncwarp();
    }

    // Per-warp state -> shared memory, then one merged record per (split, head).
    if (lane % R == 0) {
        wm[warp][hl] = m_my;
        wl[warp][hl] = l_my;
    }
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int i = 0; i < DPL; ++i) wacc[warp][h][i * 32 + lane] = acc[h][i];
    __syncthreads();

    const int rec_stride = hd + 2;
    for (int idx = threadIdx.x; idx < gc * (hd + 2); idx += blockDim.x) {
        const int h = idx / (hd + 2), e = idx - h * (hd + 2);
        float m = wm[0][h];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) m = fmaxf(m, wm[w][h]);
        float val = 0.0f;
        if (e == 0) {
            val = m;
        } else {
            for (int w = 0; w < kWarps; ++w) {
                const float f = wm[w][h] == -INFINITY ? 0.0f : expf(wm[w][h] - m);
                float x;
                if (e == 1) {
                    x = wl[w][h];
                } else {
                    const int d = e - 2;
                    int lane_d, i_d;
                    if (VEC4) { lane_d = d >> 2; i_d = d & 3; } else { lane_d = d & 31; i_d = d >> 5; }
                    x = wacc[w][h][i_d * 32 + lane_d];
                }
                val = fmaf(x, f, val);
            }
        }
        p.scratch[((long long)split * p.q_heads + h0 + h) * rec_stride + e] = val;
    }
}

// FP64 recompute of one head (the reference's arithmetic), used when FP32 scores overflowed.
__device__ void head_fp64(const AttnParams &p, int head, int T, double *sbuf, float *out)
{
    const int hd = p.head_dim, kvw = p.kv_stride;
    const int kvh = head / p.group;
    const float *q = p.q + (long long)head * hd;
    const double scale = 1.0 / sqrt((double)hd);
    __shared__ double red[128];
    // pass 1: max score
    double mx = -INFINITY;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float *k = p.keys + (long long)t * kvw + kvh * hd;
        double dot = 0;
        for (int j = 0; j < hd; ++j) dot = __dadd_rn(dot, __dmul_rn((double)q[j], (double)k[j]));
        mx = fmax(mx, __dmul_rn(dot, scale));
    }
    red[threadIdx.x] = mx;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = fmax(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    mx = red[0];
    __syncthreads();
    // pass 2: total
    double tot = 0;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float *k = p.keys + (long long)t * kvw + kvh * hd;
        double dot = 0;
        for (int j = 0; j < hd; ++j) dot = __dadd_rn(dot, __dmul_rn((double)q[j], (double)k[j]));
        tot = __dadd_rn(tot, exp(__dsub_rn(__dmul_rn(dot, scale), mx)));
    }
    red[threadIdx.x] = tot;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = __dadd_rn(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    tot = red[0];
    __syncthreads();
    // pass 3: sum_t (p_t / total) * v_t, in token order per dim
    double sum[2] = {0, 0};
    for (int tc = 0; tc < T; tc += blockDim.x) {
        const int t = tc + threadIdx.x;
        if (t < T) {
            const float *k = p.keys + (long long)t * kvw + kvh * hd;
            double dot = 0;
            for (int j = 0; j < hd; ++j) dot = __dadd_rn(dot, __dmul_rn((double)q[j], (double)k[j]));
            sbuf[threadIdx.x] = exp(__dsub_rn(__dmul_rn(dot, scale), mx));
        }
        __syncthreads();
        const int n = min((int)blockDim.x, T - tc);
        for (int r = 0; r < 2; ++r) {
            const int d = threadIdx.x + r * blockDim.x;
            if (d < hd)
                for (int j = 0; j < n; ++j)
                    sum[r] = __dadd_rn(sum[r], __dmul_rn(__ddiv_rn(sbuf[j], tot),
                                                         (double)p.values[(long long)(tc + j) * kvw + kvh * hd + d]));
        }
        __syncthreads();
    }
    for (int r = 0; r < 2; ++r) {
        const int d = threadIdx.x + r * blockDim.x;
        if (d < hd) out[d] = (float)sum[r];
    }
}

// Streaming variant for head_dim 128 and groups of up to 8 query heads (every BASELINE shape):
// a producer warp streams the split's K and V rows of one KV head in 8-token tiles with 3-D TMA
// loads (unicast) into a ring of 16 shared-memory slots, two per compute warp, so that ~64 KB per
// SM are in flight; compute warp w takes tiles w, w + 8, ... and runs the same per-token arithmetic
// as attn_partial_kernel (lane = 4 dims, transposed butterfly, per-warp online softmax), reading K and
// V from shared memory.  The per-warp states are merged into the same partial records.
constexpr int kStreamWarps = 8;
constexpr int kStreamTok = 8;                       // tokens per tile
constexpr int kStreamSlots = 2 * kStreamWarps;
constexpr int kStreamTileBytes = kStreamTok * 128 * 4;
constexpr int kStreamHeader = 384;             // full[16] + empty[16] mbarriers, then the abort flag
constexpr int kStreamPBytes = kStreamWarps * 8 * kStreamTok * 4;
constexpr size_t kStreamSmem =
    128 + kStreamHeader + kStreamPBytes + (size_t)kStreamSlots * 2 * kStreamTileBytes;

__device__ __forceinline__ void tma_load_3d(void *dst, const void *map, int c0, int c1, int c2, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
                    "r"(smem_u32(bar))
                 : "memory");
}

__global__ void __launch_bounds__((kStreamWarps + 1) * 32, 1)
    attn_stream_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const AttnParams pin)
{
    const AttnParams p = attn_at(pin, blockIdx.z);
    constexpr int GMAX = 8, DPL = 4, R = 32 / GMAX;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStreamSlots;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStreamSlots);
    // p of a warp's tile, token-major: the eight heads of token j are one 32-byte row.
    float (*P)[kStreamTok][GMAX] = reinterpret_cast<float (*)[kStreamTok][GMAX]>(smem + kStreamHeader);
    uint8_t *slots = smem + kStreamHeader + kStreamPBytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.ngroups, grp = blockIdx.y % p.ngroups;
    const int h0 = kvh * p.group + grp * GMAX;
    const int gc = min(GMAX, p.group - grp * GMAX);
    const int hd = 128;
    const int hl = lane / R;

    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStreamSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (p.use_pdl) {   // the token count and the newest K/V row come from earlier kernels
        pdl_launch_dependents();
        pdl_wait();
    }
    const int T = p.tokens_dev ? *p.tokens_dev : p.tokens;
    const int t0 = (int)(((long long)T * split) / p.nsplit);
    const int t1 = (int)(((long long)T * (split + 1)) / p.nsplit);
    const int nst = (t1 - t0 + kStreamTok - 1) / kStreamTok;

    // acc[h][c] holds dims (2c, 2c+1) of this lane's 4 for head h: FP32x2 FMAs, each component rounded
    // exactly as a scalar fmaf chain.
    float2 acc[GMAX][DPL / 2];
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int c = 0; c < DPL / 2; ++c) acc[h][c] = make_float2(0.0f, 0.0f);
    float m_my = -INFINITY, l_my = 0.0f;

    if (warp == kStreamWarps) {
        if (lane == 0) {
            auto issue = [&](int k) {
                const int s = k % kStreamSlots;
                uint8_t *dst = slots + (size_t)s * 2 * kStreamTileBytes;
                mbar_expect_tx(&full[s], 2u * kStreamTileBytes);
                tma_load_3d(dst, &kmap, 0, kvh, t0 + k * kStreamTok, &full[s]);
                tma_load_3d(dst + kStreamTileBytes, &vmap, 0, kvh, t0 + k * kStreamTok, &full[s]);
            };
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            const int first = min(kStreamSlots, nst);
            for (int k = 0; k < first; ++k) issue(k);
            int k = 0;
            for (; k + kStreamSlots < nst; ++k) {
                if (*abort_flag || !mbar_wait_bounded(&empty[k % kStreamSlots], (uint32_t)((k / kStreamSlots) & 1))) {
                    if (p.err) atomicOr(p.err, kDevErrTimeout);
                    *abort_flag = 1;
                    break;
                }
                issue(k + kStreamSlots);
            }
            // Every copy issued lands before the CTA's shared memory goes away.
            const int last = min(k + kStreamSlots, nst) - 1;
            for (int j = max(0, last - kStreamSlots + 1); j <= last; ++j)
                mbar_wait_bounded(&full[j % kStreamSlots], (uint32_t)((j / kStreamSlots) & 1));
        }
    } else {
        // q of head pairs (2g, 2g+1): one FP32x2 FMA advances both heads' dot products.
        float2 qp[GMAX / 2][DPL];
#pragma unroll
        for (int g = 0; g < GMAX / 2; ++g)
#pragma unroll
            for (int i = 0; i < DPL; ++i)
                qp[g][i] = make_float2(2 * g < gc ? p.q[(h0 + 2 * g) * hd + 4 * lane + i] : 0.0f,
                                       2 * g + 1 < gc ? p.q[(h0 + 2 * g + 1) * hd + 4 * lane + i] : 0.0f);
        for (int k = warp; k < nst; k += kStreamWarps) {
            const int s = k % kStreamSlots;
            if (*abort_flag) break;
            if (!mbar_wait_bounded(&full[s], (uint32_t)((k / kStreamSlots) & 1))) {
                if (p.err) atomicOr(p.err, kDevErrTimeout);
                *abort_flag = 1;
                break;
            }
            const uint32_t kt = smem_u32(slots + (size_t)s * 2 * kStreamTileBytes) + 16u * lane;
            const uint32_t vt = kt + kStreamTileBytes;
            const int tb = t0 + k * kStreamTok;
            const int nt = min(kStreamTok, t1 - tb);
            float sc[kStreamTok];
#pragma unroll
            for (int j = 0; j < kStreamTok; ++j) {
                if (j < nt) {
                    const float4 t4 = lds128f(kt + 512u * j);
                    const float kr[DPL] = {t4.x, t4.y, t4.z, t4.w};
                    float v[8];
#pragma unroll
                    for (int g = 0; g < GMAX / 2; ++g) {
                        float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int i = 0; i < DPL; ++i) a = __ffma2_rn(qp[g][i], make_float2(kr[i], kr[i]), a);
                        v[2 * g] = a.x;
                        v[2 * g + 1] = a.y;
                    }
                    sc[j] = transpose_reduce<GMAX>(v, lane) * p.scale;
                } else {
                    sc[j] = -INFINITY;
                }
            }
            float mb = sc[0];
#pragma unroll
            for (int j = 1; j < kStreamTok; ++j) mb = fmaxf(mb, sc[j]);
            const float m_new = fmaxf(m_my, mb);
            const float alpha = m_my == -INFINITY ? 0.0f : expf(m_my - m_new);
            float lsum = 0.0f;
#pragma unroll
            for (int j = 0; j < kStreamTok; ++j) {
                const float pj = j < nt ? expf(sc[j] - m_new) : 0.0f;
                lsum += pj;
                if ((j % R) == (lane % R)) P[warp][j][hl] = pj;
            }
            l_my = l_my * alpha + lsum;
            m_my = m_new;
#pragma unroll
            for (int h = 0; h < GMAX; ++h) {
                const float ah = __shfl_sync(0xFFFFFFFFu, alpha, h * R);
#pragma unroll
                for (int c = 0; c < DPL / 2; ++c) acc[h][c] = __fmul2_rn(acc[h][c], make_float2(ah, ah));
            }
            __syncwarp();
            for (int j = 0; j < nt; ++j) {
                const float4 t4 = lds128f(vt + 512u * j);
                const float2 v01 = make_float2(t4.x, t4.y), v23 = make_float2(t4.z, t4.w);
                const float4 pa = *reinterpret_cast<const float4 *>(&P[warp][j][0]);
                const float4 pb = *reinterpret_cast<const float4 *>(&P[warp][j][4]);
                const float pj[GMAX] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int h = 0; h < GMAX; ++h) {
                    const float2 pp = make_float2(pj[h], pj[h]);
                    acc[h][0] = __ffma2_rn(pp, v01, acc[h][0]);
                    acc[h][1] = __ffma2_rn(pp, v23, acc[h][1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);   // the producer may refill this slot
        }
    }
    __syncthreads();   // every tile consumed: the slots now hold the per-warp states

    float *wm = reinterpret_cast<float *>(slots);                    // [kStreamWarps][GMAX]
    float *wl = wm + kStreamWarps * GMAX;                             // [kStreamWarps][GMAX]
    float *wacc = wl + kStreamWarps * GMAX;                           // [kStreamWarps][GMAX][128]
    if (warp < kStreamWarps) {
        if (lane % R == 0) {
            wm[warp * GMAX + hl] = m_my;
            wl[warp * GMAX + hl] = l_my;
        }
#pragma unroll
        for (int h = 0; h < GMAX; ++h) {
            float *w = wacc + (warp * GMAX + h) * hd + 4 * lane;
            w[0] = acc[h][0].x;
            w[1] = acc[h][0].y;
            w[2] = acc[h][1].x;
            w[3] = acc[h][1].y;
        }
    }
    __syncthreads();
    const int rec_stride = hd + 2;
    // A wait that ran out left tiles unread: the split's records become NaN, which sends every head the
    // split serves to the merge kernel's FP64 recomputation from K and V instead of a silently partial
    // sum (this also covers callers that pass no error word).
    const bool aborted = *abort_flag != 0;
    for (int idx = tid; idx < gc * rec_stride; idx += blockDim.x) {
        const int h = idx / rec_stride, e = idx - h * rec_stride;
        float m = wm[h];
#pragma unroll
        for (int w = 1; w < kStreamWarps; ++w) m = fmaxf(m, wm[w * GMAX + h]);
        float val = 0.0f;
        if (e == 0) {
            val = m;
        } else {
            for (int w = 0; w < kStreamWarps; ++w) {
                const float mw = wm[w * GMAX + h];
                const float f = mw == -INFINITY ? 0.0f : expf(mw - m);
                const float x = e == 1 ? wl[w * GMAX + h] : wacc[(w * GMAX + h) * hd + (e - 2)];
                val = fmaf(x, f, val);
            }
        }
        p.scratch[((long long)split * p.q_heads + h0 + h) * rec_stride + e] = aborted ? __int_as_float(0x7fc00000) : val;
    }
}

// Prefill: the positions of a chunk attend to nearly the same prefix, so one CTA serves 8 consecutive
// positions of one KV head (warp w = position zb + w) and every K/V tile it streams is read by all 8
// warps from shared memory.  The CTA's token range [t0, t1) is split s of the LONGEST prefix of its
// positions; position z uses [t0, min(t1, T_z)) and writes its own split record (an empty range gives
// m = -inf, l = 0, which the merge weighs as zero).  Per token and head the arithmetic is the stream
// kernel's (FP32x2 dot, transposed butterfly, online softmax, FP32x2 p.v).
constexpr int kPrefillPos = kStreamWarps;            // positions per CTA

__global__ void __launch_bounds__((kStreamWarps + 1) * 32, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const AttnParams p)
{
    constexpr int GMAX = 8, DPL = 4, R = 32 / GMAX;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStreamSlots;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStreamSlots);
    float (*P)[kStreamTok][GMAX] = reinterpret_cast<float (*)[kStreamTok][GMAX]>(smem + kStreamHeader);
    uint8_t *slots = smem + kStreamHeader + kStreamPBytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.ngroups, grp = blockIdx.y % p.ngroups;
    const int h0 = kvh * p.group + grp * GMAX;
    const int gc = min(GMAX, p.group - grp * GMAX);
    const int hd = 128;
    const int hl = lane / R;
    const int zb = blockIdx.z * kPrefillPos;
    const int nz = min(kPrefillPos, p.batch - zb);             // positions of this CTA

    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStreamSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kStreamWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (p.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const int Tmax = p.tokens + zb + nz - 1;                   // prefix of the CTA's last position
    const int t0 = (int)(((long long)Tmax * split) / p.nsplit);
    const int t1 = (int)(((long long)Tmax * (split + 1)) / p.nsplit);
    const int nst = (t1 - t0 + kStreamTok - 1) / kStreamTok;

    if (warp == kStreamWarps) {
        if (lane == 0) {
            auto issue = [&](int k) {
                const int s = k % kStreamSlots;
                uint8_t *dst = slots + (size_t)s * 2 * kStreamTileBytes;
                mbar_expect_tx(&full[s], 2u * kStreamTileBytes);
                tma_load_3d(dst, &kmap, 0, kvh, t0 + k * kStreamTok, &full[s]);
                tma_load_3d(dst + kStreamTileBytes, &vmap, 0, kvh, t0 + k * kStreamTok, &full[s]);
            };
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            const int first = min(kStreamSlots, nst);
            for (int k = 0; k < first; ++k) issue(k);
            int k = 0;
            for (; k + kStreamSlots < nst; ++k) {
                if (*abort_flag || !mbar_wait_bounded(&empty[k % kStreamSlots], (uint32_t)((k / kStreamSlots) & 1))) {
                    if (p.err) atomicOr(p.err, kDevErrTimeout);
                    *abort_flag = 1;
                    break;
                }
                issue(k + kStreamSlots);
            }
            const int last = min(k + kStreamSlots, nst) - 1;
            for (int j = max(0, last - kStreamSlots + 1); j <= last; ++j)
                mbar_wait_bounded(&full[j % kStreamSlots], (uint32_t)((j / kStreamSlots) & 1));
        }
        return;
    }

    // Compute warp: position z = zb + warp (idle but still pacing the ring when z is past the batch).
    const int z = zb + warp;
    const bool live = warp < nz;
    const int Tz = p.tokens + z;
    const int tend = live ? min(t1, Tz) : t0;                  // this position's tokens: [t0, tend)
    const float *q = p.q + (long long)(live ? z : zb) * p.q_pstride;
    float2 qp[GMAX / 2][DPL];
#pragma unroll
    for (int g = 0; g < GMAX / 2; ++g)
#pragma unroll
        for (int i = 0; i < DPL; ++i)
            qp[g][i] = make_float2(2 * g < gc ? q[(h0 + 2 * g) * hd + 4 * lane + i] : 0.0f,
                                   2 * g + 1 < gc ? q[(h0 + 2 * g + 1) * hd + 4 * lane + i] : 0.0f);
    float2 acc[GMAX][DPL / 2];
#pragma unroll
    for (int h = 0; h < GMAX; ++h)
#pragma unroll
        for (int c = 0; c < DPL / 2; ++c) acc[h][c] = make_float2(0.0f, 0.0f);
    float m_my = -INFINITY, l_my = 0.0f;
    for (int k = 0; k < nst; ++k) {
        const int s = k % kStreamSlots;
        if (*abort_flag) break;
        if (!mbar_wait_bounded(&full[s], (uint32_t)((k / kStreamSlots) & 1))) {
            if (p.err) atomicOr(p.err, kDevErrTimeout);
            *abort_flag = 1;
            break;
        }
        const int tb = t0 + k * kStreamTok;
        const int nt = min(kStreamTok, tend - tb);                 // <= 0: past this position's prefix
        if (nt > 0) {
            const uint32_t kt = smem_u32(slots + (size_t)s * 2 * kStreamTileBytes) + 16u * lane;
            const uint32_t vt = kt + kStreamTileBytes;
            float sc[kStreamTok];
#pragma unroll
            for (int j = 0; j < kStreamTok; ++j) {
                if (j < nt) {
                    const float4 t4 = lds128f(kt + 512u * j);
                    const float kr[DPL] = {t4.x, t4.y, t4.z, t4.w};
                    float v[8];
#pragma unroll
                    for (int g = 0; g < GMAX / 2; ++g) {
                        float2 a = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int i = 0; i < DPL; ++i) a = __ffma2_rn(qp[g][i], make_float2(kr[i], kr[i]), a);
                        v[2 * g] = a.x;
                        v[2 * g + 1] = a.y;
                    }
                    sc[j] = transpose_reduce<GMAX>(v, lane) * p.scale;
                } else {
                    sc[j] = -INFINITY;
                }
            }
            float mb = sc[0];
#pragma unroll
            for (int j = 1; j < kStreamTok; ++j) mb = fmaxf(mb, sc[j]);
            const float m_new = fmaxf(m_my, mb);
            const float alpha = m_my == -INFINITY ? 0.0f : expf(m_my - m_new);
            float lsum = 0.0f;
#pragma unroll
            for (int j = 0; j < kStreamTok; ++j) {
                const float pj = j < nt ? expf(sc[j] - m_new) : 0.0f;
                lsum += pj;
                if ((j % R) == (lane % R)) P[warp][j][hl] = pj;
            }
            l_my = l_my * alpha + lsum;
            m_my = m_new;
#pragma unroll
            for (int h = 0; h < GMAX; ++h) {
                const float ah = __shfl_sync(0xFFFFFFFFu, alpha, h * R);
#pragma unroll
                for (int c = 0; c < DPL / 2; ++c) acc[h][c] = __fmul2_rn(acc[h][c], make_float2(ah, ah));
            }
            __syncwarp();
            for (int j = 0; j < nt; ++j) {
                const float4 t4 = lds128f(vt + 512u * j);
                const float2 v01 = make_float2(t4.x, t4.y), v23 = make_float2(t4.z, t4.w);
                const float4 pa = *reinterpret_cast<const float4 *>(&P[warp][j][0]);
                const float4 pb = *reinterpret_cast<const float4 *>(&P[warp][j][4]);
                const float pj[GMAX] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int h = 0; h < GMAX; ++h) {
                    const float2 pp = make_float2(pj[h], pj[h]);
                    acc[h][0] = __ffma2_rn(pp, v01, acc[h][0]);
                    acc[h][1] = __ffma2_rn(pp, v23, acc[h][1]);
                }
            }
            __syncwarp();
        }
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!live) return;
    // This position's record of this split; an expired wait leaves NaN for the merge's FP64 recompute.
    const bool aborted = *abort_flag != 0;
    const int rs = hd + 2;
    float *rec = p.scratch + (long long)z * p.nsplit * p.q_heads * rs + (long long)split * p.q_heads * rs;
    const float nan = __int_as_float(0x7fc00000);
    if (lane % R == 0 && hl < gc) {
        rec[(h0 + hl) * rs] = aborted ? nan : m_my;
        rec[(h0 + hl) * rs + 1] = aborted ? nan : l_my;
    }
#pragma unroll
    for (int h = 0; h < GMAX; ++h) {
        if (h < gc) {
            float *w = rec + (h0 + h) * rs + 2 + 4 * lane;
            w[0] = aborted ? nan : acc[h][0].x;
            w[1] = aborted ? nan : acc[h][0].y;
            w[2] = aborted ? nan : acc[h][1].x;
            w[3] = aborted ? nan : acc[h][1].y;
        }
    }
}

// Split records are merged in chunks staged through shared memory with cp.async, so every record
// load of a chunk is in flight at once (a thread walking the splits one global load at a time is
// latency-bound).  The arithmetic and its order are unchanged: max over splits, then l and each output
// dim as sequential fmaf sums over the splits in split order.
constexpr int kMergeThreads = 128;
constexpr int kMergeChunk = 32;   // splits staged per round (small: the next kernel shares its SM)

__device__ __forceinline__ void cp_async4(float *dst, const float *src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(const AttnParams pin)
{
    const AttnParams p = attn_at(pin, blockIdx.y);
    extern __shared__ float msm[];   // wts[nsplit] (padded to 4), then chunk[kMergeChunk][head_dim + 2]
    __shared__ float wmax[kMergeThreads / 32];
    __shared__ double sbuf[128];
    const int head = blockIdx.x, tid = threadIdx.x;
    const int hd = p.head_dim, rs = hd + 2;
    float *wts = msm;
    float *chunk = msm + ((p.nsplit + 3) & ~3);
    if (p.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    bool bad = false;   // this thread's view; combined before the result is written
    const float *rec = p.scratch + (long long)head * rs;
    const long long split_stride = (long long)p.q_heads * rs;
    // Maximum of the split maxima (order-free), each split's max read by one thread.
    float m = -INFINITY;
    for (int s = tid; s < p.nsplit; s += kMergeThreads) {
        const float ms = rec[s * split_stride];
        wts[s] = ms;
        bad |= isnan(ms) || ms == INFINITY;
        m = fmaxf(m, ms);
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((tid & 31) == 0) wmax[tid >> 5] = m;
    __syncthreads();
    m = wmax[0];
    for (int w = 1; w < kMergeThreads / 32; ++w) m = fmaxf(m, wmax[w]);
    for (int s = tid; s < p.nsplit; s += kMergeThreads) {
        const float ms = wts[s];
        wts[s] = ms == -INFINITY ? 0.0f : expf(ms - m);
    }
    float l = 0.0f, a[2] = {0.0f, 0.0f};
    for (int s0 = 0; s0 < p.nsplit; s0 += kMergeChunk) {
        const int n = min(kMergeChunk, p.nsplit - s0);
        __syncthreads();   // weights written; the previous chunk fully read
        for (int i = tid; i < n * rs; i += kMergeThreads) {
            const int s = i / rs, e = i - s * rs;
            cp_async4(chunk + i, rec + (s0 + s) * split_stride + e);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        for (int s = 0; s < n; ++s) {
            const float ls = chunk[s * rs + 1], w = wts[s0 + s];
            bad |= !isfinite(ls);
            l = fmaf(ls, w, l);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int d = tid + r * kMergeThreads;
                if (d < hd) a[r] = fmaf(chunk[s * rs + 2 + d], w, a[r]);
            }
        }
    }
    float o[2] = {0.0f, 0.0f};
    for (int r = 0; r < 2; ++r) {
        const int d = tid + r * kMergeThreads;
        if (d < hd) {
            bad |= !isfinite(a[r]);
            o[r] = a[r] / l;
        }
    }
    if (__syncthreads_or(bad) || !isfinite(l) || l <= 0.0f) {
        const int T = p.tokens_dev ? *p.tokens_dev : p.tokens;
        head_fp64(p, head, T, sbuf, p.out + (long long)head * hd);
    } else {
        for (int r = 0; r < 2; ++r) {
            const int d = tid + r * kMergeThreads;
            if (d < hd) p.out[(long long)head * hd + d] = o[r];
        }
    }
}

template <int DPL, bool VEC4, int GMAX>
cudaError_t launch_partial(const AttnParams &p, dim3 grid, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kWarps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_partial_kernel<DPL, VEC4, GMAX>, p);
}

template <int DPL, bool VEC4>
cudaError_t launch_partial_g(const AttnParams &p, int gmax, dim3 grid, cudaStream_t stream)
{
    switch (gmax) {
    case 1: return launch_partial<DPL, VEC4, 1>(p, grid, stream);
    case 2: return launch_partial<DPL, VEC4, 2>(p, grid, stream);
    case 4: return launch_partial<DPL, VEC4, 4>(p, grid, stream);
    default: return launch_partial<DPL, VEC4, 8>(p, grid, stream);
    }
}

int gmax_for(int group) { return group >= 8 ? 8 : group > 2 ? (group > 4 ? 8 : 4) : group; }

// ---------------------------------------------------------------- RoPE + append
__global__ void rope_append_kernel(RopeAppendArgs a)
{
    if (a.use_pdl) {
        pdl_launch_dependents();
        pdl_wait();
    }
    const int z = blockIdx.y;
    const int pos = (a.position_dev ? *a.position_dev : a.position) + z;
    const int hd = a.head_dim, half = a.rotary / 2;
    const int qw = a.q_heads * hd, kvw = a.kv_heads * hd;
    if (z > 0) {
        a.q += z * a.in_stride;
        a.k += z * a.in_stride;
        a.v += z * a.in_stride;
        a.q_out += (long long)z * qw;
        if (a.table) a.table += (long long)z * a.rotary;
    }
    float *kslot = a.k_cache + (long long)pos * kvw;
    float *vslot = a.v_cache + (long long)pos * kvw;
    // TransformerOps.RopeHalf (TransformerOps.cs:99-118): FP64 angle and rotation, FP32 result.
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < qw + 2 * kvw; i += gridDim.x * blockDim.x) {
        if (i < qw + kvw) {
            const bool isq = i < qw;
            const int e = isq ? i : i - qw;
            const float *src = isq ? a.q : a.k;
            float *dst = isq ? a.q_out : kslot;
            const int d = e % hd, base_i = e - d;
            float r;
            if (d < a.rotary) {
                const int k = d < half ? d : d - half;
                double sn, cs;
                if (a.table) {
                    cs = a.table[2 * k];
                    sn = a.table[2 * k + 1];
                } else {
                    const double angle = __ddiv_rn((double)pos, pow(a.base, __ddiv_rn(2.0 * k, (double)a.rotary)));
                    sincos(angle, &sn, &cs);
                }
                const double x = src[base_i + k], y = src[base_i + k + half];
                r = d < half ? (float)__dsub_rn(__dmul_rn(x, cs), __dmul_rn(y, sn))
                             : (float)__dadd_rn(__dmul_rn(x, sn), __dmul_rn(y, cs));
            } else {
                r = src[e];
            }
            dst[e] = r;
        } else {
            const int e = i - qw - kvw;
            vslot[e] = a.v[e];
        }
    }
}

__global__ void rope_half_kernel(float *v, int n, int hd, int pos, double base, int rotary)
{
    const int half = rotary / 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n / hd * half; i += gridDim.x * blockDim.x) {
        const int head = i / half, k = i - head * half;
        const double angle = __ddiv_rn((double)pos, pow(base, __ddiv_rn(2.0 * k, (double)rotary)));
        double sn, cs;
        sincos(angle, &sn, &cs);
        float *h = v + (long long)head * hd;
        const double x = h[k], y = h[k + half];
        h[k] = (float)__dsub_rn(__dmul_rn(x, cs), __dmul_rn(y, sn));
        h[k + half] = (float)__dadd_rn(__dmul_rn(x, sn), __dmul_rn(y, cs));
    }
}

}  // namespace

int attn_splits(int q_heads, int kv_heads, int head_dim, int max_tokens, int sm_count, int batch)
{
    const int group = q_heads / kv_heads;
    const int gmax = gmax_for(group);
    const int ngroups = (group + gmax - 1) / gmax;
    const int units = kv_heads * ngroups * std::max(1, batch);
    int nsplit = std::max(1, (3 * sm_count + units - 1) / units);
    nsplit = std::min(nsplit, std::max(1, max_tokens / (2 * kTokBlock)));
    (void)head_dim;
    return nsplit;
}

// Splits of the prefill kernel: about two CTAs per SM over (KV head group, 8-position block, split),
// at least 64 tokens per split of the longest prefix.
int attn_prefill_splits(int q_heads, int kv_heads, int max_tokens, int sm_count, int batch)
{
    const int group = q_heads / kv_heads;
    const int units = kv_heads * ((group + 7) / 8) * ((batch + kPrefillPos - 1) / kPrefillPos);
    int nsplit = std::max(1, (2 * sm_count + units - 1) / units);
    return std::min(nsplit, std::max(1, max_tokens / 64));
}

size_t attn_scratch_floats(int q_heads, int kv_heads, int head_dim, int max_tokens, int sm_count, int batch)
{
    int splits = attn_splits(q_heads, kv_heads, head_dim, max_tokens, sm_count, batch);
    if (batch > 1) splits = std::max(splits, attn_prefill_splits(q_heads, kv_heads, max_tokens, sm_count, batch));
    return (size_t)splits * q_heads * (head_dim + 2) * std::max(1, batch);
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn attn_encode_fn()
{
    static EncodeTiledFn fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// K or V cache of one layer as a 3-D FP32 tensor [tokens][kv_heads][128] (token rows kv_stride floats
// apart), boxes of 8 tokens x 1 head.
bool encode_kv_map(CUtensorMap *map, const float *base, int kv_heads, int kv_stride, int tokens)
{
    EncodeTiledFn enc = attn_encode_fn();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) || (kv_stride % 4) != 0) return false;
    const cuuint64_t dims[3] = {128, (cuuint64_t)kv_heads, (cuuint64_t)tokens};
    const cuuint64_t strides[2] = {128 * 4, (cuuint64_t)kv_stride * 4};
    const cuuint32_t box[3] = {128, 1, (cuuint32_t)kStreamTok};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The streaming kernel takes head_dim 128 with groups of 5..8 (or more) query heads per KV head.
// Returns false (nothing launched) when the shape or pointers do not qualify.
bool launch_stream(const AttnArgs &a, AttnParams &p, int gmax, int sm_count, cudaStream_t stream, cudaError_t *err)
{
    if (a.head_dim != 128 || gmax != 8) return false;
    const int units = a.kv_heads * p.ngroups;
    const int cap = std::max(a.max_tokens, a.tokens + p.batch - 1);
    CUtensorMap kmap, vmap;
    if (!encode_kv_map(&kmap, a.keys, a.kv_heads, p.kv_stride, cap) ||
        !encode_kv_map(&vmap, a.values, a.kv_heads, p.kv_stride, cap))
        return false;
    if (p.batch > 1) {
        // A prefill chunk: 8 positions per CTA share every K/V tile.
        p.nsplit = attn_prefill_splits(a.q_heads, a.kv_heads, a.tokens + p.batch - 1, sm_count, p.batch);
        const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(attn_prefill_kernel), kStreamSmem);
        if (e != cudaSuccess) {
            *err = e;
            return true;
        }
        attn_prefill_kernel<<<dim3(p.nsplit, units, (p.batch + kPrefillPos - 1) / kPrefillPos),
                              (kStreamWarps + 1) * 32, kStreamSmem, stream>>>(kmap, vmap, p);
        *err = cudaGetLastError();
        return true;
    }
    // About one CTA per SM (each keeps ~64 KB in flight); never more splits than the scratch holds.
    p.nsplit = std::max(1, std::min(p.nsplit, (sm_count + units * p.batch - 1) / (units * p.batch)));
    // At least 128 tokens per split (two 8-token tiles per compute warp, so the CTA-level merge of the
    // warps' states is shared by twice the work), unless that would leave fewer than about half as many
    // CTAs as SMs: short contexts keep their 64-token splits.
    p.nsplit = std::max(1, std::min(p.nsplit, std::max(cap / 128, (sm_count + 2 * units - 1) / (2 * units))));
    const cudaError_t e = opt_in_smem(reinterpret_cast<const void *>(attn_stream_kernel), kStreamSmem);
    if (e != cudaSuccess) {
        *err = e;
        return true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.nsplit, units, p.batch);
    cfg.blockDim = dim3((kStreamWarps + 1) * 32);
    cfg.dynamicSmemBytes = kStreamSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.use_pdl ? 1 : 0;
    *err = cudaLaunchKernelEx(&cfg, attn_stream_kernel, kmap, vmap, p);
    return true;
}
}  // namespace

cudaError_t launch_attention(const AttnArgs &a, int sm_count, cudaStream_t stream)
{
    if (a.head_dim <= 0 || a.head_dim > 256 || a.q_heads % a.kv_heads != 0) return cudaErrorInvalidValue;
    const int batch = std::max(1, a.batch);
    if (batch > 1 && (a.tokens_dev || a.tokens < 1 || batch > 65535)) return cudaErrorInvalidValue;
    AttnParams p;
    p.q = a.q;
    p.keys = a.keys;
    p.values = a.values;
    p.q_heads = a.q_heads;
    p.kv_heads = a.kv_heads;
    p.head_dim = a.head_dim;
    p.group = a.q_heads / a.kv_heads;
    p.kv_stride = a.kv_stride > 0 ? a.kv_stride : a.kv_heads * a.head_dim;
    const int gmax = gmax_for(p.group);
    p.ngroups = (p.group + gmax - 1) / gmax;
    p.tokens = a.tokens;
    p.tokens_dev = a.tokens_dev;
    p.nsplit = attn_splits(a.q_heads, a.kv_heads, a.head_dim, a.max_tokens, sm_count, batch);
    p.batch = batch;
    p.q_pstride = a.q_pstride;
    p.out_pstride = a.out_pstride;
    p.scale = (float)(1.0 / std::sqrt((double)a.head_dim));
    p.scratch = a.scratch;
    p.out = a.out;
    p.use_pdl = a.use_pdl;
    p.err = a.err;
    cudaError_t e;
    if (!launch_stream(a, p, gmax, sm_count, stream, &e)) {
        const dim3 grid(p.nsplit, a.kv_heads * p.ngroups, batch);
        if (a.head_dim == 128) e = launch_partial_g<4, true>(p, gmax, grid, stream);
        else e = launch_partial_g<8, false>(p, gmax, grid, stream);
    }
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.q_heads, batch);
    cfg.blockDim = dim3(kMergeThreads);
    cfg.dynamicSmemBytes = sizeof(float) * ((size_t)((p.nsplit + 3) & ~3) + (size_t)kMergeChunk * (a.head_dim + 2));
    const cudaError_t ea = opt_in_smem(reinterpret_cast<const void *>(attn_merge_kernel), cfg.dynamicSmemBytes);
    if (ea != cudaSuccess) return ea;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_merge_kernel, p);
}

cudaError_t launch_rope_append(const RopeAppendArgs &a, cudaStream_t stream)
{
    const int n = (a.q_heads + 2 * a.kv_heads) * a.head_dim;
    const int batch = std::max(1, a.batch);
    if (batch > 1 && (a.position_dev || batch > 65535)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.table ? (n + 255) / 256 : 1, batch);
    cfg.blockDim = dim3(a.table ? 256 : 512);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.use_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rope_append_kernel, a);
}

cudaError_t launch_rope_half(float *v, int n, int head_dim, int position, double base, int rotary,
                             cudaStream_t stream)
{
    rope_half_kernel<<<4, 256, 0, stream>>>(v, n, head_dim, position, base, rotary);
    return cudaGetLastError();
}

}  // namespace satori
