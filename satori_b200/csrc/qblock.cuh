// qblock.cuh -- one GGUF Q8_0 / Q4_0 block term in the reference's decode (ExecuteBatch) order.
//
// QuantizedMatVec.Dot (QuantizedMatVec.cs:300-365) reduces a 32-weight block with eight FMA lanes
// (lane l accumulates weights l, l+8, l+16, l+24 in that order, starting from 0) and the SSE horizontal
// sum ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)); the weights are QuantizedRow.DecodeQ8Block / DecodeQ4Block
// (scale * code).  block_term reproduces that bit for bit with packed FP32x2 lanes.
#pragma once

#include "common.cuh"

namespace satori {

__host__ __device__ constexpr int blk_bytes(int fmt) { return fmt == 0 ? 34 : 18; }

// Float pair of two code bytes `b0`, `b1` of `word`: each byte lands in bits 8..15 under the 2^23
// exponent, f = 2^23 + 256 * byte.  fma(f, s, c) with s = d/256 (or d/4096 for a high nibble kept
// in place) and c = -d * (2^15 + bias) (or -d * (2^11 + bias)) is exactly d * (code - bias): d has at
// most 11 significant bits, so s and c are exact and the exact result is representable.
__device__ __forceinline__ float2 code_pair(uint32_t word, int b0, int b1)
{
    return make_float2(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7404u | ((uint32_t)b0 << 4))),
                       __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7404u | ((uint32_t)b1 << 4))));
}

// One block term.  `w` = the block's words starting at the word holding its first byte; PH = byte
// offset of the block inside w[0] (0 or 2), so code byte i of the block is byte PH + 2 + i from w[0].
// `xv` = the block's 32 activations (xv[q] holds floats 4q .. 4q+3).
template <int FMT, int PH>
__device__ __forceinline__ float block_term(const uint32_t *w, const float4 (&xv)[8])
{
    const float d = half_bits_to_float(PH == 0 ? w[0] : w[0] >> 16);
    float2 S0, C0, S1, C1;
    if (FMT == 0) {
        const float s = fmul(d, 0.00390625f), c = fmul(d, -32896.0f);   // 2^-8, -(2^15 + 128)
        S0 = S1 = make_float2(s, s);
        C0 = C1 = make_float2(c, c);
    } else {
        const float s = fmul(d, 0.00390625f), c = fmul(d, -32776.0f);   // low nibble: 2^-8, -(2^15 + 8)
        const float sh = fmul(d, 0.000244140625f), ch = fmul(d, -2056.0f);  // high nibble: 2^-12, -(2^11 + 8)
        S0 = make_float2(s, s);
        C0 = make_float2(c, c);
        S1 = make_float2(sh, sh);
        C1 = make_float2(ch, ch);
    }
    float2 A[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const float2 X[4] = {make_float2(xv[2 * g].x, xv[2 * g].y), make_float2(xv[2 * g].z, xv[2 * g].w),
                             make_float2(xv[2 * g + 1].x, xv[2 * g + 1].y),
                             make_float2(xv[2 * g + 1].z, xv[2 * g + 1].w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // Dot lanes (2i, 2i+1) of group g: weights 8g + 2i, 8g + 2i + 1.
            float2 W;
            if (FMT == 0) {
                const int cb = PH + 2 + 8 * g + 2 * i;                  // byte of code 8g + 2i from w[0]
                const uint32_t u = w[cb >> 2] ^ 0x80808080u;            // biased: u = code + 128
                W = __ffma2_rn(code_pair(u, cb & 3, (cb & 3) + 1), S0, C0);
            } else {
                // Weights 0..15 are the low nibbles of code bytes 0..15, weights 16..31 the high ones.
                const int cb = PH + 2 + 8 * (g & 1) + 2 * i;
                const uint32_t word = w[cb >> 2];
                if (g < 2)
                    W = __ffma2_rn(code_pair(word & 0x0F0F0F0Fu, cb & 3, (cb & 3) + 1), S0, C0);
                else
                    W = __ffma2_rn(code_pair(word & 0xF0F0F0F0u, cb & 3, (cb & 3) + 1), S1, C1);
            }
            A[i] = __ffma2_rn(W, X[i], g == 0 ? make_float2(0.0f, 0.0f) : A[i]);
        }
    }
    const float2 h01 = __fadd2_rn(A[0], A[2]);  // (a0+a4, a1+a5)
    const float2 h23 = __fadd2_rn(A[1], A[3]);  // (a2+a6, a3+a7)
    const float2 g01 = __fadd2_rn(h01, h23);
    return fadd(g01.x, g01.y);
}

}  // namespace satori
