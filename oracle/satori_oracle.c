/*
 * satori_oracle.c -- CPU restatement of the Satori decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker; never the product).  See
 * satori_oracle.h for the contract.  Build: oracle/build.py (gcc -O2
 * -ffp-contract=off -mavx2 -mfma -fopenmp).  Parity of this restatement is
 * pinned by tests/test_oracle_golden.py against the reference's fixtures.
 *
 * Reference paths below are relative to the reference project root.
 */
#include "satori_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* helpers                                                                   */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline float rdf32(const uint8_t *p) { float f; memcpy(&f, p, 4); return f; }
static inline int isfinite_f(float f) { return (f2u(f) & 0x7f800000u) != 0x7f800000u; }

/* Exact IEEE binary16 -> binary32 (BitConverter.UInt16BitsToHalf + (float) cast,
 * QuantizedMatVec.cs:369). */
float so_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    if (exp == 0) {
        if (mant == 0) return u2f(sign);
        float f = (float)mant * 5.9604644775390625e-8f; /* mant * 2^-24, exact */
        return u2f(sign | f2u(f));
    }
    if (exp == 31) return u2f(sign | 0x7f800000u | (mant << 13));
    return u2f(sign | ((exp + 112u) << 23) | (mant << 13));
}

/* binary32 -> binary16, round to nearest even (used by fixtures and the quantizer only). */
uint16_t so_float_to_half(float value)
{
    uint32_t x = f2u(value);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (absx < 0x38800000u) { /* subnormal half or zero */
        float f = u2f(absx) * 16777216.0f;  /* scale by 2^24: exact */
        uint32_t m = (uint32_t)f;           /* truncated */
        float rem = f - (float)m;
        if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t e = ((absx >> 23) - 112u) << 10;
    uint32_t m = (absx >> 13) & 0x3ffu;
    uint32_t r = absx & 0x1fffu;
    uint32_t h = e | m;
    if (r > 0x1000u || (r == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* SSE horizontal sum used by every reference AVX2 kernel:
 * QuantizedKAvx2Kernel.HorizontalSum (QuantizedKAvx2Kernel.cs:341-347) and the
 * inline copies in Ternary2Avx2Kernel.cs:42-45 / QuantizedAvx2Kernel.cs:46-48. */
static inline float hsum256(__m256 v)
{
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    h = _mm_add_ps(h, _mm_shuffle_ps(h, h, 0x4e));
    h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 0xb1));
    return _mm_cvtss_f32(h);
}

/* The same reduction on eight scalar lanes: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)). */
static inline float hsum8(const float a[8])
{
    float h0 = a[0] + a[4], h1 = a[1] + a[5], h2 = a[2] + a[6], h3 = a[3] + a[7];
    float g0 = h0 + h2, g1 = h1 + h3;
    return g0 + g1;
}

static int clamp_threads(int threads) { return threads < 1 ? 1 : threads; }

/* ------------------------------------------------------------------------- */
/* Ternary2                                                                  */
/* ------------------------------------------------------------------------- */

/* Ternary2Shape.cs:5-22 */
int so_t2_geometry(int rows, int cols, int bs, int *blocks_per_row, int *block_bytes, int64_t *byte_length)
{
    if (rows <= 0 || cols <= 0) return SO_ERR_ARGUMENT;
    if (bs != 64 && bs != 128 && bs != 256) return SO_ERR_ARGUMENT;
    int64_t bpr = ((int64_t)cols + bs - 1) / bs;
    int64_t len = (int64_t)rows * bpr * (4 + bs / 4);
    if (len > 0x7fffffffLL) return SO_ERR_ARGUMENT; /* checked((int)...) */
    if (blocks_per_row) *blocks_per_row = (int)bpr;
    if (block_bytes) *block_bytes = 4 + bs / 4;
    if (byte_length) *byte_length = len;
    return SO_OK;
}

/* Ternary2Matrix.Quantize (Ternary2Matrix.cs:38-71) */
int so_t2_quantize(const float *w, int rows, int cols, int bs, uint8_t *out)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    for (int64_t i = 0; i < (int64_t)rows * cols; i++)
        if (!isfinite_f(w[i])) return SO_ERR_ARGUMENT;
    memset(out, 0, (size_t)len);
    for (int row = 0; row < rows; row++)
        for (int block = 0; block < bpr; block++) {
            int column = block * bs;
            int count = bs < cols - column ? bs : cols - column;
            const float *src = w + (int64_t)row * cols + column;
            double magnitude = 0;
            for (int i = 0; i < count; i++) magnitude += fabs((double)src[i]);
            float scale = (float)(magnitude / count);
            uint8_t *t = out + ((int64_t)row * bpr + block) * bb;
            memcpy(t, &scale, 4);
            if (scale == 0) continue;
            double threshold = (double)scale / 2;
            for (int i = 0; i < count; i++) {
                int code = (double)src[i] > threshold ? 1 : (double)src[i] < -threshold ? 2 : 0;
                t[4 + i / 4] |= (uint8_t)(code << (2 * (i % 4)));
            }
        }
    return SO_OK;
}

/* Ternary2Matrix.ValidatePayload (Ternary2Matrix.cs:83-101) plus the length check of
 * FromPacked (:75-76). */
int so_t2_validate(const uint8_t *data, int64_t len, int rows, int cols, int bs)
{
    int bpr, bb; int64_t want;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &want);
    if (rc) return rc;
    if (len != want) return SO_ERR_ARGUMENT;
    for (int row = 0; row < rows; row++)
        for (int block = 0; block < bpr; block++) {
            const uint8_t *b = data + ((int64_t)row * bpr + block) * bb;
            float scale = rdf32(b);
            if (!isfinite_f(scale) || scale < 0 || f2u(scale) == 0x80000000u) return SO_ERR_ARGUMENT;
            int count = bs < cols - block * bs ? bs : cols - block * bs;
            for (int i = 0; i < bs; i++) {
                int code = (b[4 + i / 4] >> (2 * (i % 4))) & 3;
                if (code == 3 || ((i >= count || scale == 0) && code != 0)) return SO_ERR_ARGUMENT;
            }
        }
    return SO_OK;
}

/* Ternary2Matrix.Dequantize (Ternary2Matrix.cs:103-120) */
int so_t2_dequantize(const uint8_t *data, int rows, int cols, int bs, float *out)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    for (int row = 0; row < rows; row++)
        for (int block = 0; block < bpr; block++) {
            const uint8_t *b = data + ((int64_t)row * bpr + block) * bb;
            float scale = rdf32(b);
            int column = block * bs;
            int count = bs < cols - column ? bs : cols - column;
            for (int i = 0; i < count; i++) {
                int code = (b[4 + i / 4] >> (2 * (i % 4))) & 3;
                out[(int64_t)row * cols + column + i] = code == 1 ? scale : code == 2 ? -scale : 0.0f;
            }
        }
    return SO_OK;
}

/* Ternary2MatVec.ExecuteScalarCore (Ternary2MatVec.cs:52-76) */
int so_t2_matvec_scalar(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    for (int row = 0; row < rows; row++) {
        float sum = 0;
        for (int block = 0; block < bpr; block++) {
            const uint8_t *b = data + ((int64_t)row * bpr + block) * bb;
            float scale = rdf32(b);
            int column = block * bs;
            int count = bs < cols - column ? bs : cols - column;
            float partial = 0;
            for (int i = 0; i < count; i++) {
                int code = (b[4 + i / 4] >> (2 * (i % 4))) & 3;
                if (code == 1) partial += x[column + i];
                else if (code == 2) partial -= x[column + i];
            }
            sum += partial * scale;
        }
        y[row] = sum;
    }
    return SO_OK;
}

/* One row of Ternary2Avx2Kernel.Execute (Ternary2Avx2Kernel.cs:10-56), same instruction
 * sequence: variable shifts of the 16-bit code group, zero/negative masks, sign XOR, AndNot,
 * eight-lane add, fixed horizontal sum, scalar tail, then sum += partial * scale. */
static void t2_avx2_row(const uint8_t *data, int row, int cols, int bs, int bpr, int bb, const float *x, float *y)
{
    const __m256i shifts = _mm256_setr_epi32(0, 2, 4, 6, 8, 10, 12, 14);
    const __m256i mask = _mm256_set1_epi32(3);
    const __m256i negative_code = _mm256_set1_epi32(2);
    const __m256i sign_bit = _mm256_set1_epi32((int)0x80000000u);
    float sum = 0;
    for (int block = 0; block < bpr; block++) {
        const uint8_t *b = data + ((int64_t)row * bpr + block) * bb;
        float scale = rdf32(b);
        int column = block * bs;
        int count = bs < cols - column ? bs : cols - column;
        __m256 acc = _mm256_setzero_ps();
        int i = 0;
        for (; i <= count - 8; i += 8) {
            uint32_t packed = rd16(b + 4 + i / 4);
            __m256i codes = _mm256_and_si256(_mm256_srlv_epi32(_mm256_set1_epi32((int)packed), shifts), mask);
            __m256i zero = _mm256_cmpeq_epi32(codes, _mm256_setzero_si256());
            __m256i neg = _mm256_and_si256(_mm256_cmpeq_epi32(codes, negative_code), sign_bit);
            __m256 act = _mm256_loadu_ps(x + column + i);
            __m256 sgn = _mm256_xor_ps(act, _mm256_castsi256_ps(neg));
            acc = _mm256_add_ps(acc, _mm256_andnot_ps(_mm256_castsi256_ps(zero), sgn));
        }
        float partial = hsum256(acc);
        for (; i < count; i++) {
            int code = (b[4 + i / 4] >> (2 * (i % 4))) & 3;
            if (code == 1) partial += x[column + i];
            else if (code == 2) partial -= x[column + i];
        }
        sum += partial * scale;
    }
    y[row] = sum;
}

int so_t2_matvec_avx2(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y, int threads)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    /* Rows are independent: a row split cannot change the result (QuantizedMatVec.cs:245-263). */
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (int row = 0; row < rows; row++) t2_avx2_row(data, row, cols, bs, bpr, bb, x, y);
    return SO_OK;
}

/* Scalar emulation of the AVX2 lane order; used to cross-check the intrinsic version. */
int so_t2_matvec_avx2_emulated(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    for (int row = 0; row < rows; row++) {
        float sum = 0;
        for (int block = 0; block < bpr; block++) {
            const uint8_t *b = data + ((int64_t)row * bpr + block) * bb;
            float scale = rdf32(b);
            int column = block * bs;
            int count = bs < cols - column ? bs : cols - column;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int i = 0;
            for (; i <= count - 8; i += 8) {
                uint32_t packed = rd16(b + 4 + i / 4);
                for (int l = 0; l < 8; l++) {
                    int code = (packed >> (2 * l)) & 3;
                    float v = x[column + i + l];
                    float t = code == 0 ? 0.0f : code == 2 ? u2f(f2u(v) ^ 0x80000000u) : v;
                    a[l] = a[l] + t;
                }
            }
            float partial = hsum8(a);
            for (; i < count; i++) {
                int code = (b[4 + i / 4] >> (2 * (i % 4))) & 3;
                if (code == 1) partial += x[column + i];
                else if (code == 2) partial -= x[column + i];
            }
            sum += partial * scale;
        }
        y[row] = sum;
    }
    return SO_OK;
}

/* Ternary2FileFormat.WriteHeader (Ternary2FileFormat.cs:9-19) */
void so_stq2_write_header(uint8_t h[32], int rows, int cols, int bs)
{
    int64_t len = 0;
    so_t2_geometry(rows, cols, bs, NULL, NULL, &len);
    memset(h, 0, 32);
    memcpy(h, "STQ2", 4);
    h[4] = 1; h[5] = 0;
    h[6] = 32; h[7] = 0;
    memcpy(h + 8, &rows, 4);
    memcpy(h + 12, &cols, 4);
    memcpy(h + 16, &bs, 4);
    memcpy(h + 24, &len, 8);
}

/* Ternary2FileFormat.ReadHeader (Ternary2FileFormat.cs:21-35) plus the whole-file length
 * check of MappedTernary2Matrix (MappedTernary2Matrix.cs:13-23); every failure maps to
 * InvalidDataException as the mapped constructor rethrows it (:25-28). */
int so_stq2_read_header(const uint8_t *h, int64_t file_len, int *rows, int *cols, int *bs)
{
    if (file_len < 32) return SO_ERR_INVALID_DATA;
    if (memcmp(h, "STQ2", 4) != 0 || rd16(h + 4) != 1 || rd16(h + 6) != 32) return SO_ERR_INVALID_DATA;
    int32_t r, c, b, pad; int64_t len, want;
    memcpy(&pad, h + 20, 4);
    if (pad != 0) return SO_ERR_INVALID_DATA;
    memcpy(&r, h + 8, 4); memcpy(&c, h + 12, 4); memcpy(&b, h + 16, 4); memcpy(&len, h + 24, 8);
    if (so_t2_geometry(r, c, b, NULL, NULL, &want) != SO_OK) return SO_ERR_INVALID_DATA;
    if (len != want) return SO_ERR_INVALID_DATA;
    if (file_len != 32 + want) return SO_ERR_INVALID_DATA;
    *rows = r; *cols = c; *bs = b;
    return SO_OK;
}

/* ------------------------------------------------------------------------- */
/* GGUF Q8_0 / Q4_0                                                          */
/* ------------------------------------------------------------------------- */

/* QuantizedMatrixShape.cs:5-22 (Q8_0: 32 weights in 34 bytes, Q4_0: 32 in 18). */
int so_q_geometry(int rows, int cols, int fmt, int *block_bytes, int64_t *byte_length)
{
    int bb;
    if (fmt == SO_Q8_0) bb = 34;
    else if (fmt == SO_Q4_0) bb = 18;
    else return SO_ERR_ARGUMENT;
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return SO_ERR_ARGUMENT;
    int64_t len = (int64_t)rows * (cols / 32) * bb;
    if (len > 0x7fffffffLL) return SO_ERR_ARGUMENT;
    if (block_bytes) *block_bytes = bb;
    if (byte_length) *byte_length = len;
    return SO_OK;
}

/* QuantizedMatVec.ValidatePayload (QuantizedMatVec.cs:28-42) */
int so_q_validate(const uint8_t *data, int64_t len, int rows, int cols, int fmt)
{
    int bb; int64_t want;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &want);
    if (rc) return rc;
    if (len != want) return SO_ERR_ARGUMENT;
    for (int64_t off = 0; off < len; off += bb)
        if (!isfinite_f(so_half_to_float(rd16(data + off)))) return SO_ERR_INVALID_DATA;
    return SO_OK;
}

/* QuantizedRow.DecodeQ8Block / DecodeQ4Block (QuantizedRow.cs:20-37) */
static void q_decode_block(const uint8_t *b, int fmt, float out[32])
{
    float scale = so_half_to_float(rd16(b));
    if (fmt == SO_Q8_0) {
        for (int j = 0; j < 32; j++) out[j] = scale * (float)(int8_t)b[2 + j];
    } else {
        for (int j = 0; j < 16; j++) {
            out[j] = scale * (float)((b[2 + j] & 15) - 8);
            out[j + 16] = scale * (float)((b[2 + j] >> 4) - 8);
        }
    }
}

/* QuantizedRow.DecodeRow (QuantizedRow.cs:60-70) */
int so_q_decode_row(const uint8_t *row_bytes, int cols, int fmt, float *out)
{
    int bb;
    if (so_q_geometry(1, cols, fmt, &bb, NULL)) return SO_ERR_ARGUMENT;
    for (int b = 0; b < cols / 32; b++) q_decode_block(row_bytes + (int64_t)b * bb, fmt, out + b * 32);
    return SO_OK;
}

/* QuantizedMatVec.ExecuteScalar (QuantizedMatVec.cs:45-78) */
int so_q_matvec_scalar(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    int bpr = cols / 32;
    for (int row = 0; row < rows; row++) {
        float total = 0;
        for (int column = 0; column < cols; column += 32) {
            const uint8_t *b = data + ((int64_t)row * bpr + column / 32) * bb;
            float sum = 0;
            if (fmt == SO_Q8_0) {
                for (int j = 0; j < 32; j++) sum += (float)(int8_t)b[2 + j] * x[column + j];
            } else {
                for (int j = 0; j < 16; j++) sum += (float)((b[2 + j] & 15) - 8) * x[column + j];
                for (int j = 0; j < 16; j++) sum += (float)((b[2 + j] >> 4) - 8) * x[column + 16 + j];
            }
            total += so_half_to_float(rd16(b)) * sum;
        }
        y[row] = total;
    }
    return SO_OK;
}

/* One row of QuantizedAvx2Kernel.Execute (QuantizedAvx2Kernel.cs:10-53): unscaled codes times
 * activations, multiply then add (no FMA), fixed horizontal sum, total += scale * partial. */
static void q_avx2_row(const uint8_t *data, int row, int cols, int fmt, int bb, const float *x, float *y)
{
    const __m256i nibble_mask = _mm256_set1_epi32(15);
    const __m256i bias = _mm256_set1_epi32(8);
    int bpr = cols / 32;
    float total = 0;
    for (int blk = 0; blk < bpr; blk++) {
        const uint8_t *b = data + ((int64_t)row * bpr + blk) * bb;
        __m256 acc = _mm256_setzero_ps();
        if (fmt == SO_Q8_0) {
            for (int j = 0; j < 32; j += 8) {
                uint64_t packed; memcpy(&packed, b + 2 + j, 8);
                __m256 codes = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_cvtsi64_si128((long long)packed)));
                __m256 values = _mm256_loadu_ps(x + blk * 32 + j);
                acc = _mm256_add_ps(acc, _mm256_mul_ps(codes, values));
            }
        } else {
            for (int j = 0; j < 16; j += 8) {
                uint64_t packed; memcpy(&packed, b + 2 + j, 8);
                __m256i codes = _mm256_cvtepu8_epi32(_mm_cvtsi64_si128((long long)packed));
                __m256 low = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_and_si256(codes, nibble_mask), bias));
                __m256 high = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_srli_epi32(codes, 4), bias));
                acc = _mm256_add_ps(acc, _mm256_mul_ps(low, _mm256_loadu_ps(x + blk * 32 + j)));
                acc = _mm256_add_ps(acc, _mm256_mul_ps(high, _mm256_loadu_ps(x + blk * 32 + j + 16)));
            }
        }
        total += so_half_to_float(rd16(b)) * hsum256(acc);
    }
    y[row] = total;
}

int so_q_matvec_avx2(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y, int threads)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (int row = 0; row < rows; row++) q_avx2_row(data, row, cols, fmt, bb, x, y);
    return SO_OK;
}

int so_q_matvec_avx2_emulated(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    int bpr = cols / 32;
    for (int row = 0; row < rows; row++) {
        float total = 0;
        for (int blk = 0; blk < bpr; blk++) {
            const uint8_t *b = data + ((int64_t)row * bpr + blk) * bb;
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            const float *xs = x + blk * 32;
            if (fmt == SO_Q8_0) {
                for (int j = 0; j < 32; j += 8)
                    for (int l = 0; l < 8; l++) a[l] = a[l] + (float)(int8_t)b[2 + j + l] * xs[j + l];
            } else {
                for (int j = 0; j < 16; j += 8)
                    for (int l = 0; l < 8; l++) {
                        a[l] = a[l] + (float)((b[2 + j + l] & 15) - 8) * xs[j + l];
                        a[l] = a[l] + (float)((b[2 + j + l] >> 4) - 8) * xs[j + 16 + l];
                    }
            }
            total += so_half_to_float(rd16(b)) * hsum8(a);
        }
        y[row] = total;
    }
    return SO_OK;
}

/* QuantizedMatVec.ExecuteBatch -> ExecuteBatchFloat -> ExecuteBatchRows -> Dot
 * (QuantizedMatVec.cs:104-120, 221-281, 308-347, 350-365), FMA host.  Per block the
 * weights are decoded exactly (QuantizedRow.DecodeBlock), dotted with the input window as
 * eight fused-multiply-add lanes, horizontally summed, and accumulator[row] += dot.  Input
 * and output are position-major.  The row tiling and thread split of the reference do not
 * change any row's result. */
static void q_batch_row(const uint8_t *data, int row, int rows, int cols, int fmt, int bb, const float *x,
                        int positions, float *y)
{
    int bpr = cols / 32;
    float w[32];
    for (int p = 0; p < positions; p++) y[(int64_t)p * rows + row] = 0;
    for (int blk = 0; blk < bpr; blk++) {
        q_decode_block(data + ((int64_t)row * bpr + blk) * bb, fmt, w);
        for (int p = 0; p < positions; p++) {
            const float *xs = x + (int64_t)p * cols + blk * 32;
            __m256 sum = _mm256_setzero_ps();
            for (int j = 0; j < 32; j += 8)
                sum = _mm256_fmadd_ps(_mm256_loadu_ps(w + j), _mm256_loadu_ps(xs + j), sum);
            float *acc = y + (int64_t)p * rows + row;
            *acc = *acc + hsum256(sum);
        }
    }
}

int so_q_matvec_batch(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions, float *y,
                      int threads)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    if (positions <= 0) return SO_ERR_ARGUMENT;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (int row = 0; row < rows; row++) q_batch_row(data, row, rows, cols, fmt, bb, x, positions, y);
    return SO_OK;
}

int so_q_matvec_batch_emulated(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions,
                               float *y)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    if (positions <= 0) return SO_ERR_ARGUMENT;
    int bpr = cols / 32;
    float w[32];
    for (int row = 0; row < rows; row++) {
        for (int p = 0; p < positions; p++) y[(int64_t)p * rows + row] = 0;
        for (int blk = 0; blk < bpr; blk++) {
            q_decode_block(data + ((int64_t)row * bpr + blk) * bb, fmt, w);
            for (int p = 0; p < positions; p++) {
                const float *xs = x + (int64_t)p * cols + blk * 32;
                float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int j = 0; j < 32; j += 8)
                    for (int l = 0; l < 8; l++) a[l] = fmaf(w[j + l], xs[j + l], a[l]);
                float *acc = y + (int64_t)p * rows + row;
                *acc = *acc + hsum8(a);
            }
        }
    }
    return SO_OK;
}

/* Not in the reference, which only decodes (the builder's own quantizer, used to build
 * seeded synthetic weights).  Q8_0: d = max|w| / 127, q = round(w / d).  Q4_0: the value m of
 * largest magnitude gives d = m / -8 and q = clamp(floor(w / d + 8.5), 0, 15) -- the
 * block layouts' usual published quantization rule. */
int so_q_quantize(const float *w, int rows, int cols, int fmt, uint8_t *out)
{
    int bb; int64_t len;
    int rc = so_q_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    int bpr = cols / 32;
    for (int row = 0; row < rows; row++)
        for (int blk = 0; blk < bpr; blk++) {
            const float *src = w + (int64_t)row * cols + blk * 32;
            uint8_t *b = out + ((int64_t)row * bpr + blk) * bb;
            if (fmt == SO_Q8_0) {
                float amax = 0;
                for (int j = 0; j < 32; j++) { float a = fabsf(src[j]); if (a > amax) amax = a; }
                float d = amax / 127.0f;
                float id = d != 0 ? 1.0f / d : 0.0f;
                uint16_t h = so_float_to_half(d);
                b[0] = (uint8_t)(h & 0xff); b[1] = (uint8_t)(h >> 8);
                for (int j = 0; j < 32; j++) {
                    float v = roundf(src[j] * id);
                    if (v > 127) v = 127;
                    if (v < -127) v = -127;
                    b[2 + j] = (uint8_t)(int8_t)v;
                }
            } else {
                float amax = 0, m = 0;
                for (int j = 0; j < 32; j++) { float a = fabsf(src[j]); if (a > amax) { amax = a; m = src[j]; } }
                float d = m / -8.0f;
                float id = d != 0 ? 1.0f / d : 0.0f;
                uint16_t h = so_float_to_half(d);
                b[0] = (uint8_t)(h & 0xff); b[1] = (uint8_t)(h >> 8);
                for (int j = 0; j < 16; j++) {
                    int lo = (int)floorf(src[j] * id + 8.5f), hi = (int)floorf(src[j + 16] * id + 8.5f);
                    lo = lo < 0 ? 0 : lo > 15 ? 15 : lo;
                    hi = hi < 0 ? 0 : hi > 15 ? 15 : hi;
                    b[2 + j] = (uint8_t)(lo | (hi << 4));
                }
            }
        }
    return SO_OK;
}

/* ------------------------------------------------------------------------- */
/* operators (TransformerOps.cs)                                             */
/* ------------------------------------------------------------------------- */

/* TransformerOps.RmsNorm (TransformerOps.cs:13-22) */
int so_rmsnorm(const float *x, const float *w, int n, float eps, float *out)
{
    if (n <= 0 || !isfinite_f(eps) || eps <= 0) return SO_ERR_ARGUMENT;
    double sum = 0;
    for (int i = 0; i < n; i++) sum += (double)x[i] * x[i];
    double scale = 1 / sqrt(sum / n + eps);
    for (int i = 0; i < n; i++) out[i] = (float)(x[i] * scale * w[i]);
    return SO_OK;
}

/* TransformerOps.RmsNormHeads (TransformerOps.cs:122-135) */
int so_rmsnorm_heads(float *v, int n, const float *w, float eps, int head_dim)
{
    if (head_dim <= 0 || n % head_dim != 0) return SO_ERR_ARGUMENT;
    if (!isfinite_f(eps) || eps <= 0) return SO_ERR_ARGUMENT;
    for (int start = 0; start < n; start += head_dim) {
        double sum = 0;
        for (int i = 0; i < head_dim; i++) sum += (double)v[start + i] * v[start + i];
        double scale = 1 / sqrt(sum / head_dim + eps);
        for (int i = 0; i < head_dim; i++) v[start + i] = (float)(v[start + i] * scale * w[i]);
    }
    return SO_OK;
}

/* TransformerOps.RopeHalf (TransformerOps.cs:99-118), NeoX half split. */
int so_rope_half(float *v, int n, int head_dim, int position, double base, int rotary)
{
    if (head_dim <= 0 || n % head_dim != 0 || position < 0) return SO_ERR_ARGUMENT;
    if (!isfinite(base) || base <= 0) return SO_ERR_ARGUMENT;
    if (rotary <= 0 || rotary > head_dim || rotary % 2 != 0) return SO_ERR_ARGUMENT;
    int half = rotary / 2;
    for (int k = 0; k < half; k++) {
        double angle = position / pow(base, 2.0 * k / rotary);
        double s = sin(angle), c = cos(angle);
        for (int start = 0; start < n; start += head_dim) {
            double a = v[start + k], b = v[start + k + half];
            v[start + k] = (float)(a * c - b * s);
            v[start + k + half] = (float)(a * s + b * c);
        }
    }
    return SO_OK;
}

/* TransformerOps.Rope (TransformerOps.cs:24-39), interleaved pairs, base 10000. */
int so_rope_interleaved(float *v, int n, int head_dim, int position)
{
    if (head_dim <= 0 || head_dim % 2 != 0 || n % head_dim != 0 || position < 0) return SO_ERR_ARGUMENT;
    for (int j = 0; j < head_dim; j += 2) {
        double angle = position / pow(10000, (double)j / head_dim);
        double s = sin(angle), c = cos(angle);
        for (int start = 0; start < n; start += head_dim) {
            double a = v[start + j], b = v[start + j + 1];
            v[start + j] = (float)(a * c - b * s);
            v[start + j + 1] = (float)(a * s + b * c);
        }
    }
    return SO_OK;
}

/* TransformerOps.SwiGlu (TransformerOps.cs:41-51) */
int so_swiglu(const float *gate, const float *up, int n, float *out)
{
    for (int i = 0; i < n; i++) {
        double x = gate[i];
        double sig = x >= 0 ? 1 / (1 + exp(-x)) : exp(x) / (1 + exp(x));
        out[i] = (float)(x * sig * up[i]);
    }
    return SO_OK;
}

/* TransformerOps.Add (TransformerOps.cs:53-58) */
int so_add(const float *a, const float *b, int n, float *out)
{
    for (int i = 0; i < n; i++) out[i] = a[i] + b[i];
    return SO_OK;
}

/* TransformerOps.GroupedAttention (TransformerOps.cs:140-179).  Heads are independent, so
 * the optional head split over threads cannot change a result; each thread keeps its own
 * score scratch (the caller's scores buffer is used when threads == 1). */
static void gqa_head(const float *q, const float *keys, const float *values, int head, int group, int head_dim,
                     int kv_width, int tokens, double *scores, float *out)
{
    int kv_head = head / group;
    int qo = head * head_dim;
    double scale = 1 / sqrt((double)head_dim);
    double mx = -INFINITY;
    for (int t = 0; t < tokens; t++) {
        const float *k = keys + (int64_t)t * kv_width + kv_head * head_dim;
        double dot = 0;
        for (int j = 0; j < head_dim; j++) dot += (double)q[qo + j] * k[j];
        scores[t] = dot * scale;
        mx = fmax(mx, scores[t]);
    }
    double total = 0;
    for (int t = 0; t < tokens; t++) total += scores[t] = exp(scores[t] - mx);
    for (int j = 0; j < head_dim; j++) {
        double sum = 0;
        for (int t = 0; t < tokens; t++)
            sum += scores[t] / total * values[(int64_t)t * kv_width + kv_head * head_dim + j];
        out[qo + j] = (float)sum;
    }
}

int so_grouped_attention(const float *q, const float *keys, const float *values, int q_heads, int kv_heads,
                         int head_dim, int tokens, double *scores, float *out, int threads)
{
    if (head_dim <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads != 0 || tokens <= 0)
        return SO_ERR_ARGUMENT;
    int group = q_heads / kv_heads;
    int kv_width = kv_heads * head_dim;
    if (clamp_threads(threads) == 1) {
        for (int h = 0; h < q_heads; h++) gqa_head(q, keys, values, h, group, head_dim, kv_width, tokens, scores, out);
        return SO_OK;
    }
#pragma omp parallel num_threads(clamp_threads(threads))
    {
        double *s = (double *)malloc(sizeof(double) * (size_t)tokens);
#pragma omp for schedule(static)
        for (int h = 0; h < q_heads; h++) gqa_head(q, keys, values, h, group, head_dim, kv_width, tokens, s, out);
        free(s);
    }
    return SO_OK;
}

/* GreedyTokenSelector.Select (GreedyTokenSelector.cs:6-16) */
int so_greedy_select(const float *logits, int n, int *token)
{
    if (n <= 0) return SO_ERR_ARGUMENT;
    int best = 0;
    for (int i = 0; i < n; i++) {
        if (!isfinite_f(logits[i])) return SO_ERR_INVALID_DATA;
        if (logits[i] > logits[best]) best = i;
    }
    *token = best;
    return SO_OK;
}

/* ------------------------------------------------------------------------- */
/* dense decode session (DenseSession.cs, DenseForward.cs)                   */
/* ------------------------------------------------------------------------- */

struct so_session {
    const so_model *m;
    int context, position, kv_width, q_width;
    float *keys, *values;   /* [layers][context][kv_width] */
    float *hidden, *normed, *q, *k, *v, *ctx, *proj, *gate, *up, *act, *final_norm;
    double *scores;
};

so_session *so_session_create(const so_model *m, int context)
{
    if (!m || context <= 0) return NULL;
    so_session *s = (so_session *)calloc(1, sizeof(so_session));
    s->m = m;
    s->context = context;
    s->kv_width = m->kv_heads * m->head_dim;
    s->q_width = m->q_heads * m->head_dim;
    size_t slots = (size_t)m->layers * context * s->kv_width;
    s->keys = (float *)calloc(slots, sizeof(float));
    s->values = (float *)calloc(slots, sizeof(float));
    s->hidden = (float *)calloc((size_t)m->hidden, sizeof(float));
    s->normed = (float *)calloc((size_t)m->hidden, sizeof(float));
    s->final_norm = (float *)calloc((size_t)m->hidden, sizeof(float));
    s->q = (float *)calloc((size_t)s->q_width, sizeof(float));
    s->ctx = (float *)calloc((size_t)s->q_width, sizeof(float));
    s->k = (float *)calloc((size_t)s->kv_width, sizeof(float));
    s->v = (float *)calloc((size_t)s->kv_width, sizeof(float));
    s->proj = (float *)calloc((size_t)m->hidden, sizeof(float));
    s->gate = (float *)calloc((size_t)m->ffn, sizeof(float));
    s->up = (float *)calloc((size_t)m->ffn, sizeof(float));
    s->act = (float *)calloc((size_t)m->ffn, sizeof(float));
    s->scores = (double *)calloc((size_t)context, sizeof(double));
    return s;
}

void so_session_destroy(so_session *s)
{
    if (!s) return;
    free(s->keys); free(s->values); free(s->hidden); free(s->normed); free(s->final_norm);
    free(s->q); free(s->ctx); free(s->k); free(s->v); free(s->proj);
    free(s->gate); free(s->up); free(s->act); free(s->scores);
    free(s);
}

void so_session_reset(so_session *s) { s->position = 0; }

/* Benchmark helper (no reference counterpart): fills cache rows [0, position) of every layer with
 * seeded values in [-1, 1) (Xorshift32) and moves the session to `position`, so a decode step at a
 * long context can be timed without running the prompt first.  Decode cost depends only on the
 * context length, not on the cached values. */
int so_session_fill_cache(so_session *s, int position, uint32_t seed)
{
    if (position < 0 || position > s->context) return SO_ERR_ARGUMENT;
    uint32_t x = seed ? seed : 1u;
    for (int l = 0; l < s->m->layers; l++) {
        float *k = s->keys + (size_t)l * s->context * s->kv_width;
        float *v = s->values + (size_t)l * s->context * s->kv_width;
        for (size_t i = 0; i < (size_t)position * s->kv_width; i++) {
            x ^= x << 13; x ^= x >> 17; x ^= x << 5;
            k[i] = (float)(x >> 8) * (1.0f / 8388608.0f) - 1.0f;
            x ^= x << 13; x ^= x >> 17; x ^= x << 5;
            v[i] = (float)(x >> 8) * (1.0f / 8388608.0f) - 1.0f;
        }
    }
    s->position = position;
    return SO_OK;
}
int so_session_position(const so_session *s) { return s->position; }

/* DenseForward.Step (DenseForward.cs:100-162) for one layer at s->position. */
static int dense_step(so_session *s, int layer, int threads)
{
    const so_model *m = s->m;
    const so_layer *L = &m->layer[layer];
    int pos = s->position, kvw = s->kv_width, qw = s->q_width, hd = m->head_dim;
    float *keys = s->keys + (size_t)layer * s->context * kvw;
    float *values = s->values + (size_t)layer * s->context * kvw;
    int rc;
    if ((rc = so_rmsnorm(s->hidden, L->attn_norm, m->hidden, m->eps, s->normed))) return rc;
    if ((rc = so_q_matvec_batch(L->q, qw, m->hidden, L->q_fmt, s->normed, 1, s->q, threads))) return rc;
    if ((rc = so_q_matvec_batch(L->k, kvw, m->hidden, L->k_fmt, s->normed, 1, s->k, threads))) return rc;
    if ((rc = so_q_matvec_batch(L->v, kvw, m->hidden, L->v_fmt, s->normed, 1, s->v, threads))) return rc;
    if (L->q_bias) {
        so_add(s->q, L->q_bias, qw, s->q);
        so_add(s->k, L->k_bias, kvw, s->k);
        so_add(s->v, L->v_bias, kvw, s->v);
    }
    so_rope_half(s->q, qw, hd, pos, m->rope_base, hd);
    so_rope_half(s->k, kvw, hd, pos, m->rope_base, hd);
    memcpy(keys + (size_t)pos * kvw, s->k, sizeof(float) * kvw);
    memcpy(values + (size_t)pos * kvw, s->v, sizeof(float) * kvw);
    if ((rc = so_grouped_attention(s->q, keys, values, m->q_heads, m->kv_heads, hd, pos + 1, s->scores, s->ctx,
                                   threads))) return rc;
    if ((rc = so_q_matvec_batch(L->o, m->hidden, qw, L->o_fmt, s->ctx, 1, s->proj, threads))) return rc;
    so_add(s->hidden, s->proj, m->hidden, s->hidden);
    if ((rc = so_rmsnorm(s->hidden, L->ffn_norm, m->hidden, m->eps, s->normed))) return rc;
    if ((rc = so_q_matvec_batch(L->gate, m->ffn, m->hidden, L->gate_fmt, s->normed, 1, s->gate, threads))) return rc;
    if ((rc = so_q_matvec_batch(L->up, m->ffn, m->hidden, L->up_fmt, s->normed, 1, s->up, threads))) return rc;
    so_swiglu(s->gate, s->up, m->ffn, s->act);
    if ((rc = so_q_matvec_batch(L->down, m->hidden, m->ffn, L->down_fmt, s->act, 1, s->proj, threads))) return rc;
    so_add(s->hidden, s->proj, m->hidden, s->hidden);
    return SO_OK;
}

/* DenseSession.Append (DenseSession.cs:111-131) with DenseForward.Embed (:87-92) and Final
 * (:298-306), then GreedyTokenSelector.Select. */
int so_session_append(so_session *s, int token, float *logits, int *argmax, int threads)
{
    const so_model *m = s->m;
    if (token < 0 || token >= m->vocab) return SO_ERR_ARGUMENT;
    if (s->position >= s->context) return SO_ERR_CONTEXT_FULL;
    /* GgufQuantizedMatrix.ReadRow (GgufQuantizedMatrix.cs:54-61): Q4_0 rows are rejected. */
    if (m->embd_fmt != SO_Q8_0) return SO_ERR_NOT_SUPPORTED;
    int64_t row_bytes = (int64_t)(m->hidden / 32) * 34;
    int rc = so_q_decode_row(m->embd + (int64_t)token * row_bytes, m->hidden, m->embd_fmt, s->hidden);
    if (rc) return rc;
    for (int layer = 0; layer < m->layers; layer++)
        if ((rc = dense_step(s, layer, threads))) return rc;
    if ((rc = so_rmsnorm(s->hidden, m->output_norm, m->hidden, m->eps, s->final_norm))) return rc;
    if ((rc = so_q_matvec_batch(m->output, m->vocab, m->hidden, m->output_fmt, s->final_norm, 1, logits, threads)))
        return rc;
    s->position++;
    if (argmax) return so_greedy_select(logits, m->vocab, argmax);
    return SO_OK;
}

int so_session_stage(const so_session *s, int which, float *out, int n)
{
    const float *src = which == 0 ? s->hidden : which == 1 ? s->final_norm : NULL;
    if (!src || n != s->m->hidden) return SO_ERR_ARGUMENT;
    memcpy(out, src, sizeof(float) * (size_t)n);
    return SO_OK;
}

/* ------------------------------------------------------------------------- */
/* GGUF K-quants: Q4_K / Q6_K weights, Q8_K activations                      */
/* ------------------------------------------------------------------------- */

/* QuantizedMatrixShape.cs:11-12: 256 weights per super-block; Q4_K 144 bytes, Q6_K 210. */
int so_k_geometry(int rows, int cols, int fmt, int *block_bytes, int64_t *byte_length)
{
    int bb;
    if (fmt == SO_Q4_K) bb = 144;
    else if (fmt == SO_Q6_K) bb = 210;
    else return SO_ERR_ARGUMENT;
    if (rows <= 0 || cols <= 0 || cols % 256 != 0) return SO_ERR_ARGUMENT;
    int64_t len = (int64_t)rows * (cols / 256) * bb;
    if (len > 0x7fffffffLL) return SO_ERR_ARGUMENT;
    if (block_bytes) *block_bytes = bb;
    if (byte_length) *byte_length = len;
    return SO_OK;
}

/* QuantizedMatVec.ValidatePayload (QuantizedMatVec.cs:28-42) with Q4KCodec.AreScalesFinite (d, dmin)
 * and Q6KCodec.AreScalesFinite (d at byte 208). */
int so_k_validate(const uint8_t *data, int64_t len, int rows, int cols, int fmt)
{
    int bb; int64_t want;
    int rc = so_k_geometry(rows, cols, fmt, &bb, &want);
    if (rc) return rc;
    if (len != want) return SO_ERR_ARGUMENT;
    for (int64_t off = 0; off < len; off += bb) {
        const uint8_t *b = data + off;
        if (fmt == SO_Q4_K) {
            if (!isfinite_f(so_half_to_float(rd16(b))) || !isfinite_f(so_half_to_float(rd16(b + 2))))
                return SO_ERR_INVALID_DATA;
        } else if (!isfinite_f(so_half_to_float(rd16(b + 208)))) {
            return SO_ERR_INVALID_DATA;
        }
    }
    return SO_OK;
}

/* Q4KCodec.GetScaleMin (Q4KCodec.cs:24-37) */
static void q4k_scale_min(int j, const uint8_t *scales, int *scale, int *min)
{
    if (j < 4) {
        *scale = scales[j] & 63;
        *min = scales[j + 4] & 63;
    } else {
        *scale = (scales[j + 4] & 0xF) | ((scales[j - 4] >> 6) << 4);
        *min = (scales[j + 4] >> 4) | ((scales[j] >> 6) << 4);
    }
}

/* Q4KCodec.DecodeBlock (Q4KCodec.cs:70-91): w = dl * q - ml, every product and difference rounded. */
static void q4k_decode_block(const uint8_t *b, float *w)
{
    float d = so_half_to_float(rd16(b)), dmin = so_half_to_float(rd16(b + 2));
    const uint8_t *scales = b + 4, *quants = b + 16;
    for (int g = 0; g < 4; g++) {
        const uint8_t *qs = quants + g * 32;
        int s0, n0, s1, n1;
        q4k_scale_min(g * 2, scales, &s0, &n0);
        q4k_scale_min(g * 2 + 1, scales, &s1, &n1);
        float dl = d * (float)s0, ml = dmin * (float)n0, dh = d * (float)s1, mh = dmin * (float)n1;
        for (int l = 0; l < 32; l++) {
            w[g * 64 + l] = dl * (float)(qs[l] & 0xF) - ml;
            w[g * 64 + 32 + l] = dh * (float)(qs[l] >> 4) - mh;
        }
    }
}

/* The 6-bit code of weight (half, l, k) of a Q6_K block (Q6KCodec.cs:38-46), already centred. */
static inline int q6k_code(const uint8_t *b, int half, int l, int k)
{
    const uint8_t *lql = b + half * 64, *lqh = b + 128 + half * 32;
    int nib = k == 0 ? (lql[l] & 0xF) : k == 1 ? (lql[l + 32] & 0xF) : k == 2 ? (lql[l] >> 4) : (lql[l + 32] >> 4);
    return (nib | (((lqh[l] >> (2 * k)) & 3) << 4)) - 32;
}

/* Q6KCodec.DecodeBlock (Q6KCodec.cs:58-85): w = d * scale * q, left to right. */
static void q6k_decode_block(const uint8_t *b, float *w)
{
    float d = so_half_to_float(rd16(b + 208));
    const int8_t *scales = (const int8_t *)(b + 192);
    for (int half = 0; half < 2; half++)
        for (int l = 0; l < 32; l++) {
            int sub = l / 16;
            for (int k = 0; k < 4; k++)
                w[half * 128 + l + 32 * k] = d * (float)scales[half * 8 + sub + 2 * k] * (float)q6k_code(b, half, l, k);
        }
}

int so_k_decode_row(const uint8_t *row_bytes, int cols, int fmt, float *out)
{
    int bb;
    if (so_k_geometry(1, cols, fmt, &bb, NULL)) return SO_ERR_ARGUMENT;
    for (int b = 0; b < cols / 256; b++) {
        if (fmt == SO_Q4_K) q4k_decode_block(row_bytes + (int64_t)b * bb, out + b * 256);
        else q6k_decode_block(row_bytes + (int64_t)b * bb, out + b * 256);
    }
    return SO_OK;
}

/* Q4KCodec.DotBlock (Q4KCodec.cs:40-66) */
static float q4k_dot_block(const uint8_t *b, const float *x)
{
    float d = so_half_to_float(rd16(b)), dmin = so_half_to_float(rd16(b + 2));
    const uint8_t *scales = b + 4, *quants = b + 16;
    float total = 0;
    for (int g = 0; g < 4; g++) {
        const uint8_t *qs = quants + g * 32;
        const float *low = x + g * 64, *high = x + g * 64 + 32;
        int s0, n0, s1, n1;
        q4k_scale_min(g * 2, scales, &s0, &n0);
        q4k_scale_min(g * 2 + 1, scales, &s1, &n1);
        float dl = d * (float)s0, ml = dmin * (float)n0, dh = d * (float)s1, mh = dmin * (float)n1;
        float acc_low = 0, acc_high = 0;
        for (int l = 0; l < 32; l++) {
            acc_low += (dl * (float)(qs[l] & 0xF) - ml) * low[l];
            acc_high += (dh * (float)(qs[l] >> 4) - mh) * high[l];
        }
        total += acc_low + acc_high;
    }
    return total;
}

/* Q6KCodec.DotBlock (Q6KCodec.cs:14-44) */
static float q6k_dot_block(const uint8_t *b, const float *x)
{
    float d = so_half_to_float(rd16(b + 208));
    const int8_t *scales = (const int8_t *)(b + 192);
    float total = 0;
    for (int half = 0; half < 2; half++)
        for (int l = 0; l < 32; l++) {
            int sub = l / 16;
            for (int k = 0; k < 4; k++)
                total += d * (float)scales[half * 8 + sub + 2 * k] * (float)q6k_code(b, half, l, k) *
                         x[half * 128 + l + 32 * k];
        }
    return total;
}

/* QuantizedMatVec.ExecuteScalar for the K formats (QuantizedMatVec.cs:45-66): total += DotBlock. */
int so_k_matvec_scalar(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y)
{
    int bb; int64_t len;
    int rc = so_k_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    int bpr = cols / 256;
    for (int row = 0; row < rows; row++) {
        float total = 0;
        for (int blk = 0; blk < bpr; blk++) {
            const uint8_t *b = data + ((int64_t)row * bpr + blk) * bb;
            total += fmt == SO_Q4_K ? q4k_dot_block(b, x + blk * 256) : q6k_dot_block(b, x + blk * 256);
        }
        y[row] = total;
    }
    return SO_OK;
}

/* One row of QuantizedKAvx2Kernel.ExecuteQ4K / ExecuteQ6K (QuantizedKAvx2Kernel.cs:225-331): eight float
 * lanes per 8-weight step (multiply then add, no FMA), the fixed horizontal sum, total += it. */
static void k_avx2_row(const uint8_t *data, int row, int cols, int fmt, int bb, const float *x, float *y)
{
    int bpr = cols / 256;
    float total = 0;
    for (int blk = 0; blk < bpr; blk++) {
        const uint8_t *b = data + ((int64_t)row * bpr + blk) * bb;
        const float *xb = x + blk * 256;
        if (fmt == SO_Q4_K) {
            float d = so_half_to_float(rd16(b)), dmin = so_half_to_float(rd16(b + 2));
            for (int g = 0; g < 4; g++) {
                const uint8_t *q = b + 16 + g * 32;
                int s0, n0, s1, n1;
                q4k_scale_min(g * 2, b + 4, &s0, &n0);
                q4k_scale_min(g * 2 + 1, b + 4, &s1, &n1);
                __m256 ls = _mm256_set1_ps(d * (float)s0), lb = _mm256_set1_ps(dmin * (float)n0);
                __m256 hs = _mm256_set1_ps(d * (float)s1), hb = _mm256_set1_ps(dmin * (float)n1);
                __m256 acc = _mm256_setzero_ps();
                for (int j = 0; j < 32; j += 8) {
                    uint64_t packed; memcpy(&packed, q + j, 8);
                    __m256i codes = _mm256_cvtepu8_epi32(_mm_cvtsi64_si128((long long)packed));
                    __m256 low = _mm256_cvtepi32_ps(_mm256_and_si256(codes, _mm256_set1_epi32(15)));
                    __m256 high = _mm256_cvtepi32_ps(_mm256_srli_epi32(codes, 4));
                    __m256 lw = _mm256_sub_ps(_mm256_mul_ps(low, ls), lb);
                    __m256 hw = _mm256_sub_ps(_mm256_mul_ps(high, hs), hb);
                    acc = _mm256_add_ps(acc, _mm256_mul_ps(lw, _mm256_loadu_ps(xb + g * 64 + j)));
                    acc = _mm256_add_ps(acc, _mm256_mul_ps(hw, _mm256_loadu_ps(xb + g * 64 + 32 + j)));
                }
                total += hsum256(acc);
            }
        } else {
            float d = so_half_to_float(rd16(b + 208));
            const int8_t *scales = (const int8_t *)(b + 192);
            for (int half = 0; half < 2; half++)
                for (int l = 0; l < 32; l += 8) {
                    int sub = l / 16;
                    __m256 acc = _mm256_setzero_ps();
                    for (int k = 0; k < 4; k++) {
                        float c[8];
                        for (int i = 0; i < 8; i++) c[i] = (float)q6k_code(b, half, l + i, k);
                        __m256 w = _mm256_mul_ps(_mm256_loadu_ps(c), _mm256_set1_ps(d * (float)scales[half * 8 + sub + 2 * k]));
                        acc = _mm256_add_ps(acc, _mm256_mul_ps(w, _mm256_loadu_ps(xb + half * 128 + l + 32 * k)));
                    }
                    total += hsum256(acc);
                }
        }
    }
    y[row] = total;
}

int so_k_matvec_avx2(const uint8_t *data, int rows, int cols, int fmt, const float *x, float *y, int threads)
{
    int bb; int64_t len;
    int rc = so_k_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (int row = 0; row < rows; row++) k_avx2_row(data, row, cols, fmt, bb, x, y);
    return SO_OK;
}

/* Q8KCodec.QuantizeBlock (Q8KCodec.cs:43-75) with NearestInteger (:104-110): 292 bytes per 256 values. */
static void q8k_quantize_block(const float *x, uint8_t *blk)
{
    float max = 0, magnitude = 0;
    for (int j = 0; j < 256; j++) {
        float a = fabsf(x[j]);
        if (a > magnitude) { magnitude = a; max = x[j]; }
    }
    if (magnitude == 0) { memset(blk, 0, 292); return; }
    float inverse = -127.0f / max;
    int8_t *codes = (int8_t *)(blk + 4);
    for (int j = 0; j < 256; j++) {
        float shifted = inverse * x[j] + 12582912.0f;
        int v = (int)(f2u(shifted) & 0x007fffffu) - 0x00400000;
        codes[j] = (int8_t)(v < 127 ? v : 127);
    }
    for (int g = 0; g < 16; g++) {
        int total = 0;
        for (int j = 0; j < 16; j++) total += codes[g * 16 + j];
        int16_t s = (int16_t)total;
        memcpy(blk + 260 + 2 * g, &s, 2);
    }
    float scale = 1.0f / inverse;
    memcpy(blk, &scale, 4);
}

int so_q8k_quantize_row(const float *x, int cols, uint8_t *out)
{
    if (cols <= 0 || cols % 256 != 0) return SO_ERR_ARGUMENT;
    for (int b = 0; b < cols / 256; b++) q8k_quantize_block(x + b * 256, out + (int64_t)b * 292);
    return SO_OK;
}

/* Q4KCodec.DotProduct / MinProduct (Q4KCodec.cs:112-153) and Q6KCodec.DotProduct (Q6KCodec.cs:103-146):
 * exact integers.  For Q4_K *min_total receives MinProduct. */
int so_k_int_dot(const uint8_t *b, int fmt, const uint8_t *act, int32_t *dot, int32_t *min_total)
{
    const int8_t *codes = (const int8_t *)(act + 4);
    int16_t sums[16];
    memcpy(sums, act + 260, 32);
    int total = 0, mins = 0;
    if (fmt == SO_Q4_K) {
        for (int g = 0; g < 4; g++) {
            const uint8_t *qs = b + 16 + g * 32;
            int ls, lm, hs, hm;
            q4k_scale_min(g * 2, b + 4, &ls, &lm);
            q4k_scale_min(g * 2 + 1, b + 4, &hs, &hm);
            int low = 0, high = 0;
            for (int l = 0; l < 32; l++) {
                low += (qs[l] & 0xF) * codes[g * 64 + l];
                high += (qs[l] >> 4) * codes[g * 64 + 32 + l];
            }
            total += ls * low + hs * high;
            mins += lm * (sums[g * 4] + sums[g * 4 + 1]) + hm * (sums[g * 4 + 2] + sums[g * 4 + 3]);
        }
    } else if (fmt == SO_Q6_K) {
        const int8_t *scales = (const int8_t *)(b + 192);
        for (int half = 0; half < 2; half++)
            for (int l = 0; l < 32; l++) {
                int sub = l / 16;
                for (int k = 0; k < 4; k++)
                    total += scales[half * 8 + sub + 2 * k] * q6k_code(b, half, l, k) * codes[half * 128 + l + 32 * k];
            }
    } else {
        return SO_ERR_ARGUMENT;
    }
    if (dot) *dot = total;
    if (min_total) *min_total = mins;
    return SO_OK;
}

/* QuantizedMatVec.ExecuteBatchQuantized -> QuantizedKAvx2Kernel.ExecuteQuantizedTiled
 * (QuantizedMatVec.cs:122-220, QuantizedKAvx2Kernel.cs:46-95): activations quantized to Q8_K once; per
 * row and block an exact integer product, then the float combine in the reference's order, summed over
 * blocks per position; all-zero activation blocks are skipped. */
int so_k_matvec_batch(const uint8_t *data, int rows, int cols, int fmt, const float *x, int positions, float *y,
                      int threads)
{
    int bb; int64_t len;
    int rc = so_k_geometry(rows, cols, fmt, &bb, &len);
    if (rc) return rc;
    if (positions <= 0 || positions > 256) return SO_ERR_ARGUMENT;
    int bpr = cols / 256;
    int64_t arow = (int64_t)bpr * 292;
    uint8_t *act = (uint8_t *)malloc((size_t)(arow * positions));
    for (int p = 0; p < positions; p++) so_q8k_quantize_row(x + (int64_t)p * cols, cols, act + p * arow);
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (int row = 0; row < rows; row++) {
        float acc[256];
        for (int p = 0; p < positions; p++) acc[p] = 0;
        for (int blk = 0; blk < bpr; blk++) {
            const uint8_t *b = data + ((int64_t)row * bpr + blk) * bb;
            float d = fmt == SO_Q4_K ? so_half_to_float(rd16(b)) : so_half_to_float(rd16(b + 208));
            float dmin = fmt == SO_Q4_K ? so_half_to_float(rd16(b + 2)) : 0;
            for (int p = 0; p < positions; p++) {
                const uint8_t *a = act + p * arow + (int64_t)blk * 292;
                float as = rdf32(a);
                if (as == 0) continue;
                int32_t dot, mins;
                so_k_int_dot(b, fmt, a, &dot, &mins);
                if (fmt == SO_Q4_K) {
                    float da = d * as, ma = dmin * as;
                    acc[p] += da * (float)dot - ma * (float)mins;
                } else {
                    acc[p] += as * d * (float)dot;
                }
            }
        }
        for (int p = 0; p < positions; p++) y[(int64_t)p * rows + row] = acc[p];
    }
    free(act);
    return SO_OK;
}

/* ------------------------------------------------------------------------- */
/* Ternary bitplane (STB1): docs/ternary-bitplane-v1.md                      */
/* ------------------------------------------------------------------------- */

/* TernaryBitplaneMatrix.FromTernary2 (TernaryBitplaneMatrix.cs:18-36): scale copied, code 1 -> P bit,
 * code 2 -> N bit, same blocks and padding. */
int so_tb_from_t2(const uint8_t *t2, int rows, int cols, int bs, uint8_t *out)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    int plane = bs / 8;
    memset(out, 0, (size_t)len);
    for (int64_t off = 0; off < len; off += bb) {
        memcpy(out + off, t2 + off, 4);
        for (int i = 0; i < bs; i++) {
            int code = (t2[off + 4 + i / 4] >> (2 * (i % 4))) & 3;
            if (code != 0) out[off + 4 + (code == 2 ? plane : 0) + i / 8] |= (uint8_t)(1 << (i % 8));
        }
    }
    return SO_OK;
}

/* TernaryBitplaneMatrix.ToTernary2 (:38-55): P -> 01, N -> 10. */
int so_tb_to_t2(const uint8_t *tb, int rows, int cols, int bs, uint8_t *out)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    int plane = bs / 8;
    memset(out, 0, (size_t)len);
    for (int64_t off = 0; off < len; off += bb) {
        memcpy(out + off, tb + off, 4);
        for (int i = 0; i < bs; i++) {
            int p = (tb[off + 4 + i / 8] >> (i % 8)) & 1;
            int n = (tb[off + 4 + plane + i / 8] >> (i % 8)) & 1;
            out[off + 4 + i / 4] |= (uint8_t)((p | n << 1) << (2 * (i % 4)));
        }
    }
    return SO_OK;
}

/* TernaryBitplaneMatrix.Validate (:66-87) */
int so_tb_validate(const uint8_t *data, int64_t len, int rows, int cols, int bs)
{
    int bpr, bb; int64_t want;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &want);
    if (rc) return rc;
    if (len != want) return SO_ERR_ARGUMENT;
    int plane = bs / 8;
    for (int row = 0; row < rows; row++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *blk = data + ((int64_t)row * bpr + b) * bb;
            float scale = rdf32(blk);
            if (!isfinite_f(scale) || scale < 0 || f2u(scale) == 0x80000000u) return SO_ERR_ARGUMENT;
            int count = bs < cols - b * bs ? bs : cols - b * bs;
            for (int i = 0; i < plane; i++) {
                uint8_t p = blk[4 + i], n = blk[4 + plane + i];
                int valid = count - i * 8;
                valid = valid < 0 ? 0 : valid > 8 ? 8 : valid;
                int padding = ~((1 << valid) - 1);
                if ((p & n) != 0 || ((p | n) & padding) != 0 || (scale == 0 && (p | n) != 0)) return SO_ERR_ARGUMENT;
            }
        }
    return SO_OK;
}

/* TernaryBitplaneMatVec.ExecuteScalar (TernaryBitplaneMatVec.cs:24-47): sequential +x / -x per block,
 * total += scale * sum. */
int so_tb_matvec_scalar(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    int plane = bs / 8;
    for (int row = 0; row < rows; row++) {
        float total = 0;
        for (int b = 0; b < bpr; b++) {
            const uint8_t *blk = data + ((int64_t)row * bpr + b) * bb;
            int column = b * bs, count = bs < cols - column ? bs : cols - column;
            float sum = 0;
            for (int i = 0; i < count; i++) {
                int mask = 1 << (i % 8);
                if (blk[4 + i / 8] & mask) sum += x[column + i];
                else if (blk[4 + plane + i / 8] & mask) sum -= x[column + i];
            }
            total += rdf32(blk) * sum;
        }
        y[row] = total;
    }
    return SO_OK;
}

/* TernaryBitplaneAvx2Kernel.Execute (TernaryBitplaneAvx2Kernel.cs:18-52): eight lanes of
 * AndNot(zero, x ^ sign), the fixed horizontal sum, a scalar tail, total += scale * partial. */
int so_tb_matvec_avx2(const uint8_t *data, int rows, int cols, int bs, const float *x, float *y)
{
    int bpr, bb; int64_t len;
    int rc = so_t2_geometry(rows, cols, bs, &bpr, &bb, &len);
    if (rc) return rc;
    int plane = bs / 8;
    const __m256i shifts = _mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7);
    const __m256i active = _mm256_set1_epi32(0x101), negative = _mm256_set1_epi32(0x100);
    for (int row = 0; row < rows; row++) {
        float total = 0;
        for (int b = 0; b < bpr; b++) {
            const uint8_t *blk = data + ((int64_t)row * bpr + b) * bb;
            int column = b * bs, count = bs < cols - column ? bs : cols - column;
            __m256 acc = _mm256_setzero_ps();
            int i = 0;
            for (; i <= count - 8; i += 8) {
                uint32_t packed = (uint32_t)(blk[4 + i / 8] | blk[4 + plane + i / 8] << 8);
                __m256i lanes = _mm256_srlv_epi32(_mm256_set1_epi32((int)packed), shifts);
                __m256i zero = _mm256_cmpeq_epi32(_mm256_and_si256(lanes, active), _mm256_setzero_si256());
                __m256i sign = _mm256_slli_epi32(_mm256_and_si256(lanes, negative), 23);
                __m256 values = _mm256_loadu_ps(x + column + i);
                acc = _mm256_add_ps(acc, _mm256_andnot_ps(_mm256_castsi256_ps(zero),
                                                          _mm256_xor_ps(values, _mm256_castsi256_ps(sign))));
            }
            float partial = hsum256(acc);
            for (; i < count; i++) {
                int mask = 1 << (i % 8);
                if (blk[4 + i / 8] & mask) partial += x[column + i];
                else if (blk[4 + plane + i / 8] & mask) partial -= x[column + i];
            }
            total += rdf32(blk) * partial;
        }
        y[row] = total;
    }
    return SO_OK;
}
