/*
 * CPU oracle for the quantized MUL_MAT path (TEST INFRASTRUCTURE ONLY:
 * the checker for the CUDA path and the timed CPU baseline; never part of
 * the product). See quant_ref.h for the reference files restated here.
 */
#include "quant_ref.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float oracle_f16_to_f32(uint16_t h) {
    /* Bit-level decode, same cases as f16BitsToF32 in
     * tests/jsep-matmul-golden.test.ts:256-272 (subnormals handled). */
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t exp = (uint32_t)(h >> 10) & 0x1fu;
    uint32_t mant = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign << 31;
        } else {
            /* subnormal: value = mant * 2^-24, renormalise into f32 */
            int e = -1;
            do {
                mant <<= 1;
                ++e;
            } while ((mant & 0x400u) == 0);
            mant &= 0x3ffu;
            bits = (sign << 31) | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        bits = (sign << 31) | 0x7f800000u | (mant << 13);
    } else {
        bits = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

int32_t oracle_block_elems(int32_t type) {
    switch (type) {
        case ORACLE_TYPE_F32: return 1;
        case ORACLE_TYPE_Q4_0: return 32;
        case ORACLE_TYPE_Q8_0: return 32;
        case ORACLE_TYPE_Q4_K: return 256;
        case ORACLE_TYPE_Q5_K: return 256;
        case ORACLE_TYPE_Q6_K: return 256;
        case ORACLE_TYPE_IQ4_XS: return 256;
        default: return 0;
    }
}

int32_t oracle_block_bytes(int32_t type) {
    /* src/models/gguf-parser.ts:273-294 (ggmlTypeSize). */
    switch (type) {
        case ORACLE_TYPE_F32: return 4;
        case ORACLE_TYPE_Q4_0: return 18;
        case ORACLE_TYPE_Q8_0: return 34;
        case ORACLE_TYPE_Q4_K: return 144;
        case ORACLE_TYPE_Q5_K: return 176;
        case ORACLE_TYPE_Q6_K: return 210;
        case ORACLE_TYPE_IQ4_XS: return 136; /* ggml block_iq4_xs; not in the reference's ggmlTypeSize */
        default: return 0;
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* get_scale_min_k4: matmul.ts:408-424 (q4k_unpack_scale_min). */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* One 144-byte Q4_K super-block -> 256 floats.
 * matmul.ts:426-460 / p2-v2-spike.src.ts:1057-1096: element e of the block
 * sits in pair p = e/64; l = e%32; the low nibble of qs[32p+l] serves
 * e < 64p+32 (sub-block 2p), the high nibble serves sub-block 2p+1;
 * y = d*sc*q - dmin*m. */
static void dequant_block_q4_K(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32(rd16(b));
    const float dmin = oracle_f16_to_f32(rd16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    for (int p = 0; p < 4; ++p) {
        int sc0, m0, sc1, m1;
        q4k_scale_min(scales, 2 * p, &sc0, &m0);
        q4k_scale_min(scales, 2 * p + 1, &sc1, &m1);
        const float d1 = d * (float)sc0, mm1 = dmin * (float)m0;
        const float d2 = d * (float)sc1, mm2 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            y[64 * p + l] = d1 * (float)(qs[32 * p + l] & 0xF) - mm1;
            y[64 * p + 32 + l] = d2 * (float)(qs[32 * p + l] >> 4) - mm2;
        }
    }
}

/* One 176-byte Q5_K super-block -> 256 floats (ggml block_q5_K: f16 d @0,
 * f16 dmin @2, scales[12] @4 packed as for Q4_K, qh[32] @16, qs[128] @48).
 * Sub-block j (0..7) holds elements 32j..32j+31; element 32j+l has the
 * nibble of qs[32(j/2)+l] (low for even j, high for odd) and bit j of
 * qh[l] as bit 4: q = 0..31, y = d*sc_j*q - dmin*m_j. */
static void dequant_block_q5_K(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32(rd16(b));
    const float dmin = oracle_f16_to_f32(rd16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        q4k_scale_min(scales, j, &sc, &m);
        const float ds = d * (float)sc, dm = dmin * (float)m;
        for (int l = 0; l < 32; ++l) {
            const int nib = (j & 1) ? (qs[32 * (j / 2) + l] >> 4) : (qs[32 * (j / 2) + l] & 0xF);
            const int q = nib | (((qh[l] >> j) & 1) << 4);
            y[32 * j + l] = ds * (float)q - dm;
        }
    }
}

/* One 18-byte Q4_0 block -> 32 floats (ggml block_q4_0: f16 d @0, qs[16]
 * @2): element l < 16 is the low nibble of qs[l], element 16+l the high
 * nibble; y = d*(q - 8). */
static void dequant_block_q4_0(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32(rd16(b));
    const uint8_t* qs = b + 2;
    for (int l = 0; l < 16; ++l) {
        y[l] = d * (float)((int)(qs[l] & 0xF) - 8);
        y[16 + l] = d * (float)((int)(qs[l] >> 4) - 8);
    }
}

/* One 210-byte Q6_K super-block -> 256 floats (ggml block_q6_K:
 * ql[128] @0, qh[64] @128, int8 scales[16] @192, f16 d @208).
 * Half h covers elements 128h..128h+127; for l in 0..31:
 *   q0 = lo4(ql[64h+l])    | bits0-1(qh[32h+l]) << 4  -> element 128h+l
 *   q1 = lo4(ql[64h+32+l]) | bits2-3(qh[32h+l]) << 4  -> element 128h+32+l
 *   q2 = hi4(ql[64h+l])    | bits4-5(qh[32h+l]) << 4  -> element 128h+64+l
 *   q3 = hi4(ql[64h+32+l]) | bits6-7(qh[32h+l]) << 4  -> element 128h+96+l
 * each minus 32, times d * scales[element/16]. */
static void dequant_block_q6_K(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = oracle_f16_to_f32(rd16(b + 208));
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q0 = (int)((ql[64 * h + l] & 0xF) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32;
            const int q1 = (int)((ql[64 * h + 32 + l] & 0xF) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32;
            const int q2 = (int)((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32;
            const int q3 = (int)((ql[64 * h + 32 + l] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32;
            y[128 * h + l] = d * (float)sc[8 * h + is + 0] * (float)q0;
            y[128 * h + 32 + l] = d * (float)sc[8 * h + is + 2] * (float)q1;
            y[128 * h + 64 + l] = d * (float)sc[8 * h + is + 4] * (float)q2;
            y[128 * h + 96 + l] = d * (float)sc[8 * h + is + 6] * (float)q3;
        }
    }
}

/* The 16 non-linear 4-bit levels of IQ4_NL / IQ4_XS (ggml's kvalues_iq4nl,
 * a fixed part of the format). */
static const int8_t kIq4Levels[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* One 136-byte IQ4_XS super-block -> 256 floats (ggml block_iq4_xs: f16 d
 * @0, u16 scales_h @2, scales_l[4] @4, qs[128] @8). The reference has no
 * IQ4_XS code of its own (ggml is in the un-vendored llama.cpp fork; the
 * type appears as file type 30 in src/models/model-loader.ts:906 and as a
 * canonical fleet quant in docs/MODEL_SUPPORT.md:135,294). Sub-block j
 * (0..7) holds elements 32j..32j+31 with the 6-bit scale
 * ls = (scales_l[j/2] >> 4(j%2)) & 15 | ((scales_h >> 2j) & 3) << 4; element
 * 32j+l (l < 16) is level[qs[16j+l] & 15], element 32j+16+l is
 * level[qs[16j+l] >> 4]; y = d*(ls - 32)*level. d*(ls - 32) has at most 16
 * significant bits and the level 7, so both products are exact in f32. */
static void dequant_block_iq4_xs(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32(rd16(b));
    const unsigned scales_h = rd16(b + 2);
    const uint8_t* scales_l = b + 4;
    const uint8_t* qs = b + 8;
    for (int j = 0; j < 8; ++j) {
        const int ls = ((scales_l[j / 2] >> (4 * (j % 2))) & 0xF) | (((scales_h >> (2 * j)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        for (int l = 0; l < 16; ++l) {
            y[32 * j + l] = dl * (float)kIq4Levels[qs[16 * j + l] & 0xF];
            y[32 * j + 16 + l] = dl * (float)kIq4Levels[qs[16 * j + l] >> 4];
        }
    }
}

/* One 34-byte Q8_0 block -> 32 floats: f16 d @0, int8 qs[32] @2; y = d*q. */
static void dequant_block_q8_0(const uint8_t* b, float* y) {
    const float d = oracle_f16_to_f32(rd16(b));
    const int8_t* qs = (const int8_t*)(b + 2);
    for (int i = 0; i < 32; ++i) y[i] = d * (float)qs[i];
}

int32_t oracle_dequantize_row(int32_t type, const void* src, float* dst, int64_t k) {
    const int32_t be = oracle_block_elems(type), bb = oracle_block_bytes(type);
    if (!src || !dst || k <= 0 || be <= 0 || (k % be) != 0) return -1;
    const uint8_t* s = (const uint8_t*)src;
    const int64_t nb = k / be;
    for (int64_t i = 0; i < nb; ++i) {
        switch (type) {
            case ORACLE_TYPE_Q4_K: dequant_block_q4_K(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_Q5_K: dequant_block_q5_K(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_Q6_K: dequant_block_q6_K(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_Q4_0: dequant_block_q4_0(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_Q8_0: dequant_block_q8_0(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_IQ4_XS: dequant_block_iq4_xs(s + i * bb, dst + i * be); break;
            case ORACLE_TYPE_F32: memcpy(dst + i, s + 4 * i, 4); break;
            default: return -1;
        }
    }
    return 0;
}

static int check_args(int32_t type, const void* w, int64_t row_bytes, const float* x,
                      int64_t x_stride, const void* out, int32_t M, int32_t K, int32_t N) {
    const int32_t be = oracle_block_elems(type), bb = oracle_block_bytes(type);
    if (!w || !x || !out || M <= 0 || K <= 0 || N <= 0) return -1;
    if (be <= 0 || (K % be) != 0) return -1;
    if (row_bytes < (int64_t)(K / be) * bb) return -1;
    if (x_stride < K) return -1;
    return 0;
}

int32_t oracle_mul_mat_f64(int32_t type, const void* w, int64_t row_bytes,
                           const float* x, int64_t x_stride,
                           double* out, int32_t M, int32_t K, int32_t N) {
    if (check_args(type, w, row_bytes, x, x_stride, out, M, K, N)) return -1;
    float* row = (float*)malloc(sizeof(float) * (size_t)K);
    if (!row) return -3;
    const uint8_t* wb = (const uint8_t*)w;
    for (int32_t m = 0; m < M; ++m) {
        oracle_dequantize_row(type, wb + (int64_t)m * row_bytes, row, K);
        for (int32_t n = 0; n < N; ++n) {
            const float* xn = x + (int64_t)n * x_stride;
            double acc = 0.0;
            for (int32_t k = 0; k < K; ++k) acc += (double)row[k] * (double)xn[k];
            out[(int64_t)m + (int64_t)M * n] = acc;
        }
    }
    free(row);
    return 0;
}

int32_t oracle_max_threads(void) {
#ifdef _OPENMP
    return (int32_t)omp_get_max_threads();
#else
    return 1;
#endif
}

/* 16 interleaved partial sums: element k goes to partial k%16; the partials
 * are added pairwise at the end. Written so the compiler vectorises it
 * without reassociating. */
static float dot16(const float* a, const float* b, int32_t K) {
    float p[16];
    for (int i = 0; i < 16; ++i) p[i] = 0.f;
    int32_t k = 0;
    for (; k + 16 <= K; k += 16)
        for (int i = 0; i < 16; ++i) p[i] += a[k + i] * b[k + i];
    for (; k < K; ++k) p[k & 15] += a[k] * b[k];
    for (int w = 8; w >= 1; w >>= 1)
        for (int i = 0; i < w; ++i) p[i] += p[i + w];
    return p[0];
}

int32_t oracle_mul_mat_f32(int32_t type, const void* w, int64_t row_bytes,
                           const float* x, int64_t x_stride,
                           float* out, int64_t out_stride,
                           int32_t M, int32_t K, int32_t N, int32_t threads) {
    if (check_args(type, w, row_bytes, x, x_stride, out, M, K, N)) return -1;
    if (out_stride < M) return -1;
    const uint8_t* wb = (const uint8_t*)w;
    int nthreads = threads > 0 ? threads : 1;
    int failed = 0;
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)K);
        if (!row) {
#ifdef _OPENMP
#pragma omp atomic write
#endif
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
            for (int32_t m = 0; m < M; ++m) {
                oracle_dequantize_row(type, wb + (int64_t)m * row_bytes, row, K);
                for (int32_t n = 0; n < N; ++n)
                    out[(int64_t)m + out_stride * n] = dot16(row, x + (int64_t)n * x_stride, K);
            }
            free(row);
        }
    }
    (void)nthreads;
    return failed ? -3 : 0;
}
