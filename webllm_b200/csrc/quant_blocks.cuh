// Device-side decoding of GGUF quant blocks (Q4_K, Q5_K, Q6_K, Q4_0, Q8_0).
//
// Block layouts (bytes):
//   Q4_K (256 elements, 144 B): f16 d @0, f16 dmin @2, scales[12] @4,
//        qs[128] @16. Pair p (0..3) owns qs[32p..32p+31]; the low nibble of
//        qs[32p+l] is element 64p+l (sub-block 2p), the high nibble element
//        64p+32+l (sub-block 2p+1). y = d*sc*q - dmin*m with (sc, m) the
//        6-bit pair unpacked as in src/inference/jsep/ops/matmul.ts:408-424.
//   Q6_K (256 elements, 210 B): ql[128] @0, qh[64] @128, int8 scales[16]
//        @192, f16 d @208. y = d*scales[e/16]*(q6 - 32).
//   Q5_K (256 elements, 176 B): f16 d @0, f16 dmin @2, scales[12] @4 (as
//        Q4_K), qh[32] @16, qs[128] @48. Element 32j+l: the nibble of
//        qs[32(j/2)+l] (low for even j) plus bit j of qh[l] as bit 4;
//        y = d*sc_j*q - dmin*m_j.
//   Q8_0 (32 elements, 34 B): f16 d @0, int8 qs[32] @2. y = d*q.
//   Q4_0 (32 elements, 18 B): f16 d @0, qs[16] @2; element l < 16 the low
//        nibble of qs[l], 16+l the high one; y = d*(q - 8).
//   IQ4_XS (256 elements, 136 B): f16 d @0, u16 scales_h @2, scales_l[4] @4,
//        qs[128] @8. Sub-block j (32 elements) has the 6-bit scale
//        ls = (scales_l[j/2] >> 4(j%2)) & 15 | ((scales_h >> 2j) & 3) << 4;
//        element 32j+l (l < 16) is level[qs[16j+l] & 15], 32j+16+l is
//        level[qs[16j+l] >> 4], with the 16 non-linear levels of kIq4Levels;
//        y = d*(ls - 32)*level.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace wllm {

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ uint32_t ldg_u32(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}

// Byte i (0..11) of the Q4_K scales, held as three little-endian words.
__device__ __forceinline__ uint32_t q4k_sbyte(const uint32_t s[3], int i) {
    return (s[i >> 2] >> (8 * (i & 3))) & 0xffu;
}

// (sc, m) of sub-block j (0..7): get_scale_min_k4 semantics
// (matmul.ts:408-424, p2-v2-spike.src.ts:1037-1055).
__device__ __forceinline__ void q4k_scale_min(const uint32_t s[3], int j, int& sc, int& m) {
    if (j < 4) {
        sc = static_cast<int>(q4k_sbyte(s, j) & 63u);
        m = static_cast<int>(q4k_sbyte(s, j + 4) & 63u);
    } else {
        sc = static_cast<int>((q4k_sbyte(s, j + 4) & 0xFu) | ((q4k_sbyte(s, j - 4) >> 6) << 4));
        m = static_cast<int>((q4k_sbyte(s, j + 4) >> 4) | ((q4k_sbyte(s, j) >> 6) << 4));
    }
}

// Exact dequantization of element e (0..255) of a Q4_K block.
__device__ __forceinline__ float q4k_dequant_elem(const uint8_t* blk, int e) {
    const uint32_t dm = ldg_u16(blk) | (ldg_u16(blk + 2) << 16);
    const float d = f16_bits_to_f32(dm), dmin = f16_bits_to_f32(dm >> 16);
    uint32_t s[3];
    s[0] = ldg_u16(blk + 4) | (ldg_u16(blk + 6) << 16);
    s[1] = ldg_u16(blk + 8) | (ldg_u16(blk + 10) << 16);
    s[2] = ldg_u16(blk + 12) | (ldg_u16(blk + 14) << 16);
    const int p = e >> 6, within = e & 63, l = within & 31;
    const int j = 2 * p + (within >= 32 ? 1 : 0);
    int sc, m;
    q4k_scale_min(s, j, sc, m);
    const uint32_t byte = blk[16 + 32 * p + l];
    const uint32_t q = within < 32 ? (byte & 0xFu) : (byte >> 4);
    // d*sc, dmin*m and (d*sc)*q are exact in f32 (<= 24 significant bits);
    // the subtraction is the single rounding, as in the oracle.
    return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                     __fmul_rn(dmin, static_cast<float>(m)));
}

// Exact dequantization of element e (0..255) of a Q6_K block.
__device__ __forceinline__ float q6k_dequant_elem(const uint8_t* blk, int e) {
    const int h = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
    const uint32_t ql = blk[64 * h + (quarter & 1) * 32 + l];
    const uint32_t qh = blk[128 + 32 * h + l];
    const uint32_t lo = (quarter < 2) ? (ql & 0xFu) : (ql >> 4);
    const uint32_t hi = (qh >> (2 * quarter)) & 3u;
    const int q = static_cast<int>(lo | (hi << 4)) - 32;
    const int sc = static_cast<int8_t>(blk[192 + (e >> 4)]);
    const float d = f16_bits_to_f32(ldg_u16(blk + 208));
    return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
}

// Exact dequantization of element e (0..255) of a Q5_K block.
__device__ __forceinline__ float q5k_dequant_elem(const uint8_t* blk, int e) {
    const uint32_t dm = ldg_u16(blk) | (ldg_u16(blk + 2) << 16);
    const float d = f16_bits_to_f32(dm), dmin = f16_bits_to_f32(dm >> 16);
    uint32_t s[3];
    s[0] = ldg_u16(blk + 4) | (ldg_u16(blk + 6) << 16);
    s[1] = ldg_u16(blk + 8) | (ldg_u16(blk + 10) << 16);
    s[2] = ldg_u16(blk + 12) | (ldg_u16(blk + 14) << 16);
    const int j = e >> 5, l = e & 31;
    int sc, m;
    q4k_scale_min(s, j, sc, m);
    const uint32_t byte = blk[48 + 32 * (j >> 1) + l];
    const uint32_t q = ((j & 1) ? (byte >> 4) : (byte & 0xFu)) | (((blk[16 + l] >> j) & 1u) << 4);
    // d*sc*q (q <= 31) and dmin*m are exact in f32; one rounding, as in the oracle
    return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                     __fmul_rn(dmin, static_cast<float>(m)));
}

// Exact dequantization of element e (0..31) of a Q4_0 block.
__device__ __forceinline__ float q4_0_dequant_elem(const uint8_t* blk, int e) {
    const float d = f16_bits_to_f32(ldg_u16(blk));
    const uint32_t byte = blk[2 + (e & 15)];
    const int q = static_cast<int>(e < 16 ? (byte & 0xFu) : (byte >> 4)) - 8;
    return __fmul_rn(d, static_cast<float>(q));
}

// The 16 non-linear 4-bit levels of IQ4_NL / IQ4_XS (ggml's kvalues_iq4nl, a
// fixed part of the format: -127 -104 -83 -65 -49 -35 -22 -10 1 13 25 38 53
// 69 89 113), as int8 bytes packed four to a word.
constexpr uint32_t kIq4Lv0 = 0xBFAD9881u, kIq4Lv1 = 0xF6EADDCFu, kIq4Lv2 = 0x26190D01u, kIq4Lv3 = 0x71594535u;

__device__ __forceinline__ int iq4_level(uint32_t i) {
    const uint32_t w = __byte_perm((i & 8u) ? kIq4Lv2 : kIq4Lv0, (i & 8u) ? kIq4Lv3 : kIq4Lv1, i & 7u);
    return static_cast<int8_t>(w & 0xFFu);
}

// Four IQ4_XS level indices (0..15, one per byte) -> their int8 levels. A
// byte permute picks from the table's low half (levels 0-7) and another from
// its high half, by the index's low 3 bits (__byte_perm reads 3 bits per
// selector nibble); bit 3 of each index, spread over its byte, selects between
// the two.
__device__ __forceinline__ uint32_t iq4_lut4(uint32_t idx) {
    const uint32_t y = idx | (idx >> 4);
    const uint32_t sel = __byte_perm(y, 0u, 0x4420u) & 0x7777u;  // i0 | i1 << 4 | i2 << 8 | i3 << 12, low 3 bits
    const uint32_t lo = __byte_perm(kIq4Lv0, kIq4Lv1, sel);
    const uint32_t hi = __byte_perm(kIq4Lv2, kIq4Lv3, sel);
    const uint32_t hsel = ((idx >> 3) & 0x01010101u) * 0xFFu;  // 0xFF where the index is 8..15
    return (hi & hsel) | (lo & ~hsel);
}

// Byte permute with the selector's sign mode: a selector nibble with bit 3
// set gives 0xFF or 0 by the sign bit of the byte it selects.
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// The levels of all eight 4-bit indices of a word of IQ4_XS index bytes: lo
// gets the low nibbles' levels (byte i: byte i's low nibble), hi the high
// nibbles'. The word itself is the selector: its nibbles in order are the
// indices of bytes 0, 0 (high), 1, 1 (high), ..., so four permutes (low and
// high half of the table, the word's low and high 16 bits) look up all eight
// by their low 3 bits; bit 3 of each index, at bit 7 of its byte in w (high
// nibbles) or in w << 4 (low nibbles), becomes a byte mask by the sign mode;
// two permutes put the levels back in byte order. 13 operations against
// about 23 for two iq4_lut4 calls and their nibble extraction.
__device__ __forceinline__ void iq4_lut8(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t s = w & 0x77777777u;
    const uint32_t a = __byte_perm(kIq4Lv0, kIq4Lv1, s), b = __byte_perm(kIq4Lv2, kIq4Lv3, s);
    const uint32_t c = __byte_perm(kIq4Lv0, kIq4Lv1, s >> 16), d = __byte_perm(kIq4Lv2, kIq4Lv3, s >> 16);
    const uint32_t w4 = w << 4;
    const uint32_t ma = prmt_sign(w4, w, 0xD9C8u), mc = prmt_sign(w4, w, 0xFBEAu);  // bit 3 of nibbles 0-3, 4-7
    const uint32_t ab = (b & ma) | (a & ~ma), cd = (d & mc) | (c & ~mc);  // levels of nibbles 0..3, 4..7
    lo = __byte_perm(ab, cd, 0x6420u);
    hi = __byte_perm(ab, cd, 0x7531u);
}

// The 6-bit scale (ls - 32, -32..31) of sub-block j (0..7) of an IQ4_XS block.
__device__ __forceinline__ int iq4xs_scale(uint32_t scales_h, uint32_t scales_l4, int j) {
    const uint32_t lo = (scales_l4 >> (4 * j)) & 0xFu;  // scales_l[j/2] >> 4(j%2), the four bytes as one word
    const uint32_t hi = (scales_h >> (2 * j)) & 3u;
    return static_cast<int>(lo | (hi << 4)) - 32;
}

// Exact dequantization of element e (0..255) of an IQ4_XS block: d*(ls - 32)
// has at most 16 significant bits and the level 7, so both products are exact.
__device__ __forceinline__ float iq4xs_dequant_elem(const uint8_t* blk, int e) {
    const float d = f16_bits_to_f32(ldg_u16(blk));
    const uint32_t sh = ldg_u16(blk + 2), sl = ldg_u16(blk + 4) | (ldg_u16(blk + 6) << 16);
    const int j = e >> 5, l = e & 31;
    const uint32_t byte = blk[8 + 16 * j + (l & 15)];
    const int q = iq4_level(l < 16 ? (byte & 0xFu) : (byte >> 4));
    return __fmul_rn(__fmul_rn(d, static_cast<float>(iq4xs_scale(sh, sl, j))), static_cast<float>(q));
}

// Exact dequantization of element e (0..31) of a Q8_0 block.
__device__ __forceinline__ float q8_0_dequant_elem(const uint8_t* blk, int e) {
    const float d = f16_bits_to_f32(ldg_u16(blk));
    const int q = static_cast<int8_t>(blk[2 + e]);
    return __fmul_rn(d, static_cast<float>(q));
}

}  // namespace wllm
