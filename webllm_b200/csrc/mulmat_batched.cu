// Small-batch quantized MUL_MAT (N >= 3 activation vectors: several sequences
// decoding together, short prefill tiles, the GEMV-to-GEMM crossover) for
// Q8_0, Q4_0, Q4_K, Q5_K and Q6_K weights on integer tensor cores
// (mma.sync m16n8k32, s8 / u8 x s8 -> s32).
//
//   y[m + M n] = sum_k W[m, k] x[k + K n]   (ggml MUL_MAT, matmul.ts:10-17)
//
// Activations: a pre-pass turns x into three int8 limbs per element,
// x = (l0 + l1 / 128 + l2 / 16384) / s with s = 127 / max|x| per 256 elements
// and vector (|error| <= max|x| / 4161536), stored as [N][3][K], with the
// factors 1 / s as [K / 256][N rounded up to 4] and, for Q4_K / Q5_K, the f32
// sums of x over each 16-element sub-block as [K / 256][N rounded up to
// 4][16]. The eight B columns of an MMA are one limb of eight vectors: each
// 32-element step takes three MMAs per vector octet, whose s32 results are
// combined in f32 as D0 + D1 / 128 + D2 / 16384.
//
// Weights, per 32-element MMA step (k = 32):
//  - Q8_0: one block; the s8 quants enter the MMA as they are and the s32
//    result is scaled by the rows' f16 d in f32;
//  - Q4_0: one block; the nibbles enter as s8 q - 8 (a 4-bit sign
//    extension), then as Q8_0;
//  - Q4_K: one 32-element sub-block; its u8 nibbles, the low ones as they are
//    and the high ones in place (16 q), the combined limbs times the 6-bit
//    scale (16 sc for the low-nibble sub-blocks) summed over the 256-element
//    block, then d / (16 s); the mins through the sub-block sums of x;
//  - Q5_K: as Q4_K with the 5-bit quants (nibble | qh bit << 4) as u8 and
//    sc for every sub-block, then d / s;
//  - Q6_K: two 16-element sub-blocks, one MMA each (the other half of the A
//    fragment zero); the quants q - 32 enter the MMA as s8 (a 6-bit sign
//    extension), times the int8 scale, then d / s.
//
// Tiling: a CTA (4 warps) computes 64 rows x NV vectors (NV = 8, 16, 32); warp w
// rows 16 w .. 16 w + 15. K is walked in chunks of 256 elements (8 Q8_0
// blocks, one K-quant block): the chunk's raw rows, limbs, factors and sums go
// to shared memory with cp.async, 2 to 4 chunks in flight. Q8_0 and Q6_K
// blocks are 34 and 210 bytes, so they sit at any even offset: their A
// fragments come from aligned 32-bit loads and a funnel shift; Q4_K rows are
// 16-byte aligned. B fragments come from ldmatrix.
//
// Split K: grids below one wave of two CTAs per SM split the chunks S ways
// (grid z); each split stores its tile in workspace and the tile's last split
// sums the S tiles in split order (deterministic).
//
// Both kernels are programmatic dependent launches: the pre-pass waits for
// the previous kernel before it reads x or writes the workspace; the GEMM
// requests its first weight chunks, then waits for the pre-pass.
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {
namespace {

constexpr int kRowsB = 64;                  // rows per CTA
constexpr int kWarpsB = 4;
constexpr int kThreadsB = 32 * kWarpsB;
constexpr int kChunk = 256;                 // K per stage
constexpr int kXRow = kChunk + 16;          // bytes of a limb row in shared memory (ldmatrix bank spread)
constexpr int kMaxVec = 32;
constexpr int kLimbsB = 3;                  // int8 limbs per activation element
constexpr int kSmemPerCta = 113 * 1024;     // two CTAs per SM
constexpr int kSlotsB = 2 * 148;            // CTAs resident at once
constexpr int kMaxSplitsB = 16;

// Split-K arrival counts, one per output tile (a launch splits K only when it
// has at most kSlotsB / 2 tiles); the tile's last split resets its count.
__device__ unsigned g_tile_counters[kSlotsB];

// Shared-memory bytes of one row's chunk (16-byte pieces copied): Q8_0 8 x 34
// = 272; Q4_0 8 x 18 = 144; Q4_K one 144-byte block; Q5_K one 176-byte block;
// Q6_K one 210-byte block at any even offset in a 240-byte window (60 words:
// the 8 rows a warp reads hit 8 bank groups); IQ4_XS one 136-byte block at
// offset 0 or 8 of a 144-byte window.
template <int TYPE>
__host__ __device__ constexpr int row_stride() {
    return TYPE == kTypeQ8_0 ? 272 : (TYPE == kTypeQ6_K ? 240 : (TYPE == kTypeQ5_K ? 176 : 144));
}
template <int TYPE>
__host__ __device__ constexpr int row_pieces() {  // 16-byte pieces copied per row (Q6_K: 14 cover any offset)
    return TYPE == kTypeQ8_0 ? 17 : (TYPE == kTypeQ6_K ? 14 : (TYPE == kTypeQ5_K ? 11 : 9));
}
template <int TYPE>
__host__ __device__ constexpr int window_block() {  // blocks copied through a 16-byte window: their bytes
    return TYPE == kTypeQ6_K ? 210 : (TYPE == kTypeIQ4_XS ? 136 : 0);
}
template <int TYPE>
__host__ __device__ constexpr int sum_floats() {  // x sub-block sums per vector and chunk (the mins)
    return (TYPE == kTypeQ4_K || TYPE == kTypeQ5_K) ? 16 : 0;
}

struct BatchedArgs {
    const uint8_t* w;
    int64_t w_nb1;
    const int8_t* xl;      // limbs [N][3][K]
    const float* inv_s;    // [K / 256][n_pad]
    const float* xsum;     // [K / 256][n_pad][16] (Q4_K)
    float* y;
    int64_t y_nb1;         // bytes between output vectors
    int32_t M, K, N, n_pad;
    int32_t splits, chunks_per_split;
    float* partial;        // [tile][split][kMaxVec][kRowsB]
};

template <int TYPE, int NV>
__host__ __device__ constexpr int stage_bytes() {
    return kRowsB * row_stride<TYPE>() + NV * kLimbsB * kXRow + NV * 4 + NV * 4 * sum_floats<TYPE>();
}
// Pipeline depth: as many chunks in flight (at most 4) as the shared memory
// of two CTAs per SM holds.
template <int TYPE, int NV>
__host__ __device__ constexpr int stages_of() {
    return kSmemPerCta / stage_bytes<TYPE, NV>() > 4 ? 4 : kSmemPerCta / stage_bytes<TYPE, NV>();
}
static_assert(stages_of<kTypeQ8_0, 32>() >= 2 && stages_of<kTypeQ6_K, 32>() >= 2, "two stages per CTA");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16 bytes global -> shared; zeros when !valid.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// Two 8x8 b16 matrices (lanes 0-15 supply the row addresses).
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

// D = A (16x32 s8, row) * B (32x8 s8, col), s32.
__device__ __forceinline__ void imma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D = A (16x32 u8, row) * B (32x8 s8, col), s32.
__device__ __forceinline__ void imma_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// 4 bytes at a 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);
    return __funnelshift_r(q[0], q[1], mis * 8);
}

// The eight (scale, min) pairs of a Q4_K block header h (get_scale_min_k4,
// src/inference/jsep/ops/matmul.ts:408-424): sc as an int, times 16 for the
// even (low-nibble) sub-blocks, whose quants enter the MMA unscaled; the mins
// as dmin * m.
__device__ __forceinline__ void q4k_scales8(const uint4 h, int (&sc)[8], float (&mdm)[8], float& d) {
    d = f16_bits_to_f32(h.x & 0xFFFFu);
    const float dmin = f16_bits_to_f32(h.x >> 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t sel = 0x4440u + static_cast<uint32_t>(j & 3);  // byte j%4, zero-extended
        uint32_t scv, mv;
        if (j < 4) {
            scv = __byte_perm(h.y, 0u, sel) & 63u;
            mv = __byte_perm(h.z, 0u, sel) & 63u;
        } else {
            const uint32_t b1 = __byte_perm(h.y, 0u, sel), b2 = __byte_perm(h.z, 0u, sel), b3 = __byte_perm(h.w, 0u, sel);
            scv = (b3 & 15u) | ((b1 >> 2) & 0x30u);
            mv = (b3 >> 4) | ((b2 >> 2) & 0x30u);
        }
        sc[j] = static_cast<int>(scv << ((j & 1) ? 0 : 4));
        mdm[j] = dmin * static_cast<float>(mv);
    }
}

// The scale of sub-block j alone (as in q4k_scales8).
__device__ __forceinline__ int q4k_scale_j(const uint4 h, int j) {
    const uint32_t sel = 0x4440u + static_cast<uint32_t>(j & 3);
    uint32_t scv;
    if (j < 4) {
        scv = __byte_perm(h.y, 0u, sel) & 63u;
    } else {
        const uint32_t b1 = __byte_perm(h.y, 0u, sel), b3 = __byte_perm(h.w, 0u, sel);
        scv = (b3 & 15u) | ((b1 >> 2) & 0x30u);
    }
    return static_cast<int>(scv << ((j & 1) ? 0 : 4));
}

// The A operand of 32-element group t of one Q6_K half-block at one fragment
// position: ql0 / ql1 hold four bytes of the half's low-quant chunks 0 / 1
// (ql[64h + l], ql[64h + 32 + l]), qh the four matching high-bit bytes
// (qh[32h + l]). Group t holds the 6-bit quants (0..63) of elements
// 128h + 32t + l: the low nibble of chunk t&1 for t < 2, the high nibble for
// t >= 2, and bits 2t, 2t+1 of qh as bits 4, 5 (ggml's dequantize_row_q6_K
// layout; the reference has no Q6_K code of its own).
__device__ __forceinline__ uint32_t q6k_group(uint32_t ql0, uint32_t ql1, uint32_t qh, int t) {
    const uint32_t ql = (t & 1) ? ql1 : ql0;
    const uint32_t lo = ((t & 2) ? (ql >> 4) : ql) & 0x0F0F0F0Fu;
    return lo | (((qh >> (2 * t)) & 0x03030303u) << 4);
}

// Four 4-bit quants q (0..15, one per byte) -> the int8 bytes q - 8: q ^ 8 is
// q - 8 as a 4-bit two's-complement number; copy its sign bit (bit 3) into
// bits 4..7 (0x08 * 0x1E = 0xF0 stays inside each byte).
__device__ __forceinline__ uint32_t q4_signed(uint32_t q) {
    const uint32_t t = q ^ 0x08080808u;
    return t | ((t & 0x08080808u) * 0x1Eu);
}

// Four 6-bit quants q (0..63, one per byte) -> the int8 bytes q - 32: q ^ 32
// is q - 32 as a 6-bit two's-complement number; copy its sign bit (bit 5)
// into bits 6 and 7.
__device__ __forceinline__ uint32_t q6_signed(uint32_t q) {
    const uint32_t t = q ^ 0x20202020u, s = t & 0x20202020u;
    return t | (s << 1) | (s << 2);
}

// Pre-pass: one warp per (vector, 256-element block). Launched as a
// programmatic dependent: it waits for the previous kernel before it reads x
// or writes the workspace.
__global__ void x_limbs_kernel(const float* __restrict__ x, int64_t x_nb1, int8_t* __restrict__ xl,
                               float* __restrict__ inv_s, float* __restrict__ xsum, int K, int N, int n_pad) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int nblk = K / 256;
    const int64_t item = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (item >= static_cast<int64_t>(n_pad) * nblk) return;
    const int n = static_cast<int>(item / nblk), b = static_cast<int>(item - static_cast<int64_t>(n) * nblk);
    float v[8];
    if (n < N) {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(x) + n * x_nb1) + b * 64 + 2 * lane;
        const float4 a = src[0], c = src[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float sc = mx > 0.f ? 127.f / mx : 0.f;
    uint32_t l0[2], l1[2], l2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int q0[4], q1[4], q2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // l0 = rint(x s) (|l0| <= 127), l1 = rint(r1) with r1 = 128 (x s - l0)
            // (|l1| <= 64), l2 = rint(128 (r1 - l1)) (|l2| <= 64); fmaf takes the
            // exact product x s, r1 - l1 and the scalings by 128 are exact
            const float e = v[4 * h + i];
            q0[i] = __float2int_rn(e * sc);
            const float r1 = fmaf(e, sc, -static_cast<float>(q0[i])) * 128.f;
            q1[i] = __float2int_rn(r1);
            q2[i] = __float2int_rn(__fsub_rn(r1, static_cast<float>(q1[i])) * 128.f);
        }
        l0[h] = __byte_perm(__byte_perm(q0[0], q0[1], 0x0040u), __byte_perm(q0[2], q0[3], 0x0040u), 0x5410u);
        l1[h] = __byte_perm(__byte_perm(q1[0], q1[1], 0x0040u), __byte_perm(q1[2], q1[3], 0x0040u), 0x5410u);
        l2[h] = __byte_perm(__byte_perm(q2[0], q2[1], 0x0040u), __byte_perm(q2[2], q2[3], 0x0040u), 0x5410u);
    }
    if (n < N) {
        int8_t* base = xl + (static_cast<int64_t>(n) * kLimbsB) * K + b * 256 + 8 * lane;
        *reinterpret_cast<uint2*>(base) = make_uint2(l0[0], l0[1]);
        *reinterpret_cast<uint2*>(base + K) = make_uint2(l1[0], l1[1]);
        *reinterpret_cast<uint2*>(base + 2 * K) = make_uint2(l2[0], l2[1]);
    }
    if (lane == 0) inv_s[static_cast<int64_t>(b) * n_pad + n] = mx * (1.f / 127.f);
    if (xsum) {
        // 16-element sums: lanes 2i, 2i+1 hold sub-block i
        const float s8 = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        const float s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
        if ((lane & 1) == 0) xsum[(static_cast<int64_t>(b) * n_pad + n) * 16 + (lane >> 1)] = s16;
    }
}

// The three limbs of one vector octet times one A fragment (32 elements at
// shared addresses xa01: limbs 0 and 1, xa2: limb 2), combined in f32:
// v = D0 + D1 / 128 + D2 / 16384 for the lane's four accumulator elements
// (rows g, g + 8 x vectors 2c, 2c + 1 of the octet). |D| < 2^20, so each
// conversion is exact and the sum is rounded twice (2^-24 relative).
template <bool U8>
__device__ __forceinline__ void mma_limbs(float (&v)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t xa01, uint32_t xa2) {
    uint32_t b01[4], b2[2];
    ldmatrix_x4(b01, xa01);
    ldmatrix_x2(b2, xa2);
    int D0[4], D1[4], D2[4];
    if (U8) {
        imma_u8(D0, a0, a1, a2, a3, b01[0], b01[1]);
        imma_u8(D1, a0, a1, a2, a3, b01[2], b01[3]);
        imma_u8(D2, a0, a1, a2, a3, b2[0], b2[1]);
    } else {
        imma_s8(D0, a0, a1, a2, a3, b01[0], b01[1]);
        imma_s8(D1, a0, a1, a2, a3, b01[2], b01[3]);
        imma_s8(D2, a0, a1, a2, a3, b2[0], b2[1]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
        v[e] = fmaf(static_cast<float>(D2[e]), 6.103515625e-05f,
                    fmaf(static_cast<float>(D1[e]), 0.0078125f, static_cast<float>(D0[e])));
}

template <int TYPE, int NV>
__global__ void __launch_bounds__(kThreadsB, 2) batched_kernel(const __grid_constant__ BatchedArgs P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RS = row_stride<TYPE>();
    constexpr int RP = row_pieces<TYPE>();
    constexpr int SB = stage_bytes<TYPE, NV>();
    constexpr int NO = NV / 8;                       // vector octets (one MMA column tile per limb)
    constexpr uint32_t OCT = 8 * kLimbsB * kXRow;   // shared bytes between octets
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int m0 = blockIdx.x * kRowsB, n0 = blockIdx.y * NV;
    const int nchunks = P.K / kChunk;
    const int ch0 = blockIdx.z * P.chunks_per_split;
    const int nch = min(nchunks - ch0, P.chunks_per_split);

    // one chunk's copies: 64 rows x RP pieces of 16 B (load_w), NV x 3 limb
    // rows x 16 pieces, NV factors (16 B pieces of 4), NV x 16 sums (load_x)
    auto load_w = [&](int ch, int buf) {
        uint8_t* sw = smem + buf * SB;
        const int k0 = (ch0 + ch) * kChunk;
        for (int i = threadIdx.x; i < kRowsB * RP; i += kThreadsB) {
            const int r = i / RP, pc = i - r * RP;
            bool ok = m0 + r < P.M;
            const uint8_t* row = P.w + static_cast<int64_t>(ok ? m0 + r : 0) * P.w_nb1;
            const uint8_t* src;
            if (TYPE == kTypeQ8_0) {
                src = row + (k0 / 32) * 34 + 16 * pc;
            } else if (TYPE == kTypeQ4_0) {
                src = row + (k0 / 32) * 18 + 16 * pc;
            } else if (TYPE == kTypeQ4_K) {
                src = row + (k0 / 256) * 144 + 16 * pc;
            } else if (TYPE == kTypeQ5_K) {
                src = row + (k0 / 256) * 176 + 16 * pc;
            } else {
                // Q6_K / IQ4_XS: the 16-byte pieces that meet the block (none past
                // the 16-byte boundary after its last byte)
                constexpr int WB = window_block<TYPE>();
                const uintptr_t a = reinterpret_cast<uintptr_t>(row + (k0 / 256) * WB);
                const uintptr_t ga = a & ~uintptr_t(15);
                ok = ok && ga + 16 * pc < a + WB;
                src = reinterpret_cast<const uint8_t*>(ga + 16 * pc);
            }
            cp_async16(sw + r * RS + 16 * pc, ok ? src : P.w, ok);
        }
    };
    auto load_x = [&](int ch, int buf) {
        uint8_t* sx = smem + buf * SB + kRowsB * RS;
        uint8_t* ss = sx + NV * kLimbsB * kXRow;
        uint8_t* su = ss + NV * 4;
        const int k0 = (ch0 + ch) * kChunk;
        for (int i = threadIdx.x; i < NV * kLimbsB * 16; i += kThreadsB) {
            const int rowl = i >> 4, pc = i & 15;  // rowl = 3 v + limb
            const int v = rowl / kLimbsB, l = rowl - v * kLimbsB;
            const bool ok = n0 + v < P.N;
            const int8_t* src = P.xl + (static_cast<int64_t>(ok ? n0 + v : 0) * kLimbsB + l) * P.K + k0 + 16 * pc;
            cp_async16(sx + rowl * kXRow + 16 * pc, src, ok);
        }
        for (int i = threadIdx.x; i < NV / 4; i += kThreadsB) {
            const int v = 4 * i;
            const bool ok = n0 + v < P.n_pad;
            cp_async16(ss + 16 * i, P.inv_s + static_cast<int64_t>(ch0 + ch) * P.n_pad + (ok ? n0 + v : 0), ok);
        }
        if (sum_floats<TYPE>() > 0) {
            for (int i = threadIdx.x; i < NV * 4; i += kThreadsB) {
                const int v = i >> 2, pc = i & 3;
                const bool ok = n0 + v < P.n_pad;
                cp_async16(su + 16 * i,
                           P.xsum + (static_cast<int64_t>(ch0 + ch) * P.n_pad + (ok ? n0 + v : 0)) * 16 + 4 * pc, ok);
            }
        }
    };

    // lane (g, c): rows g, g + 8 of the warp's 16 x vectors 8 o + 2c, 8 o + 2c + 1
    float acc[NO][4];
#pragma unroll
    for (int o = 0; o < NO; ++o) acc[o][0] = acc[o][1] = acc[o][2] = acc[o][3] = 0.f;

    // ldmatrix row addresses: matrix mi = lane/8, row rr = lane%8 = B column =
    // vector rr of the octet; x4: limb mi/2, k half mi&1; x2 (lanes 0-15):
    // limb 2, k half mi
    const int mi = lane >> 3, rr = lane & 7;
    const uint32_t xoff01 = static_cast<uint32_t>((kLimbsB * rr + (mi >> 1)) * kXRow + 16 * (mi & 1));
    const uint32_t xoff2 = static_cast<uint32_t>((kLimbsB * rr + 2) * kXRow + 16 * (mi & 1));
    // Q6_K: where row g / g+8's block sits in its 16-byte window (the window
    // offset changes by 210 mod 16 from chunk to chunk)
    const uintptr_t rowg_addr =
        reinterpret_cast<uintptr_t>(P.w) + static_cast<uintptr_t>(static_cast<int64_t>(m0 + 16 * warp + g) * P.w_nb1);
    const uintptr_t rowh_addr = rowg_addr + static_cast<uintptr_t>(8 * P.w_nb1);

    // Programmatic dependent launch: the first chunks' weights are requested
    // before the wait for the kernel that writes the activations (the x
    // pre-pass); they join the first chunk's copy group.
    constexpr int ST = stages_of<TYPE, NV>();
#pragma unroll
    for (int sidx = 0; sidx < ST - 1; ++sidx)
        if (sidx < nch) load_w(sidx, sidx);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int sidx = 0; sidx < ST - 1; ++sidx) {
        if (sidx < nch) load_x(sidx, sidx);
        cp_async_commit();
    }
    for (int ch = 0; ch < nch; ++ch) {
        cp_async_wait<ST - 2>();  // chunk ch has landed
        __syncthreads();          // ... for every thread, and chunk ch - 1's buffer is free
        if (ch + ST - 1 < nch) {
            load_w(ch + ST - 1, (ch + ST - 1) % ST);
            load_x(ch + ST - 1, (ch + ST - 1) % ST);
        }
        cp_async_commit();
        const uint8_t* sw = smem + (ch % ST) * SB;
        const uint8_t* sx = sw + kRowsB * RS;
        const float* ss = reinterpret_cast<const float*>(sx + NV * kLimbsB * kXRow);
        const float* su = ss + NV;
        const uint32_t xb01 = smem_u32(sx) + xoff01, xb2 = smem_u32(sx) + xoff2;
        const uint8_t* rg = sw + (16 * warp + g) * RS;
        const uint8_t* rh = rg + 8 * RS;
        float is[NO][2];  // 1 / s of the lane's two vectors in each octet
#pragma unroll
        for (int o = 0; o < NO; ++o) {
            is[o][0] = ss[8 * o + 2 * c];
            is[o][1] = ss[8 * o + 2 * c + 1];
        }

        if (TYPE == kTypeQ8_0 || TYPE == kTypeQ4_0) {
            constexpr int BB = TYPE == kTypeQ8_0 ? 34 : 18;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const uint8_t* bg = rg + BB * b;
                const uint8_t* bh = rh + BB * b;
                const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bg));
                const float dh = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bh));
                uint32_t a0, a1, a2, a3;
                if (TYPE == kTypeQ8_0) {
                    a0 = lds_u32_any(bg + 2 + 4 * c);
                    a1 = lds_u32_any(bh + 2 + 4 * c);
                    a2 = lds_u32_any(bg + 18 + 4 * c);
                    a3 = lds_u32_any(bh + 18 + 4 * c);
                } else {
                    // elements 4c.. are the low nibbles, 16+4c.. the high ones
                    const uint32_t wg = lds_u32_any(bg + 2 + 4 * c), wh = lds_u32_any(bh + 2 + 4 * c);
                    a0 = q4_signed(wg & 0x0F0F0F0Fu);
                    a1 = q4_signed(wh & 0x0F0F0F0Fu);
                    a2 = q4_signed((wg >> 4) & 0x0F0F0F0Fu);
                    a3 = q4_signed((wh >> 4) & 0x0F0F0F0Fu);
                }
#pragma unroll
                for (int o = 0; o < NO; ++o) {
                    float v[4];
                    mma_limbs<false>(v, a0, a1, a2, a3, xb01 + o * OCT + 32 * b, xb2 + o * OCT + 32 * b);
                    acc[o][0] = fmaf(v[0], dg * is[o][0], acc[o][0]);
                    acc[o][1] = fmaf(v[1], dg * is[o][1], acc[o][1]);
                    acc[o][2] = fmaf(v[2], dh * is[o][0], acc[o][2]);
                    acc[o][3] = fmaf(v[3], dh * is[o][1], acc[o][3]);
                }
            }
        } else if (TYPE == kTypeQ4_K || TYPE == kTypeQ5_K) {
            // Q4_K: nibbles (low as they are, high in place = 16 q) times 16 sc /
            // sc; Q5_K: the 5-bit quants (nibble | qh bit j << 4) times sc
            constexpr bool k5 = TYPE == kTypeQ5_K;
            constexpr int QS = k5 ? 48 : 16;  // quant bytes in the block
            const uint4 hg = *reinterpret_cast<const uint4*>(rg), hh4 = *reinterpret_cast<const uint4*>(rh);
            // Q5_K high-bit words qh[4c..], qh[16+4c..] of rows g / g+8
            uint32_t hb[4] = {0u, 0u, 0u, 0u};
            if (k5) {
                hb[0] = *reinterpret_cast<const uint32_t*>(rg + 16 + 4 * c);
                hb[1] = *reinterpret_cast<const uint32_t*>(rh + 16 + 4 * c);
                hb[2] = *reinterpret_cast<const uint32_t*>(rg + 32 + 4 * c);
                hb[3] = *reinterpret_cast<const uint32_t*>(rh + 32 + 4 * c);
            }
            float af[NO][4];  // the block's scaled sub-block sums
#pragma unroll
            for (int o = 0; o < NO; ++o) af[o][0] = af[o][1] = af[o][2] = af[o][3] = 0.f;
#pragma unroll 1
            for (int p = 0; p < 4; ++p) {
                // fragment words of sub-block pair p (qs bytes 32p .. 32p+31): row
                // g / g+8, k 4c.. / 16+4c..
                const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rg + QS + 32 * p + 4 * c);
                const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rh + QS + 32 * p + 4 * c);
                const uint32_t w2 = *reinterpret_cast<const uint32_t*>(rg + QS + 16 + 32 * p + 4 * c);
                const uint32_t w3 = *reinterpret_cast<const uint32_t*>(rh + QS + 16 + 32 * p + 4 * c);
#pragma unroll
                for (int hi = 0; hi < 2; ++hi) {
                    const int j = 2 * p + hi;
                    uint32_t A[4];
                    if (k5) {
                        const uint32_t w[4] = {w0, w1, w2, w3};
#pragma unroll
                        for (int r = 0; r < 4; ++r)
                            A[r] = ((hi ? (w[r] >> 4) : w[r]) & 0x0F0F0F0Fu) | (((hb[r] >> j) & 0x01010101u) << 4);
                    } else {
                        const uint32_t msk = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
                        A[0] = w0 & msk;
                        A[1] = w1 & msk;
                        A[2] = w2 & msk;
                        A[3] = w3 & msk;
                    }
                    // (q4k_scale_j gives 16 sc for even j: Q5_K takes sc)
                    const float scj = static_cast<float>(q4k_scale_j(hg, j) >> (k5 && !hi ? 4 : 0));
                    const float shj = static_cast<float>(q4k_scale_j(hh4, j) >> (k5 && !hi ? 4 : 0));
#pragma unroll
                    for (int o = 0; o < NO; ++o) {
                        float v[4];
                        mma_limbs<true>(v, A[0], A[1], A[2], A[3], xb01 + o * OCT + 32 * j, xb2 + o * OCT + 32 * j);
                        af[o][0] = fmaf(scj, v[0], af[o][0]);
                        af[o][1] = fmaf(scj, v[1], af[o][1]);
                        af[o][2] = fmaf(shj, v[2], af[o][2]);
                        af[o][3] = fmaf(shj, v[3], af[o][3]);
                    }
                }
            }
            int scg[8], sch[8];
            float mg[8], mh[8], dg, dh;
            q4k_scales8(hg, scg, mg, dg);
            q4k_scales8(hh4, sch, mh, dh);
#pragma unroll
            for (int o = 0; o < NO; ++o) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {  // the lane's vectors 8 o + 2 c + e
                    const float* xs = su + (8 * o + 2 * c + e) * 16;  // its 16-element sums
                    float og = 0.f, oh = 0.f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float X = xs[2 * j] + xs[2 * j + 1];
                        og = fmaf(mg[j], X, og);
                        oh = fmaf(mh[j], X, oh);
                    }
                    const float f = k5 ? is[o][e] : is[o][e] * 0.0625f;
                    acc[o][e] += fmaf(dg * af[o][e], f, -og);
                    acc[o][2 + e] += fmaf(dh * af[o][2 + e], f, -oh);
                }
            }
        } else if (TYPE == kTypeIQ4_XS) {
            // IQ4_XS: sub-block j's A fragment for rows g / g+8 is the levels of the
            // low nibbles of index bytes 16j + 4c .. + 3 (k = 4c ..) and of their high
            // nibbles (k = 16 + 4c ..); times ls_j - 32 in f32, then d / s per block
            const uintptr_t boff = static_cast<uintptr_t>((ch0 + ch) * 136);
            const uint8_t* pg = rg + ((rowg_addr + boff) & 15);
            const uint8_t* ph = rh + ((rowh_addr + boff) & 15);
            const uint32_t shg = *reinterpret_cast<const uint16_t*>(pg + 2), slg = *reinterpret_cast<const uint32_t*>(pg + 4);
            const uint32_t shh = *reinterpret_cast<const uint16_t*>(ph + 2), slh = *reinterpret_cast<const uint32_t*>(ph + 4);
            float af[NO][4];  // the block's scaled sub-block sums
#pragma unroll
            for (int o = 0; o < NO; ++o) af[o][0] = af[o][1] = af[o][2] = af[o][3] = 0.f;
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {
                const uint32_t wg = *reinterpret_cast<const uint32_t*>(pg + 8 + 16 * j + 4 * c);
                const uint32_t wh = *reinterpret_cast<const uint32_t*>(ph + 8 + 16 * j + 4 * c);
                uint32_t A0, A1, A2, A3;  // levels: rows g / g+8, low / high nibbles
                iq4_lut8(wg, A0, A2);
                iq4_lut8(wh, A1, A3);
                const float scj = static_cast<float>(iq4xs_scale(shg, slg, j));
                const float shj = static_cast<float>(iq4xs_scale(shh, slh, j));
#pragma unroll
                for (int o = 0; o < NO; ++o) {
                    float v[4];
                    mma_limbs<false>(v, A0, A1, A2, A3, xb01 + o * OCT + 32 * j, xb2 + o * OCT + 32 * j);
                    af[o][0] = fmaf(scj, v[0], af[o][0]);
                    af[o][1] = fmaf(scj, v[1], af[o][1]);
                    af[o][2] = fmaf(shj, v[2], af[o][2]);
                    af[o][3] = fmaf(shj, v[3], af[o][3]);
                }
            }
            const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(pg));
            const float dh = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ph));
#pragma unroll
            for (int o = 0; o < NO; ++o) {
                acc[o][0] = fmaf(dg * af[o][0], is[o][0], acc[o][0]);
                acc[o][1] = fmaf(dg * af[o][1], is[o][1], acc[o][1]);
                acc[o][2] = fmaf(dh * af[o][2], is[o][0], acc[o][2]);
                acc[o][3] = fmaf(dh * af[o][3], is[o][1], acc[o][3]);
            }
        } else {
            // Q6_K: the block of row g / g+8 at its offset in the 16-byte window
            const uintptr_t boff = static_cast<uintptr_t>((ch0 + ch) * 210);
            const uint8_t* pg = rg + ((rowg_addr + boff) & 15);
            const uint8_t* ph = rh + ((rowh_addr + boff) & 15);
            float af[NO][4];  // the block's scaled sub-block sums
#pragma unroll
            for (int o = 0; o < NO; ++o) af[o][0] = af[o][1] = af[o][2] = af[o][3] = 0.f;
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                // the fragment words of half h at position r (0: row g k 4c.., 1: row
                // g+8, 2: row g k 16+4c.., 3: row g+8): low-quant chunks 0, 1, high bits
                uint32_t q0[4], q1[4], qb[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const uint8_t* b = ((r & 1) ? ph : pg) + 4 * c + 16 * (r >> 1);
                    q0[r] = lds_u32_any(b + 64 * h);
                    q1[r] = lds_u32_any(b + 64 * h + 32);
                    qb[r] = lds_u32_any(b + 128 + 32 * h);
                }
#pragma unroll 1
                for (int gi = 0; gi < 4; ++gi) {  // elements 32i .. 32i+31 (i = 4h + gi): sub-blocks 2i, 2i+1
                    const int i = 4 * h + gi;
                    uint32_t A[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) A[r] = q6_signed(q6k_group(q0[r], q1[r], qb[r], gi));
                    const float sge = static_cast<float>(*reinterpret_cast<const int8_t*>(pg + 192 + 2 * i));
                    const float sgo = static_cast<float>(*reinterpret_cast<const int8_t*>(pg + 193 + 2 * i));
                    const float she = static_cast<float>(*reinterpret_cast<const int8_t*>(ph + 192 + 2 * i));
                    const float sho = static_cast<float>(*reinterpret_cast<const int8_t*>(ph + 193 + 2 * i));
#pragma unroll
                    for (int o = 0; o < NO; ++o) {
                        // the two 16-element sub-blocks on separate MMAs (the other
                        // half of the A fragment zero)
                        float ve[4], vo[4];
                        mma_limbs<false>(ve, A[0], A[1], 0u, 0u, xb01 + o * OCT + 32 * i, xb2 + o * OCT + 32 * i);
                        mma_limbs<false>(vo, 0u, 0u, A[2], A[3], xb01 + o * OCT + 32 * i, xb2 + o * OCT + 32 * i);
                        af[o][0] = fmaf(sge, ve[0], fmaf(sgo, vo[0], af[o][0]));
                        af[o][1] = fmaf(sge, ve[1], fmaf(sgo, vo[1], af[o][1]));
                        af[o][2] = fmaf(she, ve[2], fmaf(sho, vo[2], af[o][2]));
                        af[o][3] = fmaf(she, ve[3], fmaf(sho, vo[3], af[o][3]));
                    }
                }
            }
            const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(pg + 208));
            const float dh = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(ph + 208));
#pragma unroll
            for (int o = 0; o < NO; ++o) {
                acc[o][0] = fmaf(dg * is[o][0], af[o][0], acc[o][0]);
                acc[o][1] = fmaf(dg * is[o][1], af[o][1], acc[o][1]);
                acc[o][2] = fmaf(dh * is[o][0], af[o][2], acc[o][2]);
                acc[o][3] = fmaf(dh * is[o][1], af[o][3], acc[o][3]);
            }
        }
    }

    // ---- outputs: lane (g, c) holds rows 16 warp + g (+8) of vectors 8 o + 2 c (+1) ----
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (P.splits == 1) {
#pragma unroll
        for (int o = 0; o < NO; ++o) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int n = n0 + 8 * o + 2 * c + e;
                if (n >= P.N) continue;
                float* yn = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1);
                const int r = m0 + 16 * warp + g;
                if (r < P.M) yn[r] = acc[o][e];
                if (r + 8 < P.M) yn[r + 8] = acc[o][2 + e];
            }
        }
        return;
    }
    float* part = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kMaxVec * kRowsB);
#pragma unroll
    for (int o = 0; o < NO; ++o) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int v = 8 * o + 2 * c + e;
            part[v * kRowsB + 16 * warp + g] = acc[o][e];
            part[v * kRowsB + 16 * warp + g + 8] = acc[o][2 + e];
        }
    }
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // this split's tile before the count
        last = atomicAdd(g_tile_counters + tile, 1u) == static_cast<unsigned>(P.splits - 1);
        if (last) {
            g_tile_counters[tile] = 0u;
            __threadfence();  // the other splits' tiles after the count
        }
    }
    __syncthreads();
    if (!last) return;
    // the tile's last split: sum the splits in order; thread = one row, 4 vectors at a time
    const float* base = P.partial + static_cast<int64_t>(tile) * P.splits * (kMaxVec * kRowsB);
    for (int i = threadIdx.x; i < NV * kRowsB; i += kThreadsB) {
        const int v = i / kRowsB, r = i - v * kRowsB;
        float s = 0.f;
        for (int z = 0; z < P.splits; ++z) s += __ldcg(base + z * (kMaxVec * kRowsB) + i);
        const int n = n0 + v, row = m0 + r;
        if (n < P.N && row < P.M) reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1)[row] = s;
    }
}

// Vectors per CTA tile: N rounded up to 8, 16 or 32; wider N takes several
// 32-vector tiles (a 64-vector tile's three limb rows per vector would leave
// room for one CTA per SM).
int pick_nv(const MulMatOp& o) {
    const int N = o.N;
    return N <= 8 ? 8 : (N <= 16 ? 16 : 32);
}

void plan(const MulMatOp& o, int* nv, int* splits, int* cps) {
    *nv = pick_nv(o);
    const int tiles = ((o.M + kRowsB - 1) / kRowsB) * ((o.N + *nv - 1) / *nv);
    const int nchunks = o.K / kChunk;
    int s = kSlotsB / tiles;                         // at most one wave of two CTAs per SM
    s = s < kMaxSplitsB ? s : kMaxSplitsB;
    s = s < (nchunks + 1) / 2 ? s : (nchunks + 1) / 2;  // at least two chunks per split
    s = s > 1 ? s : 1;
    *cps = (nchunks + s - 1) / s;
    *splits = (nchunks + *cps - 1) / *cps;           // no empty split
}

int n_pad_of(const MulMatOp& o) { return (o.N + 3) & ~3; }
size_t limbs_bytes(const MulMatOp& o) { return (static_cast<size_t>(o.N) * kLimbsB * o.K + 255) & ~size_t(255); }
size_t factors_bytes(const MulMatOp& o) {
    return (static_cast<size_t>(o.K / 256) * n_pad_of(o) * 4 + 255) & ~size_t(255);
}
size_t sums_bytes(const MulMatOp& o) {
    if (o.type != kTypeQ4_K && o.type != kTypeQ5_K) return 0;
    return (static_cast<size_t>(o.K / 256) * n_pad_of(o) * 16 * 4 + 255) & ~size_t(255);
}
size_t partial_bytes(const MulMatOp& o) {
    int nv, s, cps;
    plan(o, &nv, &s, &cps);
    if (s <= 1) return 0;
    const size_t tiles = static_cast<size_t>((o.M + kRowsB - 1) / kRowsB) * ((o.N + nv - 1) / nv);
    return tiles * s * kMaxVec * kRowsB * 4;
}

template <int TYPE, int NV>
cudaError_t launch_nv(const BatchedArgs& P, dim3 grid, cudaStream_t stream) {
    constexpr int smem = stages_of<TYPE, NV>() * stage_bytes<TYPE, NV>();
    // the attribute is per device: one flag per device ordinal
    static bool configured[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return e0;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(batched_kernel<TYPE, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreadsB);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, batched_kernel<TYPE, NV>, P);
    return e == cudaSuccess ? cudaGetLastError() : e;
}

template <int TYPE>
cudaError_t launch_type(int nv, const BatchedArgs& P, dim3 grid, cudaStream_t stream) {
    switch (nv) {
        case 8: return launch_nv<TYPE, 8>(P, grid, stream);
        case 16: return launch_nv<TYPE, 16>(P, grid, stream);
        default: return launch_nv<TYPE, 32>(P, grid, stream);
    }
}

}  // namespace

bool batched_supported(const MulMatOp& o) {
    if (o.type != kTypeQ8_0 && o.type != kTypeQ4_K && o.type != kTypeQ6_K && o.type != kTypeQ5_K &&
        o.type != kTypeQ4_0 && o.type != kTypeIQ4_XS)
        return false;
    if (o.N < 3 || o.ne2 != 1 || o.ne3 != 1) return false;
    if (o.K % 256 != 0 || o.M < 1) return false;
    const uintptr_t wa = reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1);
    // 16-byte copies (Q6_K: 2-byte loads; IQ4_XS: 4-byte loads from 8-byte aligned blocks)
    if (o.type == kTypeQ6_K ? (wa & 1) : (o.type == kTypeIQ4_XS ? (wa & 7) : (wa & 15))) return false;
    if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;  // float4 reads
    return true;
}

size_t batched_workspace_bytes(const MulMatOp& o) {
    return limbs_bytes(o) + factors_bytes(o) + sums_bytes(o) + partial_bytes(o) + 256;
}

int launch_batched(const MulMatOp& o, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!batched_supported(o)) return -static_cast<int>(cudaErrorInvalidValue);
    if (!workspace || workspace_bytes < batched_workspace_bytes(o) || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return -static_cast<int>(cudaErrorInvalidValue);
    int nv, splits, cps;
    plan(o, &nv, &splits, &cps);
    BatchedArgs P{};
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    P.w = o.w;
    P.w_nb1 = o.w_nb1;
    P.xl = reinterpret_cast<int8_t*>(ws);
    P.inv_s = reinterpret_cast<float*>(ws + limbs_bytes(o));
    P.xsum = (o.type == kTypeQ4_K || o.type == kTypeQ5_K)
                 ? reinterpret_cast<float*>(ws + limbs_bytes(o) + factors_bytes(o))
                 : nullptr;
    P.y = o.y;
    P.y_nb1 = o.y_nb1;
    P.M = o.M;
    P.K = o.K;
    P.N = o.N;
    P.n_pad = n_pad_of(o);
    P.splits = splits;
    P.chunks_per_split = cps;
    const int tiles_m = (o.M + kRowsB - 1) / kRowsB, tiles_n = (o.N + nv - 1) / nv;
    if (splits > 1) P.partial = reinterpret_cast<float*>(ws + limbs_bytes(o) + factors_bytes(o) + sums_bytes(o));
    if (splits > 1 && tiles_m * tiles_n > kSlotsB) return -static_cast<int>(cudaErrorInvalidValue);  // (plan keeps it below)
    {
        const int64_t items = static_cast<int64_t>(P.n_pad) * (o.K / 256);
        const int64_t blocks = (items * 32 + 255) / 256;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(blocks));
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, x_limbs_kernel, o.x, o.x_nb1, const_cast<int8_t*>(P.xl),
                                           const_cast<float*>(P.inv_s), const_cast<float*>(P.xsum), o.K, o.N, P.n_pad);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return -static_cast<int>(e);
    }
    const dim3 grid(tiles_m, tiles_n, splits);
    cudaError_t e;
    switch (o.type) {
        case kTypeQ8_0: e = launch_type<kTypeQ8_0>(nv, P, grid, stream); break;
        case kTypeQ4_K: e = launch_type<kTypeQ4_K>(nv, P, grid, stream); break;
        case kTypeQ5_K: e = launch_type<kTypeQ5_K>(nv, P, grid, stream); break;
        case kTypeQ4_0: e = launch_type<kTypeQ4_0>(nv, P, grid, stream); break;
        case kTypeIQ4_XS: e = launch_type<kTypeIQ4_XS>(nv, P, grid, stream); break;
        default: e = launch_type<kTypeQ6_K>(nv, P, grid, stream); break;
    }
    return e == cudaSuccess ? 2 : -static_cast<int>(e);
}

}  // namespace wllm
