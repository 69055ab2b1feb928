// Decode-regime quantized MUL_MAT (N = 1 or 2 activation vectors): a
// persistent, warp-specialised streaming GEMV over raw GGUF blocks.
//
// Data movement. The weight matrix is cut into units of 16 rows (one MMA
// tile); each unit's rows into segments of at most 9 Q4_K / 6 Q6_K / 32 Q8_0
// blocks. Warp 0 (producer) moves each (unit, segment) into a ring of shared
// memory stages with ONE 2D tensor-map TMA copy (16 rows x the segment,
// rounded out to 16-byte columns; evict-first L2 policy, each weight byte is
// read once). Under load a box takes ~2 us to land, so a CTA keeps several
// stages in flight and two CTAs share an SM: ~140 KB of weights in flight per
// SM, enough to run HBM at full rate while the consumers wait for the
// activations of a dependent launch. Row layouts whose stride is not a
// multiple of 16 bytes (Q6_K with an odd number of 256-blocks per 8) fall back
// to one bulk copy per row. When a Q4_K stage lands the producer decodes its
// 6-bit scales and mins into a float table and releases the stage through a
// `ready` mbarrier. Eight consumer warps take work items (one block of a unit,
// all 16 rows) round-robin from the CTA's item sequence without CTA-wide
// barriers; the per-warp partial sums of a unit meet in shared memory and the
// warp that finishes the unit last writes it out (fixed summation order, so
// results are deterministic).
//
// Activations. After griddepcontrol.wait each CTA loads x with one L2 round
// trip and builds its shared-memory image: for Q4_K the tensor-core B
// fragments (two f16 limbs hi = f16(x s), lo = f16(x s - hi), s a power of two
// per vector so x s stays inside f16 range) and the sub-block sums of x; for
// Q6_K/Q8_0 a bank-conflict-free permutation of x.
//
// Q4_K runs on tensor cores (mma.sync m16n8k16, f16 x f16 -> f32). A 4-bit
// quant enters as the exact f16 subnormal q * 2^-24 (one LOP3 per two quants:
// low nibbles (v & 0x000F000F), high nibbles (v & 0x00F000F0) = 16 q * 2^-24),
// so every product is exact and 22 bits of x take part. Each 32-element
// sub-block is its own accumulator chain of two k16 MMAs, scaled in f32 by
// d*sc from the table; the min term dmin*m*sum(x) is subtracted in f32. The k
// order inside an MMA is a fixed permutation shared by A and B.
//
// Q6_K and Q8_0 run on CUDA cores: lanes 8j..8j+7 take row 4q+j (q = 0..3),
// lane chunk c = lane%8 owns 32 elements of a 256-element block (Q6_K) or one
// 32-element block (Q8_0). A 6-bit quant becomes the float 1 + q/128 with one
// byte permute (0x80|q in bits 16..23 of 0x3F800000); S = sum (1 + q/128) x
// runs on packed FFMA2 and the quant sum is 128 (S - X), X = sum x.
//
// Launch: programmatic dependent launch. CTAs trigger their dependents at
// entry; the producer streams weights (never written by a preceding kernel)
// at once; consumers execute griddepcontrol.wait before reading activations or
// writing outputs. Every mbarrier wait is bounded; on timeout the CTA records
// an error code for the host and stops waiting, so it still ends.
#include <cuda.h>  // CUtensorMap types only; the encoder is fetched with cudaGetDriverEntryPoint
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_stream_error = 0;

namespace {

constexpr int kCW = 8;                        // consumer warps
constexpr int kThreads = 32 * (kCW + 2);      // + copy warp + hand-off warp
constexpr int kRows = 16;                     // rows per unit (one MMA m-tile)
constexpr int kQ4kSegBlocks = 9;              // <= 1296 B per row and stage
constexpr int kQ6kSegBlocks = 6;              // <= 1260 B (+ 16-byte window slack)
constexpr int kQ80SegBlocks = 32;             // 1088 B, whole 8-block groups
constexpr int kMaxStages = 8;
constexpr int kUnitSlots = kMaxStages + 2;    // units a CTA can have in flight, plus margin
constexpr int kMaxNT = 2;
constexpr int kXF4 = 16;                      // float4 of x per consumer thread: K <= 16384
constexpr uint32_t kSpinLimit = 1u << 26;     // polls before a wait gives up (well over a second)
constexpr int kSmemBudget = 200 * 1024;       // one CTA per SM, up to 8 stages in flight

struct SOp {
    CUtensorMap tmap;             // weights as 2D [M rows][row bytes / 8] uint64 (when use_tma)
    const uint8_t* w;
    const float* x;
    float* y;
    int64_t w_nb1, x_nb1, y_nb1;  // bytes
    int32_t type, M, K, N;
    int32_t unit_begin;           // first unit of this op
    int32_t seg_blocks;           // blocks per segment (last may be shorter)
    int32_t nseg;
    int32_t wbox;                 // bytes per row in a stage (copy window, == 16 mod 32)
    int32_t use_tma;              // 1: one 2D tensor copy per stage; 0: one bulk copy per row
};

struct SList {
    SOp op[kMaxOpsPerLaunch];
    int32_t n_ops;
    int32_t total_units;
    int32_t stages;
    int32_t stage_bytes;  // 16 rows x the largest wbox
    int32_t tab_blocks;   // Q4_K scale-table blocks per stage (0: no Q4_K op)
    int32_t x_bytes;      // shared-memory bytes reserved for the activation image
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Potentially blocking test without a suspend-time hint: with a hint the
// waiting thread was measured to wake up microseconds after the phase
// completed, which halved the pipeline's throughput.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait. If the phase does not complete in time the CTA is poisoned:
// an error code is recorded for the host and every later wait of the CTA
// returns at once, so all threads run to the end (results are garbage, the
// error is reported by wllm_sync).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*poisoned) return false;
    }
    *poisoned = 1;
    atomicOr(&g_stream_error, code);
    return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// One 2D tensor-map box (x in uint64 elements, y in rows) into shared memory.
__device__ __forceinline__ void tma_2d_g2s(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar,
                                           uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory");
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1, const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__host__ __device__ __forceinline__ int seg_cap(int type) {
    return type == kTypeQ4_K ? kQ4kSegBlocks : (type == kTypeQ6_K ? kQ6kSegBlocks : kQ80SegBlocks);
}
__device__ __forceinline__ int block_elems_of(int type) { return type == kTypeQ8_0 ? 32 : 256; }
__device__ __forceinline__ int block_bytes_of(int type) {
    return type == kTypeQ4_K ? 144 : (type == kTypeQ6_K ? 210 : 34);
}

// Byte layout of the shared-memory activation image.
__host__ __device__ __forceinline__ int img_xb_bytes(int K, int N) { return (K / 256) * 16 * 8 * N * 8; }
__host__ __device__ __forceinline__ int img_bytes(int type, int K, int N) {
    if (type == kTypeQ4_K) return img_xb_bytes(K, N) + N * (K / 32) * 4 + 16;  // B frags, sub-block sums, 1/s
    return 4 * K * N;
}

// 1 + q/128 for the byte 0x80|q in byte position k of w.
template <int k>
__device__ __forceinline__ float unit_q(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7044u | (k << 8)));
}

// Element offset (within its 256-element group) of float4 f of lane chunk c
// (CUDA-core formats); the image is xs4[group][f][c].
__device__ __forceinline__ int chunk_elem(int type, int c, int f) {
    if (type == kTypeQ6_K) {
        const int h = c >> 2, l0 = 8 * (c & 3), t = f >> 1;
        return 128 * h + 32 * t + l0 + 4 * (f & 1);
    }
    return 32 * c + 4 * f;  // Q8_0: lane chunk c is block c of the group
}

// 4 bytes at any 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);
    return __funnelshift_r(q[0], q[1], mis * 8);
}
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// f16 limbs of v: hi = f16(v), lo = f16(v - hi).
__device__ __forceinline__ void limbs(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

// Power of two s with max|x s| in [2^14, 2^15) (1 when max is 0 or not finite).
__device__ __forceinline__ float limb_scale(float maxabs) {
    const uint32_t bits = __float_as_uint(maxabs);
    const int e = static_cast<int>((bits >> 23) & 0xFF);
    if (maxabs == 0.f || e == 0xFF) return 1.f;
    int se = 14 - (e - 127) + 127;  // exponent field of 2^(14 - e)
    se = se < 1 ? 1 : (se > 254 ? 254 : se);
    return __uint_as_float(static_cast<uint32_t>(se) << 23);
}

// Scale-table entries of one (row, block), pair p at out[16 p]: d*sc*2^24
// (low sub-block), d*sc*2^20 (high sub-block, whose quants enter as 16 q),
// dmin*m low, high. The table of a stage is [block][pair][16 rows], so the
// 16 rows a decoding half-warp writes and the 8 rows an MMA quad-row group
// reads are consecutive float4 (no bank conflicts).
__device__ __forceinline__ void q4k_decode_scales(const uint8_t* blk, float4* out) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    const uint32_t sc_lo4 = s0 & 0x3F3F3F3Fu, m_lo4 = s1 & 0x3F3F3F3Fu;
    const uint32_t sc_hi4 = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t m_hi4 = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    const float d24 = d * 16777216.f, d20 = d * 1048576.f;
    // byte -> float on the FP32 pipe: 0x4B0000bb is 2^23 + bb exactly
    auto byte_f = [](uint32_t w, uint32_t sel) {
        return __uint_as_float(__byte_perm(w, 0x4B000000u, sel)) - 8388608.f;
    };
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t scw = p < 2 ? sc_lo4 : sc_hi4, mw = p < 2 ? m_lo4 : m_hi4;
        const uint32_t b = 2 * (p & 1);  // bytes b, b+1 of the word: sub-blocks 2p, 2p+1
        out[16 * p] = make_float4(d24 * byte_f(scw, 0x7440u | b), d20 * byte_f(scw, 0x7440u | (b + 1)),
                             dmin * byte_f(mw, 0x7440u | b), dmin * byte_f(mw, 0x7440u | (b + 1)));
    }
}

// Q4_K: one pair p (64 elements) of one block for rows g, g+8 of the unit.
// Returns (sum A*(D_hi+D_lo) row g, same row g+8, sum dmin*m*X row g, row g+8).
__device__ __forceinline__ float4 q4_pair(const uint8_t* blk_g, int row8, const float4* tab_g,
                                          const uint2* xe, const float* xs, int p, int c, int lane, int lanes,
                                          bool has_tok) {
    const uint8_t* rq = blk_g + 16 + 32 * p + 4 * c;
    const uint32_t vg0 = *reinterpret_cast<const uint32_t*>(rq);
    const uint32_t vg1 = *reinterpret_cast<const uint32_t*>(rq + 16);
    const uint32_t vh0 = *reinterpret_cast<const uint32_t*>(rq + row8);
    const uint32_t vh1 = *reinterpret_cast<const uint32_t*>(rq + row8 + 16);
    const uint2 z = make_uint2(0u, 0u);
    const bool act = lane < lanes;
    const uint2* xp = xe + p * 4 * lanes;
    const uint2 bl0 = act ? xp[0 * lanes] : z, bh0 = act ? xp[1 * lanes] : z;
    const uint2 bl1 = act ? xp[2 * lanes] : z, bh1 = act ? xp[3 * lanes] : z;
    const float4 sg = tab_g[16 * p], sg8 = tab_g[16 * p + 8];
    const float xlo = has_tok ? xs[2 * p] : 0.f, xhi = has_tok ? xs[2 * p + 1] : 0.f;
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t vg0s = vg0 >> 8, vg1s = vg1 >> 8, vh0s = vh0 >> 8, vh1s = vh1 >> 8;
    float dlo[4], dhi[4];
    mma_f16(dlo, vg0 & 0x000F000Fu, vh0 & 0x000F000Fu, vg0s & 0x000F000Fu, vh0s & 0x000F000Fu, bl0.x, bl0.y, zero4);
    mma_f16(dhi, vg0 & 0x00F000F0u, vh0 & 0x00F000F0u, vg0s & 0x00F000F0u, vh0s & 0x00F000F0u, bh0.x, bh0.y, zero4);
    mma_f16(dlo, vg1 & 0x000F000Fu, vh1 & 0x000F000Fu, vg1s & 0x000F000Fu, vh1s & 0x000F000Fu, bl1.x, bl1.y, dlo);
    mma_f16(dhi, vg1 & 0x00F000F0u, vh1 & 0x00F000F0u, vg1s & 0x00F000F0u, vh1s & 0x00F000F0u, bh1.x, bh1.y, dhi);
    return make_float4(sg.x * (dlo[0] + dlo[1]) + sg.y * (dhi[0] + dhi[1]),
                       sg8.x * (dlo[2] + dlo[3]) + sg8.y * (dhi[2] + dhi[3]), sg.z * xlo + sg.w * xhi,
                       sg8.z * xlo + sg8.w * xhi);
}

template <int NT>
__device__ __forceinline__ void item_q6_k(const uint8_t* blk, int c, const float4 (&xr)[NT][8], const float (&xq)[NT][4],
                                          float (&acc)[NT]) {
    const int h = c >> 2, l0 = 8 * (c & 3);
    const uint8_t* ql = blk + 64 * h + l0;
    const uint8_t* qh = blk + 128 + 32 * h + l0;
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + (l0 >> 4));
    const float d = f16_bits_to_f32(lds_u16(blk + 208));
    float a[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) a[t] = 128.f * d * static_cast<float>(sc[2 * t]);
    float2 s[4][NT];
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int n = 0; n < NT; ++n) s[t][n] = make_float2(0.f, 0.f);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t qa = lds_u32_any(ql + 4 * half), qb = lds_u32_any(ql + 32 + 4 * half);
        const uint32_t hh = lds_u32_any(qh + 4 * half);
        uint32_t t4[4];
        t4[0] = (qa & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u) | 0x80808080u;
        t4[1] = (qb & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u) | 0x80808080u;
        t4[2] = ((qa >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u) | 0x80808080u;
        t4[3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u) | 0x80808080u;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 u01 = make_float2(unit_q<0>(t4[t]), unit_q<1>(t4[t]));
            const float2 u23 = make_float2(unit_q<2>(t4[t]), unit_q<3>(t4[t]));
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const float4 xv = xr[n][2 * t + half];
                s[t][n] = __ffma2_rn(u01, make_float2(xv.x, xv.y), s[t][n]);
                s[t][n] = __ffma2_rn(u23, make_float2(xv.z, xv.w), s[t][n]);
            }
        }
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        float r = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            // sum d sc (q6 - 32) x = a (S - X) - 32/128 a X = a (S - (5/4) X)
            r += a[t] * ((s[t][n].x + s[t][n].y) - 1.25f * xq[n][t]);
        }
        acc[n] += r;
    }
}

template <int NT>
__device__ __forceinline__ void item_q8_0(const uint8_t* blk, const float4 (&xr)[NT][8], float (&acc)[NT]) {
    const float d = f16_bits_to_f32(lds_u16(blk));
    // the 32 quant bytes at blk+2 (2-byte aligned): 9 aligned words, then funnel shifts
    const uint8_t* q = blk + 2;
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(q) & 3);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(q - mis);
    uint32_t wv[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) wv[i] = wp[i];
    float2 s[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n] = make_float2(0.f, 0.f);
#pragma unroll
    for (int f = 0; f < 8; ++f) {
        const uint32_t w = __funnelshift_r(wv[f], wv[f + 1], mis * 8) ^ 0x80808080u;  // u = q + 128
        // 2^23 + u exactly, minus 2^23 + 128 -> q
        const float q0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u)) - 8388736.f;
        const float q1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441u)) - 8388736.f;
        const float q2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442u)) - 8388736.f;
        const float q3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443u)) - 8388736.f;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const float4 xv = xr[n][f];
            s[n] = __ffma2_rn(make_float2(q0, q1), make_float2(xv.x, xv.y), s[n]);
            s[n] = __ffma2_rn(make_float2(q2, q3), make_float2(xv.z, xv.w), s[n]);
        }
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n] += d * (s[n].x + s[n].y);
}

// Walks the (unit, segment) sequence of this CTA.
// Per-op fields the kernel reads in its loops, copied from the parameter
// block into shared memory at entry: the parameter block (with one tensor map
// per op) is larger than the constant cache, and dynamically indexed reads of
// it miss there.
struct OpInfo {
    const uint8_t* w;
    const float* x;
    float* y;
    int64_t w_nb1, x_nb1, y_nb1;
    int32_t type, M, K, N;
    int32_t unit_begin, seg_blocks, nseg, wbox, use_tma;
};

struct OpTable {
    OpInfo op[kMaxOpsPerLaunch];
    int32_t n_ops, total_units;
};

struct SeqCursor {
    int u, sg, oi;
    __device__ __forceinline__ void start(const OpTable& T) {
        u = blockIdx.x;
        sg = 0;
        oi = 0;
        while (oi + 1 < T.n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
    }
    __device__ __forceinline__ bool done(const OpTable& T) const { return u >= T.total_units; }
    __device__ __forceinline__ void next(const OpTable& T) {
        if (++sg >= T.op[oi].nseg) {
            sg = 0;
            u += gridDim.x;
            while (oi + 1 < T.n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
        }
    }
};

// Builds the activation image of `op` in shared memory (all consumer threads;
// one L2 round trip per vector). `wred` holds kCW floats.
__device__ __forceinline__ void stage_activations(const OpInfo& op, uint8_t* xsm, float* wred, int ct, int lane, int cw) {
    const int K = op.K, N = op.N, per4 = K / 4;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(op.x);
    if (op.type == kTypeQ4_K) {
        const int lanes = 8 * N;
        uint2* xB = reinterpret_cast<uint2*>(xsm);
        float* Xs = reinterpret_cast<float*>(xsm + img_xb_bytes(K, N));
        float* inv = reinterpret_cast<float*>(xsm + img_bytes(kTypeQ4_K, K, N) - 16);
        constexpr int kB = 4;  // float4 loads in flight per thread
        for (int t = 0; t < N; ++t) {
            const float4* xv = reinterpret_cast<const float4*>(xb + t * op.x_nb1);
            // pass 1: max|x| (loads from L2, batched)
            float mx = 0.f;
            for (int i0 = 0; i0 < kXF4 && i0 * kCW * 32 < per4; i0 += kB) {
                float4 v[kB];
#pragma unroll
                for (int i = 0; i < kB; ++i) {
                    const int f = (i0 + i) * kCW * 32 + ct;
                    v[i] = f < per4 ? __ldg(xv + f) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < kB; ++i)
                    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) wred[cw] = mx;
            consumers_sync();
            float m = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) m = fmaxf(m, wred[w]);
            const float sc = limb_scale(m);
            // pass 2 (L1-resident reload): limbs in B-fragment order and sub-block sums
            for (int i0 = 0; i0 < kXF4 && i0 * kCW * 32 < per4; i0 += kB) {
              float4 v[kB];
#pragma unroll
              for (int i = 0; i < kB; ++i) {
                  const int f = (i0 + i) * kCW * 32 + ct;
                  v[i] = f < per4 ? __ldg(xv + f) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int ii = 0; ii < kB; ++ii) {
                const int f = (i0 + ii) * kCW * 32 + ct;
                const int i = ii;
                if (f < per4) {  // warp-uniform: per4 is a multiple of 64
                    const int k = 4 * f;
                    const int b = k >> 8, r = k & 255, p = r >> 6, h = (r >> 5) & 1, jj = (r >> 4) & 1;
                    const int cp = (r >> 2) & 3;
                    const int e = ((b * 4 + p) * 2 + jj) * 2 + h;
                    __half h0, l0, h1, l1, h2, l2, h3, l3;
                    limbs(v[i].x * sc, h0, l0);
                    limbs(v[i].y * sc, h1, l1);
                    limbs(v[i].z * sc, h2, l2);
                    limbs(v[i].w * sc, h3, l3);
                    // b0 = (k 2c, 2c+1) <- elements (4c, 4c+2); b1 = (2c+8, 2c+9) <- (4c+1, 4c+3)
                    xB[e * lanes + 4 * (2 * t) + cp] = make_uint2(pack_h2(h0, h2), pack_h2(h1, h3));
                    xB[e * lanes + 4 * (2 * t + 1) + cp] = make_uint2(pack_h2(l0, l2), pack_h2(l1, l3));
                    float a = (v[i].x + v[i].y) + (v[i].z + v[i].w);
                    a += __shfl_xor_sync(0xffffffffu, a, 1);
                    a += __shfl_xor_sync(0xffffffffu, a, 2);
                    a += __shfl_xor_sync(0xffffffffu, a, 4);
                    if ((ct & 7) == 0) Xs[t * (K / 32) + (k >> 5)] = a;
                }
              }
            }
            if (ct == 0) inv[t] = 1.f / sc;
            consumers_sync();  // wred is reused by the next vector
        }
    } else {
        float4* xs4 = reinterpret_cast<float4*>(xsm);
        constexpr int kB = 8;  // float4 loads in flight per thread
        for (int t = 0; t < N; ++t) {
            const float* xf = reinterpret_cast<const float*>(xb + t * op.x_nb1);
            for (int i0 = 0; i0 < kXF4 && i0 * kCW * 32 < per4; i0 += kB) {
                float4 v[kB];
#pragma unroll
                for (int i = 0; i < kB; ++i) {
                    const int idx = (i0 + i) * kCW * 32 + ct;
                    if (idx < per4) {
                        const int g = idx >> 6, f = (idx >> 3) & 7, c = idx & 7;
                        v[i] = __ldg(reinterpret_cast<const float4*>(xf + g * 256 + chunk_elem(op.type, c, f)));
                    }
                }
#pragma unroll
                for (int i = 0; i < kB; ++i) {
                    const int idx = (i0 + i) * kCW * 32 + ct;
                    if (idx < per4) xs4[t * per4 + idx] = v[i];
                }
            }
        }
        consumers_sync();
    }
}

template <int NT>
__global__ void __maxnreg__(112) stream_gemv_kernel(const __grid_constant__ SList L) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = L.stages;
    const int SB = L.stage_bytes;
    const int TB = L.tab_blocks;                                      // table blocks per stage
    uint8_t* stages = smem;
    float4* tabs = reinterpret_cast<float4*>(smem + S * SB);           // [S][TB][4][16]
    uint8_t* xsm = reinterpret_cast<uint8_t*>(tabs) + S * kRows * TB * 64;
    float* ubuf = reinterpret_cast<float*>(xsm + L.x_bytes);          // [kUnitSlots][kCW][16][NT]
    int* ucnt = reinterpret_cast<int*>(ubuf + kUnitSlots * kCW * kRows * NT);
    float* wred = reinterpret_cast<float*>(ucnt + kUnitSlots);        // [kCW]
    uint64_t* full = reinterpret_cast<uint64_t*>(wred + kCW);
    uint64_t* empty = full + kMaxStages;
    uint64_t* ready = empty + kMaxStages;
    volatile int* poisoned = reinterpret_cast<volatile int*>(ready + kMaxStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kUnitSlots; i += kThreads) ucnt[i] = 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
            mbar_init(&ready[s], 1);
        }
        *poisoned = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __shared__ OpTable T;
    if (threadIdx.x < L.n_ops) {
        const SOp& o = L.op[threadIdx.x];
        OpInfo& d = T.op[threadIdx.x];
        d.w = o.w;
        d.x = o.x;
        d.y = o.y;
        d.w_nb1 = o.w_nb1;
        d.x_nb1 = o.x_nb1;
        d.y_nb1 = o.y_nb1;
        d.type = o.type;
        d.M = o.M;
        d.K = o.K;
        d.N = o.N;
        d.unit_begin = o.unit_begin;
        d.seg_blocks = o.seg_blocks;
        d.nseg = o.nseg;
        d.wbox = o.wbox;
        d.use_tma = o.use_tma;
        if (o.use_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&o.tmap) : "memory");
    }
    if (threadIdx.x == 0) {
        T.n_ops = L.n_ops;
        T.total_units = L.total_units;
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ---------------- copy warp: waits only for released slots ----------------
        const uint64_t policy = evict_first_policy();
        SeqCursor ci;
        ci.start(T);
        for (uint32_t issued = 0; !ci.done(T); ++issued, ci.next(T)) {
            const int s = issued % S;
            int ok = 0;
            if (lane == 0) ok = mbar_wait(&empty[s], ((issued / S) & 1) ^ 1, 1u, poisoned);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            {
                const OpInfo& op = T.op[ci.oi];
                const int bb = block_bytes_of(op.type);
                const int r0 = (ci.u - op.unit_begin) * kRows;
                const int b0 = ci.sg * op.seg_blocks;
                uint8_t* dst = stages + s * SB;
                if (op.use_tma) {
                    // one box: 16 rows x wbox bytes from the 16-byte-aligned column at
                    // or below the segment start (rows past M and columns past the row
                    // end read as zeros)
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(kRows * op.wbox));
                        tma_2d_g2s(dst, &L.op[ci.oi].tmap, ((b0 * bb) & ~15) / 8, r0, &full[s], policy);
                    }
                } else {
                    // one bulk copy per row: the row's segment rounded out to 16 bytes
                    const int nblocks = op.K / block_elems_of(op.type);
                    const int nrows = min(kRows, op.M - r0);
                    const bool active = lane < nrows;
                    const int nbytes = min(op.seg_blocks, nblocks - b0) * bb;
                    const uintptr_t g = reinterpret_cast<uintptr_t>(
                        op.w + static_cast<int64_t>(r0 + (active ? lane : 0)) * op.w_nb1 + b0 * bb);
                    const uintptr_t ga = g & ~uintptr_t(15);
                    const uint32_t bytes = active ? static_cast<uint32_t>(((g + nbytes + 15) & ~uintptr_t(15)) - ga) : 0u;
                    const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
                    __syncwarp();
                    if (active) bulk_g2s(dst + lane * op.wbox, reinterpret_cast<const void*>(ga), bytes, &full[s], policy);
                }
            }
        }
        return;
    }
    if (warp == 1) {
        // ---------------- hand-off warp: waits for landed stages, decodes Q4_K scales ----------------
        SeqCursor cd;
        cd.start(T);
        for (uint32_t decoded = 0; !cd.done(T); ++decoded, cd.next(T)) {
            const int s = decoded % S;
            int ok = 0;
            if (lane == 0) ok = mbar_wait(&full[s], (decoded / S) & 1, 1u, poisoned);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const OpInfo& op = T.op[cd.oi];
            if (op.type == kTypeQ4_K) {
                const int nb = min(op.seg_blocks, op.K / 256 - cd.sg * op.seg_blocks);
                const uint8_t* stage = stages + s * SB;
                float4* tab = tabs + s * kRows * TB * 4;
                for (int e = lane; e < kRows * nb; e += 32) {
                    const int r = e & 15, bl = e >> 4;
                    q4k_decode_scales(stage + r * op.wbox + bl * 144, tab + bl * 64 + r);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[s]);
        }
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ct = threadIdx.x - 64;  // 0..255
    const int cw = warp - 2;          // 0..7
    uint32_t seq = 0;                 // stage sequence number
    uint32_t item_base = 0;           // items of the CTA's sequence before the current segment
    int staged = -1, uslot = 0;
    SeqCursor cur;
    cur.start(T);
    while (!cur.done(T)) {
        const int oi = cur.oi;
        const OpInfo& op = T.op[oi];
        const int N = op.N, K = op.K;
        // ---- activation image (re)built when the op's x or layout changes ----
        if (staged < 0 || T.op[staged].x != op.x || T.op[staged].K != K || T.op[staged].N != N ||
            T.op[staged].x_nb1 != op.x_nb1 || (T.op[staged].type == kTypeQ4_K) != (op.type == kTypeQ4_K) ||
            (op.type != kTypeQ4_K && T.op[staged].type != op.type)) {
            consumers_sync();  // nobody still reads the previous image
            stage_activations(op, xsm, wred, ct, lane, cw);
            staged = oi;
        }
        const int bb = block_bytes_of(op.type);
        const int nblocks = K / block_elems_of(op.type);
        const int r0 = (cur.u - op.unit_begin) * kRows;
        // this warp's partial sums of the unit: every warp writes all 16 rows
        float* ub = ubuf + (uslot * kCW + cw) * kRows * NT;

        if (op.type == kTypeQ4_K) {
            // ================= Q4_K, tensor cores =================
            const int g = lane >> 2, c = lane & 3;
            const int lanes = 8 * N;
            const bool has_tok = c < N;
            const uint2* xB = reinterpret_cast<const uint2*>(xsm);
            const float* Xs = reinterpret_cast<const float*>(xsm + img_xb_bytes(K, N)) + (has_tok ? c : 0) * (K / 32);
            float accm_g = 0.f, accm_g8 = 0.f, accn_g = 0.f, accn_g8 = 0.f;
            for (int sg = 0; sg < op.nseg; ++sg, ++seq) {
                const int s = seq % S;
                mbar_wait(&ready[s], (seq / S) & 1, 2u, poisoned);
                const int b0 = sg * op.seg_blocks;
                const int nb = min(op.seg_blocks, nblocks - b0);
                const uint8_t* stage = stages + s * SB;
                const float4* tab = tabs + s * kRows * TB * 4;
                const int row8 = 8 * op.wbox;
                for (int i = (cw - static_cast<int>(item_base % kCW) + kCW) % kCW; i < nb; i += kCW) {
                    const int bg = b0 + i;
                    const uint8_t* blk_g = stage + g * op.wbox + i * 144;
                    const float4* tab_g = tab + i * 64 + g;
                    const uint2* xe = xB + (bg * 16) * lanes + (lane < lanes ? lane : 0);
                    const float* xs = Xs + bg * 8;
                    const float4 r0v = q4_pair(blk_g, row8, tab_g, xe, xs, 0, c, lane, lanes, has_tok);
                    const float4 r1v = q4_pair(blk_g, row8, tab_g, xe, xs, 1, c, lane, lanes, has_tok);
                    const float4 r2v = q4_pair(blk_g, row8, tab_g, xe, xs, 2, c, lane, lanes, has_tok);
                    const float4 r3v = q4_pair(blk_g, row8, tab_g, xe, xs, 3, c, lane, lanes, has_tok);
                    accm_g += (r0v.x + r1v.x) + (r2v.x + r3v.x);
                    accm_g8 += (r0v.y + r1v.y) + (r2v.y + r3v.y);
                    accn_g += (r0v.z + r1v.z) + (r2v.z + r3v.z);
                    accn_g8 += (r0v.w + r1v.w) + (r2v.w + r3v.w);
                }
                item_base += nb;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (has_tok) {
                const float inv = reinterpret_cast<const float*>(xsm + img_bytes(kTypeQ4_K, K, N) - 16)[c];
                ub[g * NT + c] = accm_g * inv - accn_g;
                ub[(g + 8) * NT + c] = accm_g8 * inv - accn_g8;
            }
        } else {
            // ================= Q6_K / Q8_0, CUDA cores =================
            const int j = lane >> 3, c = lane & 7;
            const int K256 = K / 256;
            const float4* xs4 = reinterpret_cast<const float4*>(xsm);
            const uint32_t wlo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0) * op.w_nb1));
            const uint32_t nb1lo = static_cast<uint32_t>(op.w_nb1);
            const bool q8 = op.type == kTypeQ8_0;
            float acc[4][NT];
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int n = 0; n < NT; ++n) acc[q][n] = 0.f;
            for (int sg = 0; sg < op.nseg; ++sg, ++seq) {
                const int s = seq % S;
                mbar_wait(&ready[s], (seq / S) & 1, 2u, poisoned);
                const int b0 = sg * op.seg_blocks;
                const int nb = min(op.seg_blocks, nblocks - b0);
                const uint8_t* stage = stages + s * SB;
                const uint32_t glo = wlo + static_cast<uint32_t>(b0 * bb);
                const uint8_t* base[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int r = 4 * q + j;
                    // each row's copy window starts at its segment start rounded down to 16 bytes
                    base[q] = stage + r * op.wbox + ((glo + static_cast<uint32_t>(r) * nb1lo) & 15u);
                }
                const int gpb = q8 ? 8 : 1;
                const int ngroups = (nb + gpb - 1) / gpb;
                for (int gi = (cw - static_cast<int>(item_base % kCW) + kCW) % kCW; gi < ngroups; gi += kCW) {
                    const int gg = b0 / gpb + gi;  // 256-element group index
                    float4 xr[NT][8];
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const int nn = n < N ? n : 0;
#pragma unroll
                        for (int f = 0; f < 8; ++f) xr[n][f] = xs4[(nn * K256 + gg) * 64 + f * 8 + c];
                    }
                    if (q8) {
                        const int blk = gg * 8 + c;
                        if (blk < b0 + nb) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) item_q8_0<NT>(base[q] + (blk - b0) * 34, xr, acc[q]);
                        }
                    } else {
                        float xq[NT][4];
#pragma unroll
                        for (int n = 0; n < NT; ++n)
#pragma unroll
                            for (int t = 0; t < 4; ++t)
                                xq[n][t] = (xr[n][2 * t].x + xr[n][2 * t].y) + (xr[n][2 * t].z + xr[n][2 * t].w) +
                                           (xr[n][2 * t + 1].x + xr[n][2 * t + 1].y) +
                                           (xr[n][2 * t + 1].z + xr[n][2 * t + 1].w);
#pragma unroll
                        for (int q = 0; q < 4; ++q) item_q6_k<NT>(base[q] + (gg - b0) * 210, c, xr, xq, acc[q]);
                    }
                }
                item_base += ngroups;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    float v = acc[q][n];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    if (c == 0 && n < N) ub[(4 * q + j) * NT + n] = v;
                }
        }
        // ---- unit hand-off: the last of the 8 warps sums the partials and writes the unit ----
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&ucnt[uslot], 1) == kCW - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < kRows * N) {
                // fixed summation order over the warps: results are deterministic
                const int r = lane / N, n = lane % N;
                const volatile float* vb = ubuf + uslot * kCW * kRows * NT + r * NT + n;
                float v = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < kCW; ++w2) v += vb[w2 * kRows * NT];
                if (r0 + r < op.M)
                    *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(op.y) + n * op.y_nb1 + 4LL * (r0 + r)) = v;
            }
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                *reinterpret_cast<volatile int*>(&ucnt[uslot]) = 0;
            }
        }
        uslot = uslot + 1 == kUnitSlots ? 0 : uslot + 1;
        // advance to the next unit (the segment loop above consumed all of this unit's stages)
        cur.sg = op.nseg - 1;
        cur.next(T);
    }
}

size_t smem_bytes(int stages, int stage_bytes, int tab_blocks, int x_bytes, int nt) {
    return static_cast<size_t>(stages) * (static_cast<size_t>(stage_bytes) + kRows * tab_blocks * 64) +
           static_cast<size_t>(x_bytes) + 4ull * kUnitSlots * kCW * kRows * nt + 4ull * kUnitSlots + 4ull * kCW +
           8ull * (3 * kMaxStages) + 16;
}

typedef CUresult (*TensorMapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

TensorMapEncodeFn tensor_map_encoder() {
    static TensorMapEncodeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        cudaGetLastError();
        return reinterpret_cast<TensorMapEncodeFn>(p);
    }();
    return fn;
}

// Weights as a 2D tensor of uint64 elements, [M rows][row bytes / 8] with row
// stride w_nb1, boxes of 16 rows x wbox bytes; false if the layout does not
// allow it (row stride or base not 16-byte aligned, row bytes not a multiple
// of 8), in which case rows are copied one by one.
bool encode_weight_map(SOp& s, int row_bytes) {
    const TensorMapEncodeFn enc = tensor_map_encoder();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(s.w) | static_cast<uintptr_t>(s.w_nb1)) & 15) return false;
    if (row_bytes % 8 || s.wbox % 16 || s.wbox / 8 > 256) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 8), static_cast<cuuint64_t>(s.M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(s.w_nb1)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(s.wbox / 8), static_cast<cuuint32_t>(kRows)};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = enc(&s.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(s.w), dims, strides, box,
                           elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

// Whether the streaming kernel can run this op list; else the caller uses
// the general kernel.
bool stream_supported(const MulMatOp* ops, int n_ops) {
    for (int i = 0; i < n_ops; ++i) {
        const MulMatOp& o = ops[i];
        if (o.ne2 != 1 || o.ne3 != 1) return false;
        if (o.N < 1 || o.N > kMaxNT) return false;
        if (o.K % 256 != 0) return false;  // whole 256-element groups (Q8_0 too)
        if (o.K > kXF4 * kCW * 32 * 4) return false;
        if (o.type == kTypeQ4_K && ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15))
            return false;  // 16-byte header loads from shared memory
        if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;
    }
    return true;
}

int launch_stream(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms) {
    SList L{};
    L.n_ops = n_ops;
    int units = 0, max_n = 1, x_bytes = 0, tab_blocks = 0, wmax = 0;
    for (int i = 0; i < n_ops; ++i) {
        const MulMatOp& o = ops[i];
        SOp& s = L.op[i];
        s.w = o.w;
        s.x = o.x;
        s.y = o.y;
        s.w_nb1 = o.w_nb1;
        s.x_nb1 = o.x_nb1;
        s.y_nb1 = o.y_nb1;
        s.type = o.type;
        s.M = o.M;
        s.K = o.K;
        s.N = o.N;
        s.unit_begin = units;
        const int nblocks = o.K / block_elems(o.type);
        const int cap = seg_cap(o.type);
        const int nseg = (nblocks + cap - 1) / cap;
        int seg = (nblocks + nseg - 1) / nseg;
        if (o.type == kTypeQ8_0) seg = (seg + 7) / 8 * 8;
        s.seg_blocks = seg;
        s.nseg = (nblocks + seg - 1) / seg;
        // stage row width: the segment plus room for the 16-byte window rounding,
        // made == 16 mod 32 so the 8 rows a warp reads hit 8 different bank groups
        const int bb = block_bytes(o.type);
        int wbox = o.type == kTypeQ4_K ? seg * bb : (seg * bb + 30 + 15) / 16 * 16;
        if (wbox % 32 == 0) wbox += 16;
        s.wbox = wbox;
        s.use_tma = encode_weight_map(s, nblocks * bb) ? 1 : 0;
        if (o.type == kTypeQ4_K) tab_blocks = seg > tab_blocks ? seg : tab_blocks;
        wmax = wbox > wmax ? wbox : wmax;
        units += (o.M + kRows - 1) / kRows;
        max_n = o.N > max_n ? o.N : max_n;
        const int xb = (img_bytes(o.type, o.K, o.N) + 15) / 16 * 16;
        x_bytes = xb > x_bytes ? xb : x_bytes;
    }
    L.total_units = units;
    L.x_bytes = x_bytes;
    L.stage_bytes = kRows * wmax;
    L.tab_blocks = tab_blocks;
    const int nt = max_n <= 1 ? 1 : 2;
    const size_t fixed = smem_bytes(0, L.stage_bytes, tab_blocks, x_bytes, nt);
    const size_t per_stage = smem_bytes(1, L.stage_bytes, tab_blocks, x_bytes, nt) - fixed;
    int stages = fixed >= static_cast<size_t>(kSmemBudget)
                     ? 0
                     : static_cast<int>((static_cast<size_t>(kSmemBudget) - fixed) / per_stage);
    stages = stages > kMaxStages ? kMaxStages : stages;
    if (stages < 2) stages = 2;
    L.stages = stages;
    const size_t smem = smem_bytes(stages, L.stage_bytes, tab_blocks, x_bytes, nt);
    if (smem > 227 * 1024) return -static_cast<int>(cudaErrorInvalidValue);
    // CTAs per SM: two by default (~140 KB of weights in flight per SM, and a
    // finished CTA's slot goes to the next launch early); one via the
    // environment for experiments.
    static const int ctas_per_sm = [] {
        const char* e = getenv("WLLM_STREAM_CTAS_PER_SM");
        const int v = e ? atoi(e) : 1;
        return v == 2 ? 2 : 1;
    }();
    const int cap = ctas_per_sm * num_sms;
    const int grid = units < cap ? units : cap;

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // raise the kernel's dynamic shared-memory limit to this launch's need
    // (once per size increase; the attribute call is not a stream operation)
    static size_t configured[2] = {0, 0};
    const int ti = nt - 1;
    cudaError_t e;
    if (configured[ti] < smem) {
        e = ti == 0 ? cudaFuncSetAttribute(stream_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem))
                    : cudaFuncSetAttribute(stream_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
        if (e != cudaSuccess) return -static_cast<int>(e);
        configured[ti] = smem;
    }
    e = ti == 0 ? cudaLaunchKernelEx(&cfg, stream_gemv_kernel<1>, L) : cudaLaunchKernelEx(&cfg, stream_gemv_kernel<2>, L);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -static_cast<int>(e);
}

unsigned read_and_clear_stream_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_stream_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_stream_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace wllm
