// Small-batch quantized MUL_MAT on tcgen05 tensor cores for Q4_K, Q5_K, Q6_K,
// Q8_0 and IQ4_XS weights (several sequences decoding together: N up to 64
// vectors), exact to about 2^-22 of every activation element, like the
// integer decode kernels.
//
//   y[m + M n] = sum_k W[m, k] x[k + K n]   (ggml MUL_MAT, matmul.ts:10-17)
//
// Per 256-element block b of row m, W = d sc_s q - dmin m_s (sub-block s of
// 32 elements), so
//   y[m, n] = sum_b d_mb (sum_k A[m, k] x[k, n]) - dmin_mb (sum_s m_ms X[s, n])
// with A = sc_s q (Q4_K at most 63 x 15, Q5_K 63 x 31: integers exact in f16)
// and X[s, n] the sum of x over sub-block s. Both inner sums are f16 MMAs
// with f32 accumulators in tensor memory, read back once per block and scaled
// there by the block's d and dmin in f32:
//  - activations: per vector and 256-element block a power-of-two scale 2^e
//    (the block's maximum lands in [2^14, 2^15)) and two f16 parts,
//    hi = f16(x 2^-e), lo = f16(x 2^-e - hi), about 22 bits of each element
//    whatever its neighbours (an outlier channel costs nothing); hi and lo are
//    stacked along N, so one MMA of N = 2 nv per K step covers both (the
//    epilogue adds the two columns);
//  - the mins: A_min = (m_0 .. m_7, m_0 .. m_7) (K = 16) against the sub-block
//    sums split the same way (scale 2^(e + 5)), one MMA per block.
// A pre-pass (btc_prep_kernel, one warp per vector and block) writes the
// activation image, the sums image and the scales into workspace.
//
// Q8_0 (ggml's dequantize_row_q8_0: w = d q per 32-element block) has no
// integer form that fits f16: d is an f16 of 11 significant bits, so d q has
// up to 18. It goes in as two exact weight planes, hi = f16(d q) and
// lo = d q - hi (one f16 FMA; the residual has at most 7 significant bits
// on hi's grid, never below f16's smallest subnormal, so it is exact), each
// against the same activations: the accumulator gets sum (hi + lo) x, and the
// epilogue scales it by 2^e only. Chunk by chunk (64 K), both planes of a
// chunk share one half of the A stage. Q6_K (w = d sc (q - 32), int8 sc per
// 16 elements) takes the same two planes for A = sc (q - 32), which reaches
// 4096 in magnitude where f16 holds only even integers (lo is 0 or +-1), with
// d applied per block in the epilogue; IQ4_XS likewise for A = (ls - 32)
// level (up to 4064).
//
// One thread issues a tcgen05.mma in about 50 cycles and waits on an mbarrier
// in about 150, whatever the MMA's N (16 to 128), so at these sizes the issue
// loop, not the tensor pipe, is the limit; two issuing warps run at twice the
// rate. The kernel is laid out for that:
//
// CTA: 128 rows x nv vectors (nv = 16 or 32; N > 32 runs two vector groups as
// grid y, except the two-plane types, whose CTA then takes both groups: its
// issuer i MMAs group i of every block from the one dequantized A stage, into
// two accumulators of its own by block parity). Per block everything moves as
// one unit:
//  - warp 0 (TMA): the 128 rows' raw blocks and the block's scales into a raw
//    slot (4 slots); the block's four hi+lo activation boxes (64 x 2 nv,
//    128-byte swizzle) and its sums box into a B stage (2 or 4 stages);
//  - warps 1 and 2: MMA issuer i (one thread) takes the blocks b = i mod 2,
//    with its own accumulators (main 2 nv columns, mins nv), its own A stage
//    (the block's 4 x 64 f16 per row, 128 TMEM columns) and A_min: per block
//    three waits, the mins MMA and 16 main MMAs, three commits;
//  - warps 3..10: dequantize A = sc q straight into TMEM (tcgen05.st), A_min
//    too, one store wait and one arrival per block;
//  - warps 11..18: the epilogue of each block (tcgen05.ld of its accumulators,
//    y += d s_n main - dmin s'_n mins, with d, dmin and the block's scales s_n,
//    s'_n from the raw slot, which they release).
// Split K as in the prefill GEMM.
//
// Every mbarrier wait is bounded; on timeout the CTA records an error code
// (read by wllm_sync), stops issuing work, drains what it issued and still
// releases its TMEM.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_btc_error = 0;

namespace {

constexpr int kTM = 128;      // rows of W per CTA (TMEM lanes)
constexpr int kMaxNP = 64;    // vectors per launch
constexpr int kMaxNV = 32;    // vectors per vector group
constexpr int kMaxVPC = 64;   // vectors per CTA (two groups in a wide CTA)
constexpr int kChunk = 64;    // K per activation box (one 128-byte swizzle atom of f16)
constexpr int kMaxStB = 4;    // B stages (blocks of activations), at most
constexpr int kMaxRaw = 8;    // raw blocks in flight, at most (8, or 4 where B stages need the room)
constexpr int kDq = 8;        // dequant warps
constexpr int kEp = 8;        // epilogue warps
constexpr int kFirstDq = 3;   // warps: 0 TMA, 1-2 MMA issuers, then dequant, then epilogue
constexpr int kFirstEp = kFirstDq + kDq;
constexpr int kThr = 32 * (kFirstEp + kEp);
constexpr int kACols = 128;   // TMEM columns of one A stage (256 f16 per row, two per column)
// TMEM, issuer i (block parity): the main accumulator at columns W i (2 nv:
// hi then lo), the mins accumulator after it (nv); W (accw) leaves room for the
// epilogue's 16-column loads past the last vector; A_min of issuer i at 2 W +
// 8 i; A stage i at acol0 + 128 i
constexpr int kTmemCols = 512;
constexpr uint32_t kSpin = 1u << 26;
constexpr int kMaxSplits = 16;

struct BtcArgs {
    CUtensorMap wmap;     // weights [M][row bytes / 8] uint64, box (block bytes / 8) x 128
    CUtensorMap xmap;     // activations [groups][hi, lo][nv][K] f16, box 64 x 2 nv, 128-byte swizzle
    CUtensorMap smap;     // sub-block sums [blocks x np][64] f16 (k 0..7 hi, 8..15 lo, rest 0), box 64 x nv
    const float* vscale;  // [block][group][2][nv]: 2^e (activations), 2^(e + 5) (sums)
    float* y;
    int64_t y_nb1;        // bytes between output vectors
    int32_t M, K, N;
    int32_t nv, groups;   // vectors per group, vector groups (grid y, or both in one wide CTA)
    int32_t wide;         // two-plane types above 32 vectors: one CTA, issuer i takes group i of every block
    int32_t nstb, nraw;   // B stages (2 or 4), raw slots (4 or 8)
    int32_t accw, acol0;  // TMEM columns of one issuer's accumulators; first A column
    int32_t splits, kb_split;
    float* partial;       // [tile][split][kMaxVPC][128] (split K)
    unsigned* counters;   // [tile] (split K, zero at launch)
};

// Bytes per row of one 256-element block in a raw slot: Q4_K 144, Q5_K 176,
// Q8_0 272 (8 blocks), Q6_K 240 (the 210-byte block from its start rounded
// down to 16: at most 14 + 210 bytes, a 16-byte multiple), IQ4_XS 144 (the
// 136-byte block at offset 0 or 8).
template <int TYPE>
__host__ __device__ constexpr int blk_bytes() {
    return TYPE == kTypeQ5_K ? 176 : (TYPE == kTypeQ8_0 ? 272 : (TYPE == kTypeQ6_K ? 240 : 144));
}
// Q8_0, Q6_K and IQ4_XS weights go in as two f16 planes (no mins, no sums box).
template <int TYPE>
__host__ __device__ constexpr bool two_planes() {
    return TYPE == kTypeQ8_0 || TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS;
}
// Q6_K and IQ4_XS rows are mapped in bytes: the bytes of one block.
template <int TYPE>
__host__ __device__ constexpr int row_blk_bytes() {
    return TYPE == kTypeQ6_K ? 210 : 136;
}
// The weight box's x coordinate for K block kb: byte-mapped rows from the
// block's start rounded down to 16, the others in uint64 words.
template <int TYPE>
__device__ __forceinline__ int raw_box_x(int kb) {
    if constexpr (TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS) return (kb * row_blk_bytes<TYPE>()) & ~15;
    return kb * (blk_bytes<TYPE>() / 8);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
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
// Bounded wait; a timeout poisons the CTA (every later wait returns at once).
// SLEEP_NS > 0 backs off between polls: warps whose waits are long and off the
// critical path (the copy warp, the epilogue) then leave the issue slots to
// the dequantizing warps on the same scheduler.
template <int SLEEP_NS = 0>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned) {
    for (uint32_t i = 0; i < kSpin; ++i) {
        if (mbar_try(bar, parity)) return true;
        if (SLEEP_NS > 0) __nanosleep(SLEEP_NS);
        if ((i & 255u) == 255u && *poisoned) return false;
    }
    *poisoned = 1;
    atomicOr(&g_btc_error, code);
    return false;
}
// Bounded wait for a phase whatever the poison flag says (draining what was
// issued before the CTA exits); false on time-out.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpin; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Adds to the barrier's expected transaction bytes without arriving.
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1024
// bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}
// D (TMEM) (+)= A (TMEM, K-major, f16) * B (shared memory, f16), f32 accumulators.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        :
        : "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 8 consecutive 32-bit TMEM columns of this warp's 32 lanes. No memory
// clobber: it reads registers only, so the compiler may schedule shared-memory
// loads around it (volatile asm statements keep their order among themselves,
// and tcgen05.wait::st, which does clobber memory, orders it before the
// barrier arrivals).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]));
}
// 16 consecutive f32 columns of this warp's 32 TMEM lanes at three column
// addresses, with one wait for all of them inside the same statement (so no
// use of the registers can be scheduled before the wait).
#define WLLM_R16(o) "=r"(r[o]), "=r"(r[o + 1]), "=r"(r[o + 2]), "=r"(r[o + 3]), "=r"(r[o + 4]), "=r"(r[o + 5]), \
    "=r"(r[o + 6]), "=r"(r[o + 7]), "=r"(r[o + 8]), "=r"(r[o + 9]), "=r"(r[o + 10]), "=r"(r[o + 11]), "=r"(r[o + 12]), \
    "=r"(r[o + 13]), "=r"(r[o + 14]), "=r"(r[o + 15])
__device__ __forceinline__ void tmem_ld16x3(uint32_t t0, uint32_t t1, uint32_t t2, float (&v0)[16], float (&v1)[16],
                                            float (&v2)[16]) {
    uint32_t r[48];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%48];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%49];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, [%50];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : WLLM_R16(0), WLLM_R16(16), WLLM_R16(32)
        : "r"(t0), "r"(t1), "r"(t2)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v0[i] = __uint_as_float(r[i]);
        v1[i] = __uint_as_float(r[16 + i]);
        v2[i] = __uint_as_float(r[32 + i]);
    }
}
__device__ __forceinline__ void tmem_ld16x2(uint32_t t0, uint32_t t1, float (&v0)[16], float (&v1)[16]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : WLLM_R16(0), WLLM_R16(16)
        : "r"(t0), "r"(t1)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v0[i] = __uint_as_float(r[i]);
        v1[i] = __uint_as_float(r[16 + i]);
    }
}
#undef WLLM_R16
// 8 f32 columns at each of two column addresses, one wait.
__device__ __forceinline__ void tmem_ld8x2(uint32_t t0, uint32_t t1, float (&v0)[8], float (&v1)[8]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(t0), "r"(t1)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v0[i] = __uint_as_float(r[i]);
        v1[i] = __uint_as_float(r[8 + i]);
    }
}

// Shared-memory layout (from a 1024-byte aligned base): B stages (four hi+lo
// activation boxes, then the sums box unless the type has no mins), raw
// slots, scale slots, barriers.
struct Smem {
    uint32_t box_bytes, s_bytes, b_bytes, raw_bytes, v_bytes, nstb, nraw;
    __host__ __device__ Smem(int nv, int bb, int nstb_, int nraw_, bool sums, bool wide) {
        box_bytes = static_cast<uint32_t>(2 * nv * 128);  // hi + lo rows of one 64-element chunk
        s_bytes = sums ? static_cast<uint32_t>(nv * 128) : 0u;
        b_bytes = (wide ? 8u : 4u) * box_bytes + s_bytes;  // wide: chunk c of group g at box 2c + g
        raw_bytes = static_cast<uint32_t>(kTM * bb);
        v_bytes = static_cast<uint32_t>((wide ? 2 : 1) * 2 * nv * 4);  // the block's 2 nv scales per group
        nstb = static_cast<uint32_t>(nstb_);
        nraw = static_cast<uint32_t>(nraw_);
    }
    __host__ __device__ uint32_t b_off(int s) const { return s * b_bytes; }
    __host__ __device__ uint32_t raw_off(int r) const { return nstb * b_bytes + r * raw_bytes; }
    __host__ __device__ uint32_t v_off(int r) const { return nstb * b_bytes + nraw * raw_bytes + r * v_bytes; }
    __host__ __device__ uint32_t bar_off() const { return nstb * b_bytes + nraw * (raw_bytes + v_bytes); }
    // barriers: b_full, b_free [kMaxStB], raw_full, raw_free [kMaxRaw], a_full,
    // a_free [4] (A stage i, half f at 2 i + f), acc_full, acc_free [4] (issuer
    // i's accumulator, wide: 2 i + block parity); then the TMEM base address
    // word and the poison flag
    static constexpr uint32_t kBars = 2 * kMaxStB + 2 * kMaxRaw + 16;
    __host__ __device__ uint32_t total() const {
        return bar_off() + 8 * kBars + 16 + 1024;  // + alignment slack
    }
};

// Both f16 planes of Q8_0 block J of a row (272 bytes: eight 34-byte blocks,
// an f16 d then 32 int8 quants): hi = f16(d q) and lo = d q - hi, exact
// (ggml's dequantize_row_q8_0, w = d q), elements 16 qq .. 16 qq + 15 in
// hw[qq] / lw[qq], f16 pairs in element order. The quants start a = 34 J + 2
// bytes into the row; they are read as 16-byte words from a rounded down to
// 16 (conflict-free at the 272-byte row stride) and shifted into place.
template <int J>
__device__ __forceinline__ void q8_block_planes(const uint8_t* row, uint32_t (&hw)[2][8], uint32_t (&lw)[2][8]) {
    constexpr int a = 34 * J + 2, w0 = a & ~15, sh = a & 15;  // sh even: 0 .. 14
    uint32_t win[12];
#pragma unroll
    for (int t = 0; t < 3; ++t) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (t < 2 || sh > 0) v = *reinterpret_cast<const uint4*>(row + w0 + 16 * t);
        win[4 * t] = v.x;
        win[4 * t + 1] = v.y;
        win[4 * t + 2] = v.z;
        win[4 * t + 3] = v.w;
    }
    const __half2 d2 = __half2half2(*reinterpret_cast<const __half*>(row + 34 * J));
    const __half2 k1152 = __float2half2_rn(1152.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        constexpr int q4 = sh >> 2;
        const uint32_t w = (sh & 3) ? __funnelshift_r(win[q4 + k], win[q4 + k + 1], 16) : win[q4 + k];
        // f16 1024 + (q + 128) for bytes (0, 1) and (2, 3), minus 1152: q exactly
        const uint32_t u = w ^ 0x80808080u;
        const uint32_t e01 = __byte_perm(u, 0x00006464u, 0x5140u), e23 = __byte_perm(u, 0x00006464u, 0x5342u);
        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1152);
        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1152);
        const __half2 h01 = __hmul2(q01, d2), h23 = __hmul2(q23, d2);
        const __half2 l01 = __hfma2(q01, d2, __hneg2(h01)), l23 = __hfma2(q23, d2, __hneg2(h23));
        hw[k >> 2][2 * (k & 3)] = *reinterpret_cast<const uint32_t*>(&h01);
        hw[k >> 2][2 * (k & 3) + 1] = *reinterpret_cast<const uint32_t*>(&h23);
        lw[k >> 2][2 * (k & 3)] = *reinterpret_cast<const uint32_t*>(&l01);
        lw[k >> 2][2 * (k & 3) + 1] = *reinterpret_cast<const uint32_t*>(&l23);
    }
}
// Block 2 f + H of the row (this warp's block of chunk f).
template <int H>
__device__ __forceinline__ void q8_chunk_planes(const uint8_t* row, int f, uint32_t (&hw)[2][8], uint32_t (&lw)[2][8]) {
    switch (f) {
        case 0: q8_block_planes<H>(row, hw, lw); break;
        case 1: q8_block_planes<2 + H>(row, hw, lw); break;
        case 2: q8_block_planes<4 + H>(row, hw, lw); break;
        default: q8_block_planes<6 + H>(row, hw, lw); break;
    }
}

// 16 bytes at byte O + c of a Q6_K box row (c a multiple of 16, O the block's
// offset, even, known at compile time): from the aligned 16-byte words at c,
// the words from O / 4 on, funnel-shifted by 8 (O % 4) bits.
template <int O>
__device__ __forceinline__ uint4 q6_load16(const uint8_t* row, int c) {
    constexpr int q4 = O >> 2;
    constexpr uint32_t sh = 8u * (O & 3);
    const uint4* a = reinterpret_cast<const uint4*>(row + c);
    const uint4 lo = a[0];
    if constexpr (O == 0) {
        return lo;
    } else {
        const uint4 hi = a[1];
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        if constexpr (sh == 0)
            return make_uint4(w[q4], w[q4 + 1], w[q4 + 2], w[q4 + 3]);
        else
            return make_uint4(__funnelshift_r(w[q4], w[q4 + 1], sh), __funnelshift_r(w[q4 + 1], w[q4 + 2], sh),
                              __funnelshift_r(w[q4 + 2], w[q4 + 3], sh), __funnelshift_r(w[q4 + 3], w[q4 + 4], sh));
    }
}
// This thread's ql and qh bytes of half n of a Q6_K block at offset O.
template <int O>
__device__ __forceinline__ void q6_half_loads(const uint8_t* row, int n, int h, uint4 (&ql)[2], uint4 (&qh)[2]) {
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
        ql[qq] = q6_load16<O>(row, 64 * n + 32 * h + 16 * qq);
        qh[qq] = q6_load16<O>(row, 128 + 32 * n + 16 * qq);
    }
}

// Both f16 planes of chunk f (64 elements) of a Q6_K block, this warp's half
// h (ggml's dequantize_row_q6_K layout): element 64f + 32h + 16qq + l is in
// half n = f / 2 of the block, j = 2 (f % 2) + h: ql byte 64n + 32h + 16qq + l
// (its high nibble when f is odd), qh byte 128 + 32n + 16qq + l shifted by
// 2j, int8 scale 192 + 8n + 2j + qq; w = d sc (q - 32). A = sc (q - 32)
// reaches 4096 in magnitude, one bit past f16's exact integers, so it goes in
// as hi = f16(A) and lo = A - hi (0 or +-1); d is applied per block when the
// accumulator is read. ql and qh serve both chunks of a half: loaded when f
// is even. o: the block's offset in its 240-byte box row (2 kb mod 16, the
// same for every row: one uniform branch to the loads for that offset).
__device__ __forceinline__ void q6_chunk_planes(const uint8_t* row, int f, int h, int o, uint4 (&ql)[2],
                                                uint4 (&qh)[2], uint32_t (&hw)[2][8], uint32_t (&lw)[2][8]) {
    const int n = f >> 1, t = f & 1, j = 2 * t + h;
    if (t == 0) {
        switch (o) {
            case 0: q6_half_loads<0>(row, n, h, ql, qh); break;
            case 2: q6_half_loads<2>(row, n, h, ql, qh); break;
            case 4: q6_half_loads<4>(row, n, h, ql, qh); break;
            case 6: q6_half_loads<6>(row, n, h, ql, qh); break;
            case 8: q6_half_loads<8>(row, n, h, ql, qh); break;
            case 10: q6_half_loads<10>(row, n, h, ql, qh); break;
            case 12: q6_half_loads<12>(row, n, h, ql, qh); break;
            default: q6_half_loads<14>(row, n, h, ql, qh); break;
        }
    }
    const __half2 k1056 = __float2half2_rn(1056.f);
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
        const __half2 sc2 = __half2half2(__int2half_rn(static_cast<int8_t>(row[o + 192 + 8 * n + 2 * j + qq])));
        const uint32_t lq[4] = {ql[qq].x, ql[qq].y, ql[qq].z, ql[qq].w}, hq[4] = {qh[qq].x, qh[qq].y, qh[qq].z, qh[qq].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t qv = ((lq[i] >> (4 * t)) & 0x0F0F0F0Fu) | (((hq[i] >> (2 * j)) & 0x03030303u) << 4);
            // f16 1024 + q (exact, q < 64), minus 1056: q - 32 exactly
            const uint32_t e01 = __byte_perm(qv, 0x00006464u, 0x5140u), e23 = __byte_perm(qv, 0x00006464u, 0x5342u);
            const __half2 v01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1056);
            const __half2 v23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1056);
            const __half2 h01 = __hmul2(v01, sc2), h23 = __hmul2(v23, sc2);
            const __half2 l01 = __hfma2(v01, sc2, __hneg2(h01)), l23 = __hfma2(v23, sc2, __hneg2(h23));
            hw[qq][2 * i] = *reinterpret_cast<const uint32_t*>(&h01);
            hw[qq][2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h23);
            lw[qq][2 * i] = *reinterpret_cast<const uint32_t*>(&l01);
            lw[qq][2 * i + 1] = *reinterpret_cast<const uint32_t*>(&l23);
        }
    }
}

// WIDE (two-plane types above 32 vectors, P.wide set): both vector groups in
// one CTA, a separate instantiation so the others carry none of its code.
// Both f16 planes of chunk f of an IQ4_XS block (136 B: f16 d, u16 scales_h,
// 4 B of 4-bit scales_l, 128 B of level indices), this warp's sub-block
// j = 2f + h: its 16 index bytes at o + 8 + 16j hold elements 0..15 (low
// nibbles) and 16..31 (high); w = d (ls_j - 32) level (dequantize_row_iq4_xs).
// A = (ls_j - 32) level reaches 32 * 127 = 4064, past f16's exact integers,
// so hi = f16(A) and lo = A - hi; d is applied per block in the epilogue. The
// level comes from the 16-entry table as f16 1024 + (level + 128), minus 1152.
// o (0 or 8) is the block's offset in its 144-byte box row, the same for
// every row.
__device__ __forceinline__ void iq4_chunk_planes(const uint8_t* row, int f, int h, int o, uint32_t shb, uint32_t slb,
                                                 uint32_t (&hw)[2][8], uint32_t (&lw)[2][8]) {
    const int j = 2 * f + h;
    const uint4 v = o == 0 ? q6_load16<8>(row, 16 * j) : q6_load16<0>(row, 16 + 16 * j);
    const __half2 s2 = __half2half2(__int2half_rn(iq4xs_scale(shb, slb, j)));
    const __half2 k1152 = __float2half2_rn(1152.f);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint32_t lv[2][4];  // levels of the low (qq = 0) and high nibbles
#pragma unroll
    for (int i = 0; i < 4; ++i) iq4_lut8(wv[i], lv[0][i], lv[1][i]);
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t u = lv[qq][i] ^ 0x80808080u;  // level + 128
            const uint32_t e01 = __byte_perm(u, 0x00006464u, 0x5140u), e23 = __byte_perm(u, 0x00006464u, 0x5342u);
            const __half2 v01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1152);
            const __half2 v23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1152);
            const __half2 h01 = __hmul2(v01, s2), h23 = __hmul2(v23, s2);
            const __half2 l01 = __hfma2(v01, s2, __hneg2(h01)), l23 = __hfma2(v23, s2, __hneg2(h23));
            hw[qq][2 * i] = *reinterpret_cast<const uint32_t*>(&h01);
            hw[qq][2 * i + 1] = *reinterpret_cast<const uint32_t*>(&h23);
            lw[qq][2 * i] = *reinterpret_cast<const uint32_t*>(&l01);
            lw[qq][2 * i + 1] = *reinterpret_cast<const uint32_t*>(&l23);
        }
    }
}

template <int TYPE, bool WIDE>
__global__ void __launch_bounds__(kThr, 1) btc_kernel(const __grid_constant__ BtcArgs P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int BB = blk_bytes<TYPE>();
    constexpr bool TWO = two_planes<TYPE>();
    const int nv = P.nv, nstb = P.nstb, nraw = P.nraw;
    constexpr bool wide = TWO && WIDE;
    const Smem L(nv, BB, nstb, nraw, !TWO, wide);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off());
    uint64_t* b_full = bars;
    uint64_t* b_free = b_full + kMaxStB;
    uint64_t* raw_full = b_free + kMaxStB;
    uint64_t* raw_free = raw_full + kMaxRaw;
    uint64_t* a_full = raw_free + kMaxRaw;
    uint64_t* a_free = a_full + 4;
    uint64_t* acc_full = a_free + 4;
    uint64_t* acc_free = acc_full + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_free + 4);
    volatile int* poisoned = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTM;
    const int grp = blockIdx.y;                // vector group: vectors nv grp ..
    const int kb0 = blockIdx.z * P.kb_split;  // first K block of this split
    const int nblk = min(P.K / 256 - kb0, P.kb_split);
    const int accw = P.accw;
    const uint32_t mincol0 = static_cast<uint32_t>(2 * accw);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxStB; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_free[i], wide ? 2 : 1);  // wide: both issuers read every stage
        }
        for (int r = 0; r < kMaxRaw; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_free[r], kDq + kEp);
        }
        for (int p = 0; p < 4; ++p) {
            mbar_init(&a_full[p], kDq);
            mbar_init(&a_free[p], wide ? 2 : 1);
        }
        for (int p = 0; p < 4; ++p) {
            mbar_init(&acc_full[p], 1);
            mbar_init(&acc_free[p], wide ? kEp / 2 : kEp);  // wide: the four epilogue warps of the group
        }
        *poisoned = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int lgb = nstb == 4 ? 2 : 1;  // log2 of the B stages (2 or 4)
    const int lgr = nraw == 8 ? 3 : (nraw == 4 ? 2 : 1);  // log2 of the raw slots (2, 4 or 8)
    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&P.wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&P.xmap) : "memory");
            if (!TWO) asm volatile("prefetch.tensormap [%0];" ::"l"(&P.smap) : "memory");
            // the weights do not depend on the pre-pass: the first raw slots' boxes
            // go out before the wait for it (their barrier's arrival comes with the
            // scales, after the wait, so no phase can complete early)
            const int pre = min(nblk, nraw);
            for (int b = 0; b < pre; ++b) {
                mbar_expect_tx_only(&raw_full[b], L.raw_bytes);
                tma_2d(smem + L.raw_off(b), &P.wmap, raw_box_x<TYPE>(kb0 + b), m0, &raw_full[b]);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            int armed = 0;   // blocks whose raw slot copies are all issued and armed
            int issued = 0;  // blocks whose B stage copies are issued
            for (int b = 0; b < nblk; ++b) {
                const int r = b & (nraw - 1), s = b & (nstb - 1), kb = kb0 + b;
                if (b >= nraw) {
                    if (!mbar_wait<64>(&raw_free[r], ((b >> lgr) - 1) & 1, 1u, poisoned)) break;
                    mbar_expect_tx(&raw_full[r], L.raw_bytes + L.v_bytes);
                    tma_2d(smem + L.raw_off(r), &P.wmap, raw_box_x<TYPE>(kb), m0, &raw_full[r]);
                } else {
                    mbar_expect_tx(&raw_full[r], L.v_bytes);
                }
                bulk_copy(smem + L.v_off(r), P.vscale + (static_cast<int64_t>(kb) * P.groups + grp) * 2 * nv, L.v_bytes,
                          &raw_full[r]);  // wide: both groups' scales (grp = 0)
                armed = b + 1;
                if (b >= nstb && !mbar_wait<64>(&b_free[s], ((b >> lgb) - 1) & 1, 1u, poisoned)) break;
                uint8_t* dst = smem + L.b_off(s);
                mbar_expect_tx(&b_full[s], L.b_bytes);
                if constexpr (wide) {
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        tma_2d(dst + c * L.box_bytes, &P.xmap, kb * 256 + kChunk * (c >> 1), (c & 1) * 2 * nv, &b_full[s]);
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tma_2d(dst + c * L.box_bytes, &P.xmap, kb * 256 + kChunk * c, grp * 2 * nv, &b_full[s]);
                }
                if (!TWO) tma_2d(dst + 4 * L.box_bytes, &P.smap, 0, kb * P.groups * nv + grp * nv, &b_full[s]);
                issued = b + 1;
            }
            // before the CTA exits, the last copy into every slot and stage has
            // landed (bounded, whatever the poison flag says); a pre-issued slot
            // that was never armed gets its arrival now
            for (int b = armed; b < pre; ++b) mbar_arrive(&raw_full[b]);
            const int raw_issued = max(armed, pre);
            for (int b = max(0, raw_issued - nraw); b < raw_issued; ++b)
                if (!mbar_wait_drain(&raw_full[b & (nraw - 1)], (b >> lgr) & 1)) atomicOr(&g_btc_error, 16u);
            for (int b = max(0, issued - nstb); b < issued; ++b)
                if (!mbar_wait_drain(&b_full[b & (nstb - 1)], (b >> lgb) & 1)) atomicOr(&g_btc_error, 16u);
        }
    } else if (warp < kFirstDq) {
        // ---------------- MMA issuer i: blocks b = i, i + 2, ... ----------------
        const int i = warp - 1;
        if (lane == 0) {
            uint64_t* last_bar = nullptr;  // the last commit (it tracks every MMA before it)
            uint32_t last_par = 0;
            const uint64_t bdesc0 = umma_desc_sw128(smem_u32(smem));  // + (byte offset >> 4)
            const uint32_t dmain = tmem + static_cast<uint32_t>(accw * i), dmin = dmain + static_cast<uint32_t>(2 * nv);
            const uint32_t amin = tmem + mincol0 + static_cast<uint32_t>(8 * i);
            const uint32_t a0 = tmem + static_cast<uint32_t>(P.acol0 + kACols * i);
            // f32 accumulators, f16 A and B (K-major), M = 128; N = 2 nv (hi, lo) or nv (mins)
            const uint32_t idesc_main =
                (1u << 4) | (static_cast<uint32_t>((2 * nv) >> 3) << 17) | (static_cast<uint32_t>(kTM >> 4) << 24);
            const uint32_t idesc_min = (1u << 4) | (static_cast<uint32_t>(nv >> 3) << 17) | (static_cast<uint32_t>(kTM >> 4) << 24);
            if constexpr (TWO) {
              if constexpr (wide) {
                // every block, vector group i, into accumulator 2 i + (b & 1); the
                // block's A stage (b & 1) and B stage are shared with the other
                // issuer, whose commits the barriers also count
                for (int b = 0; b < nblk; ++b) {
                    const int s = b & (nstb - 1), q = b & 1, ai = 2 * i + q;
                    const uint32_t u = static_cast<uint32_t>(b >> 1);  // uses of this accumulator and A stage
                    const uint32_t dw = tmem + static_cast<uint32_t>(accw * ai);
                    if (b >= 2 && !mbar_wait(&acc_free[ai], (u - 1) & 1, 2u, poisoned)) break;
                    if (!mbar_wait(&b_full[s], (b >> lgb) & 1, 2u, poisoned)) break;
                    const uint64_t bd = bdesc0 + (L.b_off(s) >> 4);
                    const uint32_t aq = tmem + static_cast<uint32_t>(P.acol0 + kACols * q);
                    bool all = true;  // every chunk arrived
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const uint32_t use = 2 * u + static_cast<uint32_t>(f >> 1);
                        if (!mbar_wait(&a_full[2 * q + (f & 1)], use & 1, 2u, poisoned)) {
                            all = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t bc = bd + (((2 * f + i) * L.box_bytes) >> 4);
                        const uint32_t ah = aq + static_cast<uint32_t>(64 * (f & 1));
#pragma unroll
                        for (int ks = 0; ks < kChunk / 16; ++ks) {
                            umma_f16_ts(dw, ah + 8 * ks, bc + 2 * ks, idesc_main, (f | ks) ? 1u : 0u);
                            umma_f16_ts(dw, ah + 32 + 8 * ks, bc + 2 * ks, idesc_main, 1u);
                        }
                        umma_commit(&a_free[2 * q + (f & 1)]);
                    }
                    // (after a time-out, the accumulator's barrier, counted once, still
                    // tracks every MMA issued for the drain below)
                    if (all) umma_commit(&b_free[s]);
                    umma_commit(&acc_full[ai]);
                    last_bar = &acc_full[ai];
                    last_par = u & 1;
                    if (!all) break;
                }
              } else {
                // chunk f (64 K) of the block: both planes in half f & 1 of A stage i
                // (hi at columns 0..31, lo at 32..63), use 2 u + f / 2 of that half
                for (int b = i, u = 0; b < nblk; b += 2, ++u) {
                    const int s = b & (nstb - 1);
                    if (u >= 1 && !mbar_wait(&acc_free[i], (u - 1) & 1, 2u, poisoned)) break;
                    if (!mbar_wait(&b_full[s], (b >> lgb) & 1, 2u, poisoned)) break;
                    const uint64_t bd = bdesc0 + (L.b_off(s) >> 4);
                    bool all = true;  // every chunk arrived
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const uint32_t use = static_cast<uint32_t>(2 * u + (f >> 1));
                        if (!mbar_wait(&a_full[2 * i + (f & 1)], use & 1, 2u, poisoned)) {
                            all = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t bc = bd + ((f * L.box_bytes) >> 4);
                        const uint32_t ah = a0 + static_cast<uint32_t>(64 * (f & 1));
#pragma unroll
                        for (int ks = 0; ks < kChunk / 16; ++ks) {
                            umma_f16_ts(dmain, ah + 8 * ks, bc + 2 * ks, idesc_main, (f | ks) ? 1u : 0u);
                            umma_f16_ts(dmain, ah + 32 + 8 * ks, bc + 2 * ks, idesc_main, 1u);
                        }
                        umma_commit(&a_free[2 * i + (f & 1)]);
                        last_bar = &a_free[2 * i + (f & 1)];
                        last_par = use & 1;
                    }
                    if (!all) break;
                    umma_commit(&b_free[s]);
                    umma_commit(&acc_full[i]);
                    last_bar = &acc_full[i];
                    last_par = static_cast<uint32_t>(u & 1);
                }
              }
            } else {
                for (int b = i, u = 0; b < nblk; b += 2, ++u) {  // u: this issuer's block count (its phases)
                    const int s = b & (nstb - 1);
                    if (u >= 1 && !mbar_wait(&acc_free[i], (u - 1) & 1, 2u, poisoned)) break;
                    // the A stage comes in two halves (chunks 0-1, 2-3): the MMAs of the
                    // first overlap the dequantization of the second
                    if (!mbar_wait(&b_full[s], (b >> lgb) & 1, 2u, poisoned) ||
                        !mbar_wait(&a_full[2 * i], u & 1, 2u, poisoned))
                        break;
                    tc_fence_after();
                    const uint64_t bd = bdesc0 + (L.b_off(s) >> 4);
                    bool second = true;  // the second half arrived
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (c == 2) {
                            umma_commit(&a_free[2 * i]);  // the first half is free once these have read it
                            last_bar = &a_free[2 * i];
                            last_par = static_cast<uint32_t>(u & 1);
                            if (!mbar_wait(&a_full[2 * i + 1], u & 1, 2u, poisoned)) {
                                second = false;
                                break;
                            }
                            tc_fence_after();
                            // the mins: A_min (K = 16, written with the second half) against the sums box
                            umma_f16_ts(dmin, amin, bd + ((4 * L.box_bytes) >> 4), idesc_min, 0u);
                        }
                        const uint64_t bc = bd + ((c * L.box_bytes) >> 4);
#pragma unroll
                        for (int ks = 0; ks < kChunk / 16; ++ks)  // K = 16 per MMA: 8 A columns, 32 bytes of B rows
                            umma_f16_ts(dmain, a0 + 32 * c + 8 * ks, bc + 2 * ks, idesc_main, (c | ks) ? 1u : 0u);
                    }
                    if (!second) break;  // the first half's MMAs are tracked by their commit
                    umma_commit(&a_free[2 * i + 1]);  // the second half, A_min and the B stage are read
                    umma_commit(&b_free[s]);
                    umma_commit(&acc_full[i]);
                    last_bar = &acc_full[i];
                    last_par = static_cast<uint32_t>(u & 1);
                }
            }
            // a time-out: the MMAs already issued still write TMEM, which is freed
            // at the end; wait (bounded) for the last commit
            if (*poisoned && last_bar && !mbar_wait_drain(last_bar, last_par)) atomicOr(&g_btc_error, 16u);
        }
        __syncwarp();
    } else if (warp < kFirstEp) {
        // ---------------- dequant: A and A_min of each block ----------------
        const int quarter = warp & 3;                // TMEM lanes this warp may access
        const int h = (warp - kFirstDq) >> 2;        // sub-block 2p + h of chunk p (both halves)
        const int r = 32 * quarter + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
        const uint32_t sel_a = 0x4440u + static_cast<uint32_t>(h);      // byte h, zero-extended
        const uint32_t sel_b = 0x4440u + 2u + static_cast<uint32_t>(h);  // byte 2 + h
        const __half2 k1024 = __float2half2_rn(1024.f), km1024 = __float2half2_rn(-1024.f);
        if constexpr (TWO) {
            // two planes per chunk f (64 K): Q8_0's blocks 2f and 2f + 1 (this
            // warp's 2f + h), Q6_K's elements 64f + 32h .. +31; both planes go to
            // half f & 1 of A stage i (use 2 (b / 2) + f / 2 of it), hi at columns
            // 16h .. 16h + 15, lo 32 further on
            for (int b = 0; b < nblk; ++b) {
                const int rs = b & (nraw - 1), i = b & 1;
                if (!mbar_wait(&raw_full[rs], (b >> lgr) & 1, 3u, poisoned)) break;
                const uint8_t* row = smem + L.raw_off(rs) + r * BB;
                // Q6_K / IQ4_XS: the block starts o = 210 kb (136 kb) mod 16 bytes
                // into its box row
                const int o = (TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS) ? ((kb0 + b) * row_blk_bytes<TYPE>()) & 15 : 0;
                uint4 ql[2], qh[2];
                uint32_t shb = 0u, slb = 0u;  // IQ4_XS: scales_h, scales_l
                if constexpr (TYPE == kTypeIQ4_XS) {
                    shb = *reinterpret_cast<const uint16_t*>(row + o + 2);
                    slb = *reinterpret_cast<const uint32_t*>(row + o + 4);
                }
                bool stop = false;
#pragma unroll
                for (int f = 0; f < 4; ++f) {
                    uint32_t hw[2][8], lw[2][8];
                    if constexpr (TYPE == kTypeQ6_K)
                        q6_chunk_planes(row, f, h, o, ql, qh, hw, lw);
                    else if constexpr (TYPE == kTypeIQ4_XS)
                        iq4_chunk_planes(row, f, h, o, shb, slb, hw, lw);
                    else if (h == 0)
                        q8_chunk_planes<0>(row, f, hw, lw);
                    else
                        q8_chunk_planes<1>(row, f, hw, lw);
                    const uint32_t use = static_cast<uint32_t>(2 * (b >> 1) + (f >> 1));
                    if (use >= 1 && !mbar_wait(&a_free[2 * i + (f & 1)], (use - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t acol = static_cast<uint32_t>(P.acol0 + kACols * i + 64 * (f & 1) + 16 * h);
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq) {
                        tmem_st8(trow + acol + static_cast<uint32_t>(8 * qq), hw[qq]);
                        tmem_st8(trow + acol + static_cast<uint32_t>(32 + 8 * qq), lw[qq]);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[2 * i + (f & 1)]);
                }
                if (stop) break;
                if (lane == 0) mbar_arrive(&raw_free[rs]);
            }
        } else {
            for (int b = 0; b < nblk; ++b) {
                const int rs = b & (nraw - 1), i = b & 1;
                if (!mbar_wait(&raw_full[rs], (b >> lgr) & 1, 3u, poisoned)) break;
                const uint8_t* blk = smem + L.raw_off(rs) + r * BB;
                // scales of this thread's sub-blocks j = 2p + h (p = 0..3), get_scale_min_k4
                // (src/inference/jsep/ops/matmul.ts:408-424) on the bytes of the three scale words
                const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
                const uint32_t w1a = __byte_perm(hdr.y, 0u, sel_a), w1b = __byte_perm(hdr.y, 0u, sel_b);
                const uint32_t w3a = __byte_perm(hdr.w, 0u, sel_a), w3b = __byte_perm(hdr.w, 0u, sel_b);
                const uint32_t scv[4] = {w1a & 63u, w1b & 63u, (w3a & 15u) | ((w1a >> 6) << 4),
                                         (w3b & 15u) | ((w1b >> 6) << 4)};
                // the block's quants (and Q5_K high bits), read before the stage wait
                const uint4* qs = reinterpret_cast<const uint4*>(blk + (TYPE == kTypeQ5_K ? 48 : 16));
                uint4 qv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) qv[j] = qs[j];
                uint32_t hv[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
                if constexpr (TYPE == kTypeQ5_K) {
#pragma unroll
                    for (int qq = 0; qq < 2; ++qq) {
                        const uint4 t = *reinterpret_cast<const uint4*>(blk + 16 + 16 * qq);
                        hv[qq][0] = t.x;
                        hv[qq][1] = t.y;
                        hv[qq][2] = t.z;
                        hv[qq][3] = t.w;
                    }
                }
                // A stage i, half f (chunks 2f, 2f + 1; A_min with the second half) is
                // free once issuer i's MMAs of block b - 2 have read it
                const uint32_t acol = static_cast<uint32_t>(P.acol0 + kACols * i + 16 * h);
                bool stop = false;
#pragma unroll
                for (int f = 0; f < 2; ++f) {
                    if (b >= 2 && !mbar_wait(&a_free[2 * i + f], ((b >> 1) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int pp = 0; pp < 2; ++pp) {
                        const int p = 2 * f + pp;
                        // A = sc q exactly: (1024 + q) sc - 1024 sc in one f16 FMA (the
                        // exact result, at most 1953, is an f16 integer); sc itself as the
                        // f16 (1024 + sc) - 1024, both halves
                        const uint32_t sbits = 0x64006400u | (scv[p] * 0x00010001u);
                        const __half2 sc2 = __hsub2(*reinterpret_cast<const __half2*>(&sbits), k1024);
                        const __half2 mn2 = __hmul2(sc2, km1024);
#pragma unroll
                        for (int qq = 0; qq < 2; ++qq) {
                            // bytes 16 qq .. 16 qq + 15 of pair p; this thread's quants are their
                            // low (h = 0) or high (h = 1) nibbles: elements 64p + 32h + 16qq + l
                            const uint4 v0 = qv[2 * p + qq];
                            const uint32_t wv[4] = {v0.x, v0.y, v0.z, v0.w};
                            uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                uint32_t nib = (wv[j] >> (4 * h)) & 0x0F0F0F0Fu;
                                if constexpr (TYPE == kTypeQ5_K) nib |= ((hv[qq][j] >> (2 * p + h)) & 0x01010101u) << 4;
                                // f16 1024 + q (exact) for bytes (0, 1) and (2, 3): 0x64 in each high byte
                                const uint32_t e01 = __byte_perm(nib, 0x00006464u, 0x5140u);
                                const uint32_t e23 = __byte_perm(nib, 0x00006464u, 0x5342u);
                                const __half2 w01 = __hfma2(*reinterpret_cast<const __half2*>(&e01), sc2, mn2);
                                const __half2 w23 = __hfma2(*reinterpret_cast<const __half2*>(&e23), sc2, mn2);
                                out[2 * j] = *reinterpret_cast<const uint32_t*>(&w01);
                                out[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                            }
                            // k = 64p + 32h + 16qq + l of the block: TMEM columns 32p + 16h + 8qq .. +7 of A stage i
                            tmem_st8(trow + acol + static_cast<uint32_t>(32 * p + 8 * qq), out);
                        }
                    }
                    if (f == 1 && h == 0) {
                        // A_min of this block: the eight 6-bit mins (get_scale_min_k4), twice,
                        // as f16 pairs (k 0..7 meet the sums' hi parts, 8..15 their lo parts)
                        const uint32_t mlo = hdr.z & 0x3F3F3F3Fu;                                                  // m_0..m_3
                        const uint32_t mhi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | (((hdr.z >> 6) & 0x03030303u) << 4);  // m_4..m_7
                        uint32_t mm[4];
                        const uint32_t mq[2] = {mlo, mhi};
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            const uint32_t e01 = __byte_perm(mq[t], 0x00006464u, 0x5140u);
                            const uint32_t e23 = __byte_perm(mq[t], 0x00006464u, 0x5342u);
                            const __half2 m01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1024);
                            const __half2 m23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1024);
                            mm[2 * t] = *reinterpret_cast<const uint32_t*>(&m01);
                            mm[2 * t + 1] = *reinterpret_cast<const uint32_t*>(&m23);
                        }
                        const uint32_t amin[8] = {mm[0], mm[1], mm[2], mm[3], mm[0], mm[1], mm[2], mm[3]};
                        tmem_st8(trow + mincol0 + static_cast<uint32_t>(8 * i), amin);
                    }
                    // one wait for the half's stores, then its arrival
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[2 * i + f]);
                }
                if (stop) break;
                if (lane == 0) mbar_arrive(&raw_free[rs]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3;
        const int r = 32 * quarter + lane;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
        if constexpr (TWO) {
          if constexpr (wide) {
            // wide: the four warps of group g = (warp - kFirstEp) / 4 read issuer
            // g's accumulator of every block, all 32 of the group's vectors
            const int g = (warp - kFirstEp) >> 2;
            float ya[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) ya[j] = 0.f;
            for (int b = 0; b < nblk; ++b) {
                const int rs = b & (nraw - 1), ai = 2 * g + (b & 1);
                if (!mbar_wait<64>(&raw_full[rs], (b >> lgr) & 1, 4u, poisoned)) break;
                float d = 1.f;
                if constexpr (TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS) {
                    const int o = ((kb0 + b) * row_blk_bytes<TYPE>()) & 15;
                    d = __half2float(*reinterpret_cast<const __half*>(smem + L.raw_off(rs) + r * BB + o +
                                                                     (TYPE == kTypeQ6_K ? 208 : 0)));
                }
                const float* vs = reinterpret_cast<const float*>(smem + L.v_off(rs)) + g * 2 * nv;  // group g's scales
                if (!mbar_wait<64>(&acc_full[ai], (b >> 1) & 1, 4u, poisoned)) break;
                tc_fence_after();
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {  // 8 vectors at a time (registers)
                    float mv[8], lv[8];
                    tmem_ld8x2(trow + static_cast<uint32_t>(accw * ai + 8 * hh),
                               trow + static_cast<uint32_t>(accw * ai + nv + 8 * hh), mv, lv);  // hi part, lo part
#pragma unroll
                    for (int j = 0; j < 8; ++j) ya[8 * hh + j] = fmaf(mv[j] + lv[j], d * vs[8 * hh + j], ya[8 * hh + j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_free[ai]);
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_free[rs]);
            }
            const int row = m0 + r, tile = blockIdx.x;
            if (P.splits == 1) {
                if (row < P.M) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = 32 * g + j;
                        if (n < P.N)
                            *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * row) = ya[j];
                    }
                }
            } else {
                float* ptile = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kMaxVPC * kTM);
#pragma unroll
                for (int j = 0; j < 32; ++j) ptile[(32 * g + j) * kTM + r] = ya[j];
                // the tile's last split sums all of them in split order, as below
                __shared__ int last_w;
                asm volatile("bar.sync 1, %0;" ::"n"(kEp * 32) : "memory");
                if (threadIdx.x == 32 * kFirstEp) {
                    __threadfence();
                    const unsigned add = 1u + (*poisoned ? 0x10000u : 0u);
                    const unsigned old = atomicAdd(P.counters + tile, add);
                    last_w = (old & 0xFFFFu) == static_cast<unsigned>(P.splits - 1);
                    if (last_w) {
                        if ((old + add) >> 16) last_w = 0;
                        P.counters[tile] = 0u;
                        __threadfence();
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"n"(kEp * 32) : "memory");
                if (last_w) {
                    // thread t sums elements t + 256 k (k < 32: 64 vectors) over the
                    // splits, 16 at a time
                    const float* base = P.partial + static_cast<int64_t>(tile) * P.splits * (kMaxVPC * kTM);
                    const int t = threadIdx.x - 32 * kFirstEp;
#pragma unroll 1
                    for (int part = 0; part < 2; ++part) {
                        float acc[16];
#pragma unroll
                        for (int k = 0; k < 16; ++k) acc[k] = 0.f;
                        for (int z = 0; z < P.splits; ++z) {
                            const float* src = base + z * (kMaxVPC * kTM) + t + kEp * 32 * 16 * part;
#pragma unroll
                            for (int k = 0; k < 16; ++k) acc[k] += __ldcg(src + kEp * 32 * k);
                        }
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int e = t + kEp * 32 * (16 * part + k), n = e / kTM, rr = e - n * kTM;
                            if (n < P.N && m0 + rr < P.M)
                                *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * (m0 + rr)) =
                                    acc[k];
                        }
                    }
                }
            }
          }
        }
        if constexpr (!wide) {
            const int ep = (warp - kFirstEp) >> 2;  // half of the group's vectors
            const int nh = nv / 2, n0 = ep * nh;  // this warp's vectors (8 or 16)
            float yacc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) yacc[j] = 0.f;
            for (int b = 0; b < nblk; ++b) {
                const int i = b & 1, rs = b & (nraw - 1);
                // the block's d, dmin and scales first (they need only the raw slot);
                // Q8_0's d is inside its weight planes, Q6_K's at byte 208 of the
                // block, IQ4_XS's at byte 0
                if (!mbar_wait<64>(&raw_full[rs], (b >> lgr) & 1, 4u, poisoned)) break;
                float d = 1.f, dmin = 0.f;
                if constexpr (TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS) {
                    const int o = ((kb0 + b) * row_blk_bytes<TYPE>()) & 15;
                    d = __half2float(*reinterpret_cast<const __half*>(smem + L.raw_off(rs) + r * BB + o +
                                                                     (TYPE == kTypeQ6_K ? 208 : 0)));
                } else if constexpr (!TWO) {
                    const uint32_t dm = *reinterpret_cast<const uint32_t*>(smem + L.raw_off(rs) + r * BB);
                    d = f16_bits_to_f32(dm);
                    dmin = f16_bits_to_f32(dm >> 16);
                }
                const float* vs = reinterpret_cast<const float*>(smem + L.v_off(rs)) + n0;  // [2][nv] from vector n0
                if (!mbar_wait<64>(&acc_full[i], (b >> 1) & 1, 4u, poisoned)) break;
                tc_fence_after();
                float mv[16], lv[16], sv[16];
                if constexpr (TWO)
                    tmem_ld16x2(trow + static_cast<uint32_t>(accw * i + n0), trow + static_cast<uint32_t>(accw * i + nv + n0),
                                mv, lv);  // hi part, lo part
                else
                    tmem_ld16x3(trow + static_cast<uint32_t>(accw * i + n0), trow + static_cast<uint32_t>(accw * i + nv + n0),
                                trow + static_cast<uint32_t>(accw * i + 2 * nv + n0), mv, lv, sv);  // hi part, lo part, mins
                // the accumulators are read: the issuer may start on block b + 2
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_free[i]);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (j >= nh) continue;
                    if constexpr (TWO)
                        yacc[j] = fmaf(mv[j] + lv[j], d * vs[j], yacc[j]);
                    else
                        yacc[j] = fmaf(mv[j] + lv[j], d * vs[j], fmaf(-sv[j], dmin * vs[nv + j], yacc[j]));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_free[rs]);
            }
            // ---------------- outputs ----------------
            const int row = m0 + r;
            const int nbase = grp * nv;  // first vector of this group
            const int tile = blockIdx.y * gridDim.x + blockIdx.x;
            if (P.splits == 1) {
                if (row < P.M) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = nbase + n0 + j;
                        if (j < nh && n < P.N)
                            *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * row) = yacc[j];
                    }
                }
            } else {
                float* ptile = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kMaxVPC * kTM);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (j < nh) ptile[(n0 + j) * kTM + r] = yacc[j];
                // the tile's last split sums all of them in split order (deterministic);
                // a split that gave up waiting counts in the high half and nobody sums
                __shared__ int last;
                asm volatile("bar.sync 1, %0;" ::"n"(kEp * 32) : "memory");
                if (threadIdx.x == 32 * kFirstEp) {
                    __threadfence();
                    const unsigned add = 1u + (*poisoned ? 0x10000u : 0u);
                    const unsigned old = atomicAdd(P.counters + tile, add);
                    last = (old & 0xFFFFu) == static_cast<unsigned>(P.splits - 1);
                    if (last) {
                        if ((old + add) >> 16) last = 0;
                        P.counters[tile] = 0u;
                        __threadfence();
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"n"(kEp * 32) : "memory");
                if (last) {
                    // thread t sums elements t + 256 k (k < nv / 2) over the splits, in
                    // split order, with each split's loads issued together
                    const float* base = P.partial + static_cast<int64_t>(tile) * P.splits * (kMaxVPC * kTM);
                    const int t = threadIdx.x - 32 * kFirstEp, per = nv * kTM / (kEp * 32);
                    float acc[kMaxNV * kTM / (kEp * 32)];
#pragma unroll
                    for (int k = 0; k < kMaxNV * kTM / (kEp * 32); ++k) acc[k] = 0.f;
                    for (int z = 0; z < P.splits; ++z) {
                        const float* src = base + z * (kMaxVPC * kTM) + t;
#pragma unroll
                        for (int k = 0; k < kMaxNV * kTM / (kEp * 32); ++k)
                            if (k < per) acc[k] += __ldcg(src + kEp * 32 * k);
                    }
#pragma unroll
                    for (int k = 0; k < kMaxNV * kTM / (kEp * 32); ++k) {
                        const int e = t + kEp * 32 * k, n = e / kTM, rr = e - n * kTM;
                        if (k < per && nbase + n < P.N && m0 + rr < P.M)
                            *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + (nbase + n) * P.y_nb1 + 4LL * (m0 + rr)) =
                                acc[k];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// The activation image, one warp per vector n and 256-element block b (lane
// l holds elements 8 l .. 8 l + 7): the block's power-of-two scale 2^e (its
// maximum |x| in [2^14, 2^15) after scaling), the hi / lo f16 parts, and the
// f16 hi / lo parts of its eight 32-element sums at scale 2^(e + 5) (each sum
// in double over four lanes); zeros past N. Vector n is vector n % nv of group
// n / nv; a group's hi rows are followed by its lo rows. CTA (0, 0) also zeroes
// the split-K tile counters. The GEMM that follows may start at once (its
// prologue and first weight loads overlap this kernel; it waits for the
// image with griddepcontrol.wait).
__global__ void btc_prep_kernel(const float* __restrict__ x, int64_t x_nb1, __half* __restrict__ ximg,
                                __half* __restrict__ simg, float* __restrict__ vscale, int K, int N, int nv, int groups,
                                unsigned* __restrict__ counters, int ncounters) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int t = threadIdx.x; t < ncounters; t += blockDim.x) counters[t] = 0u;
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int b = blockIdx.x;
    const int np = nv * groups, g = n / nv, l = n - g * nv;
    if (n >= np) return;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (n < N) {
        const float* xn = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(x) + n * x_nb1) + 256 * b + 8 * lane;
        if ((reinterpret_cast<uintptr_t>(xn) & 15) == 0) {
            const float4 a0 = __ldg(reinterpret_cast<const float4*>(xn));
            const float4 a1 = __ldg(reinterpret_cast<const float4*>(xn) + 1);
            v[0] = a0.x, v[1] = a0.y, v[2] = a0.z, v[3] = a0.w, v[4] = a1.x, v[5] = a1.y, v[6] = a1.z, v[7] = a1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = __ldg(xn + i);
        }
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int E = 0;
    frexpf(mx, &E);  // mx < 2^E
    const int e = (mx > 0.f && isfinite(mx)) ? E - 15 : 0;
    uint32_t hw[4], lw[4];
    double acc = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float s0 = ldexpf(v[2 * i], -e), s1 = ldexpf(v[2 * i + 1], -e);
        const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
        const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
        hw[i] = static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
        lw[i] = static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
        acc += static_cast<double>(v[2 * i]) + static_cast<double>(v[2 * i + 1]);
    }
    const int64_t k = 256LL * b + 8 * lane;
    const int64_t hrow = static_cast<int64_t>(g) * 2 * nv + l;
    *reinterpret_cast<uint4*>(ximg + hrow * K + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(ximg + (hrow + nv) * K + k) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    // sub-block lane / 4: the four lanes' partial sums
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    __half* row = simg + (static_cast<int64_t>(b) * np + n) * 64;  // 128 bytes
    if ((lane & 3) == 0) {
        const double sv = ldexp(acc, -(e + 5));
        const __half hs = __double2half(sv);
        row[lane >> 2] = hs;
        row[8 + (lane >> 2)] = __double2half(sv - static_cast<double>(__half2float(hs)));
    } else if (lane < 8) {
        // bytes 32 .. 127 of the row are zero (the mins MMA reads K = 16): lanes
        // 1, 2, 3, 5, 6, 7 write one 16-byte piece each
        const int j = lane - 1 - (lane >> 2);  // 0 .. 5
        reinterpret_cast<uint4*>(row)[2 + j] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (lane == 0) {
        float* vsb = vscale + ((static_cast<int64_t>(b) * groups + g) * 2) * nv + l;
        vsb[0] = ldexpf(1.f, e);
        vsb[nv] = ldexpf(1.f, e + 5);
    }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn btc_encoder() {
    static EncodeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        cudaGetLastError();
        return reinterpret_cast<EncodeFn>(p);
    }();
    return fn;
}

// Vectors per CTA (16 or 32) and vector groups: N <= 32 is one group of N
// rounded up to 16; N = 33..64 is two groups of 32.
int nv_of(const MulMatOp& o) { return o.N <= 16 ? 16 : 32; }
int groups_of(const MulMatOp& o) { return (o.N + nv_of(o) - 1) / nv_of(o); }
int np_of(const MulMatOp& o) { return nv_of(o) * groups_of(o); }
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
size_t ximg_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(2) * np_of(o) * o.K * 2); }
size_t simg_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(o.K / 256) * np_of(o) * 128); }
size_t vscale_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(o.K / 256) * 2 * np_of(o) * 4); }
// Two-plane types (Q8_0, Q6_K, IQ4_XS) above 32 vectors run both vector groups in one
// CTA: its two MMA issuers take one group each of every block.
bool two_of(const MulMatOp& o) { return o.type == kTypeQ8_0 || o.type == kTypeQ6_K || o.type == kTypeIQ4_XS; }
bool wide_of(const MulMatOp& o) { return two_of(o) && groups_of(o) == 2; }
int tiles_of(const MulMatOp& o) { return (o.M + kTM - 1) / kTM * (wide_of(o) ? 1 : groups_of(o)); }

// K splits: about one wave of CTAs (one per SM), at least two blocks per split.
int plan_splits(const MulMatOp& o, int num_sms) {
    const int tiles = tiles_of(o), nblk = o.K / 256;
    int s = num_sms / tiles;
    s = s < kMaxSplits ? s : kMaxSplits;
    s = s < nblk / 2 ? s : nblk / 2;
    return s > 1 ? s : 1;
}
size_t split_bytes(const MulMatOp& o, int splits) {
    if (splits <= 1) return 0;
    const size_t tiles = static_cast<size_t>(tiles_of(o));
    return align256(tiles * splits * kMaxVPC * kTM * 4) + align256(tiles * 4);
}

// Bytes per row of one 256-element block in a raw slot, and in the weights.
int host_blk_bytes(int type) {
    return type == kTypeQ5_K ? 176 : (type == kTypeQ8_0 ? 272 : (type == kTypeQ6_K ? 240 : 144));
}
int host_row_blk_bytes(int type) {
    return type == kTypeQ6_K ? 210 : (type == kTypeIQ4_XS ? 136 : host_blk_bytes(type));
}

}  // namespace

bool batched_tc_supported(const MulMatOp& o) {
    if (o.type != kTypeQ4_K && o.type != kTypeQ5_K && o.type != kTypeQ8_0 && o.type != kTypeQ6_K &&
        o.type != kTypeIQ4_XS)
        return false;
    if (o.N < 1 || o.N > kMaxNP || o.ne2 != 1 || o.ne3 != 1) return false;
    if (o.K % 256 != 0 || o.M < 1) return false;
    // TMA rows: 16-byte aligned base and row stride
    if ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15) return false;
    if (o.w_nb1 < static_cast<int64_t>(o.K / 256) * host_row_blk_bytes(o.type)) return false;
    // the 240- or 144-byte box stays within a row's width
    if ((o.type == kTypeQ6_K || o.type == kTypeIQ4_XS) && o.K < 512) return false;
    if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 3) return false;
    return btc_encoder() != nullptr;
}

size_t batched_tc_workspace_bytes(const MulMatOp& o) {
    // room for the most splits any device plans (plan_splits caps them)
    return ximg_bytes(o) + simg_bytes(o) + vscale_bytes(o) + split_bytes(o, plan_splits(o, 1 << 20)) + 256;
}

int launch_batched_tc(const MulMatOp& o, void* workspace, size_t workspace_bytes, cudaStream_t stream, int num_sms) {
    if (!batched_tc_supported(o)) return -static_cast<int>(cudaErrorInvalidValue);
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255)) return -static_cast<int>(cudaErrorInvalidValue);
    int splits = plan_splits(o, num_sms);
    const size_t base = ximg_bytes(o) + simg_bytes(o) + vscale_bytes(o);
    if (base + split_bytes(o, splits) > workspace_bytes) splits = 1;
    if (base > workspace_bytes) return -static_cast<int>(cudaErrorInvalidValue);
    const int nv = nv_of(o), groups = groups_of(o), np = np_of(o), nblk = o.K / 256;
    const int kb_split = (nblk + splits - 1) / splits;
    splits = (nblk + kb_split - 1) / kb_split;  // no empty split
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* ximg = reinterpret_cast<__half*>(ws);
    __half* simg = reinterpret_cast<__half*>(ws + ximg_bytes(o));
    float* vscale = reinterpret_cast<float*>(ws + ximg_bytes(o) + simg_bytes(o));
    cudaError_t e = cudaSuccess;
    BtcArgs P{};
    const EncodeFn enc = btc_encoder();
    const int bb = host_blk_bytes(o.type);
    const bool two = two_of(o);  // two weight planes, no mins
    const bool q6 = o.type == kTypeQ6_K, iq4 = o.type == kTypeIQ4_XS;
    const bool bytemap = q6 || iq4;  // rows mapped in bytes, 240- or 144-byte boxes
    const cuuint32_t es[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {bytemap ? static_cast<cuuint64_t>(nblk) * host_row_blk_bytes(o.type)
                                            : static_cast<cuuint64_t>(nblk) * (bb / 8),
                                    static_cast<cuuint64_t>(o.M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.w_nb1)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(bytemap ? bb : bb / 8), static_cast<cuuint32_t>(kTM)};
        if (enc(&P.wmap, bytemap ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(o.w),
                dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(o.K), static_cast<cuuint64_t>(2 * np)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.K) * 2};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), static_cast<cuuint32_t>(2 * nv)};
        if (enc(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ximg, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(nblk) * np};
        const cuuint64_t strides[1] = {128};
        const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(nv)};
        if (enc(&P.smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, simg, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    // TMEM: per issuer the accumulators (an epilogue warp reads 16-column
    // groups from its first vector, nv / 2 of them: the columns cover the
    // overhang; no mins columns for two-plane types; wide: two per issuer),
    // then A_min (8 columns each, K-quants) and the two A stages from a
    // 32-column boundary
    const bool wide = wide_of(o);
    P.wide = wide ? 1 : 0;
    {
        const int nh = nv / 2;
        const int need = two ? max(2 * nv, nv + nh + 16) : max(3 * nv, 2 * nv + nh + 16);
        P.accw = (need + 31) / 32 * 32;
        P.acol0 = ((wide ? 4 : 2) * P.accw + (two ? 0 : 16) + 31) / 32 * 32;
        if (P.acol0 + 2 * kACols > kTmemCols) return -static_cast<int>(cudaErrorInvalidValue);
    }
    // raw slots and B stages within 224 KB: 8 raw slots where 4 B stages still
    // fit, else 4 raw slots and as many B stages (4 or 2) as fit (wide, whose
    // B stages hold both groups: 2 raw slots where 4 leave room for one)
    {
        const auto stages_with = [&](int nraw) {
            const Smem s0(nv, bb, 0, nraw, !two, wide);
            return (static_cast<int>(224u << 10) - static_cast<int>(s0.total())) / static_cast<int>(s0.b_bytes);
        };
        int nb = stages_with(8);
        P.nraw = 8;
        if (nb < 4) {
            nb = stages_with(4);
            P.nraw = 4;
        }
        if (nb < 2 && wide) {
            nb = stages_with(2);
            P.nraw = 2;
        }
        if (nb < 2) return -static_cast<int>(cudaErrorInvalidValue);
        P.nstb = nb >= 4 ? 4 : 2;
    }
    P.vscale = vscale;
    P.y = o.y;
    P.y_nb1 = o.y_nb1;
    P.M = o.M;
    P.K = o.K;
    P.N = o.N;
    P.nv = nv;
    P.groups = groups;
    P.splits = splits;
    P.kb_split = kb_split;
    const int tiles = tiles_of(o);
    if (splits > 1) {
        P.partial = reinterpret_cast<float*>(ws + base);
        P.counters = reinterpret_cast<unsigned*>(ws + base + align256(static_cast<size_t>(tiles) * splits * kMaxVPC * kTM * 4));
    }
    btc_prep_kernel<<<dim3(nblk, np / 8), 256, 0, stream>>>(o.x, o.x_nb1, ximg, simg, vscale, o.K, o.N, nv, groups,
                                                            P.counters, splits > 1 ? tiles : 0);
    if ((e = cudaGetLastError()) != cudaSuccess) return -static_cast<int>(e);
    const size_t smem = Smem(nv, bb, P.nstb, P.nraw, !two, wide).total();
    static size_t configured[kMaxDevices][8] = {};
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return -static_cast<int>(e);
    if (dev < 0 || dev >= kMaxDevices) return -static_cast<int>(cudaErrorInvalidDevice);
    const int ti = o.type == kTypeQ5_K   ? 1
                   : o.type == kTypeQ8_0 ? (wide ? 4 : 2)
                   : q6                  ? (wide ? 5 : 3)
                   : iq4                 ? (wide ? 7 : 6)
                                         : 0;
    void (*const kernel)(BtcArgs) = ti == 1   ? btc_kernel<kTypeQ5_K, false>
                                    : ti == 2 ? btc_kernel<kTypeQ8_0, false>
                                    : ti == 3 ? btc_kernel<kTypeQ6_K, false>
                                    : ti == 4 ? btc_kernel<kTypeQ8_0, true>
                                    : ti == 5 ? btc_kernel<kTypeQ6_K, true>
                                    : ti == 6 ? btc_kernel<kTypeIQ4_XS, false>
                                    : ti == 7 ? btc_kernel<kTypeIQ4_XS, true>
                                              : btc_kernel<kTypeQ4_K, false>;
    if (configured[dev][ti] < smem) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return -static_cast<int>(e);
        configured[dev][ti] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((o.M + kTM - 1) / kTM, wide ? 1 : groups, splits);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, P);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? 2 : -static_cast<int>(e);
}

unsigned read_and_clear_btc_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_btc_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_btc_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace wllm
