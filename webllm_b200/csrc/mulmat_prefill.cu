// Prefill-regime quantized MUL_MAT (N >= kPrefillMinN activation vectors, Q4_K,
// Q5_K, Q6_K, Q8_0 or Q4_0 weights): a tcgen05 tensor-core GEMM that dequantizes the GGUF blocks
// to f16 on the way into tensor memory.
//
//   y[m + M n] = sum_k W[m, k] x[k + K n]   (ggml MUL_MAT, matmul.ts:10-17)
//
// One CTA computes a 128 (rows of W) x 256 (vectors) tile of y with the
// accumulator in tensor memory (TMEM, 128 lanes x 256 f32 columns): each
// dequantized weight feeds 256 vectors, which keeps the dequantization (the
// CUDA-core side) ahead of the MMAs. K is walked in chunks of 64.
//
//  - warp 0 (TMA): per 256-element block, one 2D box of the 128 rows' raw
//    blocks into a raw ring (Q4_K: 128 x 144 B; Q6_K: 128 x 240 B, the 210-byte
//    block from the 16-byte boundary at or below its start, which is 2 kb mod 16
//    bytes into the row's box); per 64-chunk, one 2D box of the
//    f16 activations (64 x 256, TMA 128-byte swizzle) into a B stage: the
//    canonical K-major UMMA layout (vector n at (n/8)*1024 + (n%8)*128 bytes,
//    its 16-byte piece j at position j ^ (n%8)).
//  - warps 2..17 (dequant, 512 threads): warp w handles rows 32 (w%4) + lane
//    (the TMEM lanes it may access) and quarter (w-2)/4 of each chunk: it turns
//    16 quants of sub-block 2p+h (chunk p of the block) into f16
//    d*sc*q - dmin*m (the quant enters as the exact f16 1024 + q, minus 1024,
//    then one f16 FMA) and stores them with tcgen05.st straight into the A
//    operand's TMEM columns (row = lane, two f16 per column). The weights thus
//    never pass through shared memory, whose bandwidth the MMAs' B reads and
//    the TMA writes need.
//  - warp 1 (MMA): TMEM allocation; one elected thread issues the 4 K=16
//    tcgen05.mma (A from TMEM, B from shared memory; M=128, N=256,
//    f16 x f16 -> f32) of each chunk and commits them to the chunk's "stage
//    free" barrier.
//  - epilogue (warps 2..17): tcgen05.ld of the accumulator (warp w reads TMEM
//    lanes 32 (w%4) .. +31, i.e. rows, and a quarter of the columns), f32
//    stores to y.
//
// The activations are converted to f16 by a pre-pass (x_to_f16_kernel) into
// library workspace: N x K x 2 bytes, read by every row tile from L2.
//
// Split K: grids far below two CTAs per SM (few row tiles) or with long K run
// S splits of the K blocks per tile (grid z, one cluster per tile). Each split
// stores its f32 tile in workspace; after a cluster barrier each split sums
// its slice of the tile's columns over the S tiles in split order, so results
// do not depend on timing and the reduction runs on S SMs.
//
// Every mbarrier wait is bounded; on timeout the CTA records an error code
// (read by wllm_sync), stops issuing work, and still releases its TMEM.
#include <algorithm>
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_prefill_error = 0;

namespace {

constexpr int kTileM = 128;                      // rows of W per CTA (TMEM lanes)
constexpr int kTileN = 256;                      // vectors per CTA (TMEM columns)
constexpr int kChunkK = 64;                      // K per stage (one 128-byte swizzle atom of f16)
constexpr int kStages = 4;                       // B stages in smem, A stages in TMEM
constexpr int kRawSlots = 2;                     // raw blocks in flight (each feeds 4 chunks)
constexpr int kQ6Box = 240;                      // bytes of a Q6_K box row: offset (<= 14) + 210, rounded to 16
                                                 // and made 60 words (16-byte loads of 8 rows hit 32 banks)
template <int TYPE>
__host__ __device__ constexpr int raw_row_bytes() {
    return TYPE == kTypeQ6_K ? kQ6Box : (TYPE == kTypeQ5_K ? 176 : (TYPE == kTypeQ8_0 ? 272 : 144));
}
// one box row per 256 elements: Q4_K 144 B, Q5_K 176 B, Q8_0 272 B (8 blocks),
// Q4_0 144 B (8 blocks), Q6_K 240 B; all rows 16-byte multiples with
// conflict-free 16-byte loads
template <int TYPE>
__host__ __device__ constexpr int raw_bytes() { return kTileM * raw_row_bytes<TYPE>(); }
constexpr int kBBytes = kTileN * kChunkK * 2;    // 32768
constexpr int kDqWarps = 16;
constexpr int kThreads = 32 * (2 + kDqWarps);    // TMA warp, MMA warp, dequant/epilogue warps
constexpr int kACols = kChunkK / 2;              // TMEM columns of one A stage (two f16 per column)
// accumulator (kTileN) + kStages A stages = 384 columns, allocated as 512: one
// CTA per SM (about 165 KB of shared memory)
constexpr int kTmemCols = 512;
static_assert(kTileN + kStages * kACols <= kTmemCols, "TMEM budget");
constexpr uint32_t kSpinLimit = 1u << 26;

struct PrefillArgs {
    CUtensorMap wmap;   // weights: Q4_K [M rows][row_bytes / 8] uint64, box 18 x 128 (one block column);
                        // Q6_K [M rows][row_bytes] uint8, box 240 x 128 (rows grouped by
                        // G = 2, 4, 8: [M / G][G w_nb1] uint8, box 240 x 128 / G)
    CUtensorMap xmap;   // f16 activations: [N][K], box 64 x 128, 128-byte swizzle
    float* y;
    int64_t y_nb1;      // bytes between output vectors
    int32_t M, K, N;
    // split-K (splits > 1): CTA z of a tile covers K blocks [z kb_split, (z+1) kb_split)
    // and writes its f32 tile to partial[tile][z][col][row]; the tile's splits
    // are one cluster, and after a cluster barrier CTA z sums slice z of the
    // tile's columns over the splits in order. counters[tile] (zeroed by the
    // pre-pass) marks a tile one of whose splits gave up waiting
    int32_t splits, kb_split;
    // byte-mapped rows (Q6_K, IQ4_XS) whose stride is not a multiple of 16
    // bytes (Q6_K K = 3072: 2520 B, K = 2304: 1890 B): the map is over groups
    // of G = 2^row_lg rows (G w_nb1 bytes, a legal stride), and each block
    // takes G boxes of 128 / G groups, box j from the block's start in row j
    // of the group; 0 for rows 16-byte apart
    int32_t row_lg;
    int32_t w_nb1;
    float* partial;
    unsigned* counters;
};

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
// Bounded wait for a phase whatever the poison flag says (draining copies and
// MMAs in flight before the CTA exits); false on time-out.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}

// Bounded wait; a timeout poisons the CTA (every later wait returns at once).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 255u) == 255u && *poisoned) return false;
    }
    *poisoned = 1;
    atomicOr(&g_prefill_error, code);
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor, kind::f16: f16 A and B (K-major), f32 accumulator,
// M = 128, N = kTileN.
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kTileN >> 3) << 17) | (static_cast<uint32_t>(kTileM >> 4) << 24);

// D (TMEM) += A (TMEM, K-major) * B (shared memory descriptor).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        :
        : "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// 8 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive f32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 bytes at byte o + c of a Q6_K box row (c a multiple of 16, o the block's
// offset: even, the same for every row and thread of the block), from the two
// aligned 16-byte words at c: word select by o / 4, then a funnel shift by
// 8 (o % 4) bits.
__device__ __forceinline__ uint4 q6_load16(const uint8_t* rowp, int c, int q4, uint32_t sh) {
    const uint4* a = reinterpret_cast<const uint4*>(rowp + c);
    const uint4 lo = a[0], hi = (q4 | sh) ? a[1] : lo;  // an aligned piece needs no second word
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = q4 == 0 ? w[i] : (q4 == 1 ? w[i + 1] : (q4 == 2 ? w[i + 2] : w[i + 3]));
    return make_uint4(__funnelshift_r(v[0], v[1], sh), __funnelshift_r(v[1], v[2], sh), __funnelshift_r(v[2], v[3], sh),
                      __funnelshift_r(v[3], v[4], sh));
}

// The weight box's x coordinate for K block kb: Q6_K (210 B) and IQ4_XS
// (136 B) blocks are mapped in bytes, from the block's start rounded down to
// 16; the others in uint64 words, block-aligned.
template <int TYPE>
__device__ __forceinline__ int byte_box_x(int kb) {
    if constexpr (TYPE == kTypeQ6_K) return (kb * 210) & ~15;
    if constexpr (TYPE == kTypeIQ4_XS) return (kb * 136) & ~15;
    return kb * (raw_row_bytes<TYPE>() / 8);
}

// Bytes of one block column (256 elements) of a byte-mapped row.
template <int TYPE>
__host__ __device__ constexpr int byte_blk_bytes() { return TYPE == kTypeQ6_K ? 210 : 136; }

// Copies K block kb of the tile's 128 rows from row m0 into a raw slot. Row
// r of the tile lands in box row (r mod G) (128 / G) + r / G of the slot.
template <int TYPE>
__device__ __forceinline__ void issue_raw(uint8_t* dst, const PrefillArgs& P, int kb, int m0, uint64_t* bar) {
    if constexpr (TYPE == kTypeQ6_K || TYPE == kTypeIQ4_XS) {
        const int lg = P.row_lg;
        for (int j = 0; j < (1 << lg); ++j)
            tma_2d(dst + j * (kTileM >> lg) * raw_row_bytes<TYPE>(), &P.wmap,
                   (kb * byte_blk_bytes<TYPE>() + j * P.w_nb1) & ~15, m0 >> lg, bar);
    } else {
        tma_2d(dst, &P.wmap, byte_box_x<TYPE>(kb), m0, bar);
    }
}

// A byte-mapped row's place in a raw slot (box row) and its block's offset
// in that box row (0..15).
template <int TYPE>
__device__ __forceinline__ int byte_row_slot(const PrefillArgs& P, int r) {
    const int j = r & ((1 << P.row_lg) - 1);
    return j * (kTileM >> P.row_lg) + (r >> P.row_lg);
}
template <int TYPE>
__device__ __forceinline__ int byte_row_off(const PrefillArgs& P, int kb, int r) {
    return (kb * byte_blk_bytes<TYPE>() + (r & ((1 << P.row_lg) - 1)) * P.w_nb1) & 15;
}

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillArgs P) {
    constexpr int kRawBytes = raw_bytes<TYPE>();
    constexpr bool kOneWait = TYPE != kTypeQ6_K && TYPE != kTypeIQ4_XS;  // the MMA thread waits on a_full alone
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* B = smem;                                   // [kStages][kBBytes]
    uint8_t* raw = B + kStages * kBBytes;                // [kRawSlots][kRawBytes]
    uint64_t* b_full = reinterpret_cast<uint64_t*>(raw + kRawSlots * kRawBytes);
    uint64_t* a_full = b_full + kStages;
    uint64_t* st_free = a_full + kStages;
    uint64_t* raw_full = st_free + kStages;
    uint64_t* raw_free = raw_full + kRawSlots;
    uint64_t* acc_full = raw_free + kRawSlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* poisoned = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTileM, n0 = blockIdx.y * kTileN;
    const int kb0 = blockIdx.z * P.kb_split;                          // first K block of this split
    const int nblk = min(P.K / 256 - kb0, P.kb_split), nchunk = nblk * 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&a_full[s], kDqWarps);
            mbar_init(&st_free[s], 1);
        }
        for (int r = 0; r < kRawSlots; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_free[r], kDqWarps);
        }
        mbar_init(acc_full, 1);
        *poisoned = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // TMEM: 128 columns x 128 lanes of f32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&P.wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&P.xmap) : "memory");
            int raw_issued = 0, b_issued = 0;  // copies issued (for the drain below)
            // the weights do not depend on the f16 pre-pass: the first raw slots
            // go out before the wait for it (programmatic launch)
            const int pre = min(nchunk >> 2, kRawSlots);
            for (int kb = 0; kb < pre; ++kb) {
                mbar_expect_tx(&raw_full[kb], kRawBytes);
                issue_raw<TYPE>(raw + kb * kRawBytes, P, kb0 + kb, m0, &raw_full[kb]);
                raw_issued = kb + 1;
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int q = 0; q < nchunk; ++q) {
                const int kb = q >> 2, c = q & 3;
                if (c == 0 && kb >= pre) {
                    const int r = kb % kRawSlots;
                    if (kb >= kRawSlots && !mbar_wait(&raw_free[r], ((kb / kRawSlots) - 1) & 1, 1u, poisoned)) break;
                    mbar_expect_tx(&raw_full[r], kRawBytes);
                    issue_raw<TYPE>(raw + r * kRawBytes, P, kb0 + kb, m0, &raw_full[r]);
                    raw_issued = kb + 1;
                }
                const int s = q % kStages;
                if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 1u, poisoned)) break;
                mbar_expect_tx(&b_full[s], kBBytes);
                tma_2d(B + s * kBBytes, &P.xmap, (4 * kb0 + q) * kChunkK, n0, &b_full[s]);
                b_issued = q + 1;
            }
            // Before the CTA can exit: the last copy into every raw slot and
            // stage has landed (bounded, whatever the poison flag says). In a
            // healthy launch the consumers waited for all of them already; after
            // a time-out they may not have, and a copy still in flight would
            // write into the shared memory of the next CTA on this SM.
            for (int kb = max(0, raw_issued - kRawSlots); kb < raw_issued; ++kb)
                if (!mbar_wait_drain(&raw_full[kb % kRawSlots], (kb / kRawSlots) & 1)) atomicOr(&g_prefill_error, 16u);
            for (int q = max(0, b_issued - kStages); q < b_issued; ++q)
                if (!mbar_wait_drain(&b_full[q % kStages], (q / kStages) & 1)) atomicOr(&g_prefill_error, 16u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread) ----------------
        // The loop runs on lane 0 alone, with the B descriptors advanced from
        // one base: warp-wide broadcasts and syncs around each chunk's waits
        // cost the issuing thread as much as the chunk's four MMAs take.
        // Chunks go in pairs (q, q + 1; nchunk is a multiple of 4): one wait on
        // chunk q + 1's A barrier covers both, since every dequant warp arrives
        // for q before q + 1 (and with kOneWait the first one waited for each
        // chunk's B box before arriving).
        if (lane == 0) {
            int committed = 0;  // chunks whose MMAs were committed
            const uint64_t bdesc0 = umma_desc_sw128(smem_u32(B));  // + (byte offset >> 4)
            for (int q = 0; q < nchunk; q += 2) {
                const int s0 = q % kStages;  // chunk q + 1 is in stage s0 + 1 of the same round
                const uint32_t par = (q / kStages) & 1;
                if ((!kOneWait &&
                     (!mbar_wait(&b_full[s0], par, 2u, poisoned) || !mbar_wait(&b_full[s0 + 1], par, 2u, poisoned))) ||
                    !mbar_wait(&a_full[s0 + 1], par, 2u, poisoned)) {
                    // a time-out: the MMAs already issued still write TMEM, which is
                    // freed at the end; wait (bounded) for the last commit, which
                    // tracks all of them
                    if (committed > 0 &&
                        !mbar_wait_drain(&st_free[(committed - 1) % kStages], ((committed - 1) / kStages) & 1))
                        atomicOr(&g_prefill_error, 16u);
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    const int s = s0 + c2;
                    const uint32_t a0 = tmem + static_cast<uint32_t>(kTileN + s * kACols);
                    const uint64_t bd = bdesc0 + static_cast<uint64_t>((s * kBBytes) >> 4);
#pragma unroll
                    for (int ks = 0; ks < kChunkK / 16; ++ks)  // K = 16 per MMA: 8 TMEM columns of A, 32 bytes of B's row
                        umma_f16_ts(tmem, a0 + 8 * ks, bd + 2 * ks, (q + c2 > 0 || ks > 0) ? 1u : 0u);
                    umma_commit(&st_free[s]);  // the stage is free once these MMAs have read it
                }
                if (q + 2 == nchunk) umma_commit(acc_full);
                committed = q + 2;
            }
        }
        __syncwarp();
    } else {
        // ---------------- dequant (then epilogue) ----------------
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int dw = warp - 2;
        const int part = dw >> 2;      // quarter of each chunk's K
        const int r = 32 * quarter + lane, h = part >> 1, qq = part & 1;  // row; sub-block 2p + h, its half qq
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
        const uint32_t sel_a = 0x4440u + static_cast<uint32_t>(h);      // byte h, zero-extended
        const uint32_t sel_b = 0x4440u + 2u + static_cast<uint32_t>(h);  // byte 2 + h
        const __half2 k1024 = __float2half2_rn(1024.f);
        int q = 0;
        bool stop = false;
        for (int kb = 0; kb < nblk && !stop; ++kb) {
            const int rs = kb % kRawSlots;
            if (!mbar_wait(&raw_full[rs], (kb / kRawSlots) & 1, 3u, poisoned)) break;
            if constexpr (TYPE == kTypeQ6_K) {
                // Q6_K (ggml's dequantize_row_q6_K layout, as in quant_blocks.cuh):
                // element 64p + 32h + 16qq + l of the block is in half p/2,
                // j = 2 (p%2) + h: ql byte 64 (p/2) + 32 h + 16 qq + l (high nibble when
                // p is odd), qh byte 128 + 32 (p/2) + 16 qq + l shifted by 2 j, scale
                // 192 + 8 (p/2) + 2 j + qq; w = d sc (q - 32)
                // grouped rows: the offset depends on the row's place in its group
                // (per thread, not per warp)
                const int o = byte_row_off<TYPE>(P, kb0 + kb, r);
                const uint8_t* rowp = raw + rs * kRawBytes + byte_row_slot<TYPE>(P, r) * kQ6Box;
                const int q4 = o >> 2;
                const uint32_t sh = 8u * static_cast<uint32_t>(o & 3);
                const float d = __half2float(*reinterpret_cast<const __half*>(rowp + o + 208));
                const __half2 k1056 = __float2half2_rn(1056.f);
                uint4 ql = make_uint4(0u, 0u, 0u, 0u), qh = ql;
#pragma unroll
                for (int p = 0; p < 4; ++p, ++q) {
                    const int s = q % kStages;
                    if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    const int ip = p >> 1, hb = p & 1, j = 2 * hb + h;
                    if (hb == 0) {  // one load of each array per half
                        ql = q6_load16(rowp, 64 * ip + 32 * h + 16 * qq, q4, sh);
                        qh = q6_load16(rowp, 128 + 32 * ip + 16 * qq, q4, sh);
                    }
                    const float sc = static_cast<float>(static_cast<int8_t>(rowp[o + 192 + 8 * ip + 2 * j + qq]));
                    const __half2 ds2 = __float2half2_rn(d * sc);
                    const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
                    uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t qv = ((lw[i] >> (4 * hb)) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * j)) & 0x03030303u) << 4);
                        // f16 1024 + q (exact, q < 64), minus 1056: q - 32 exactly
                        const uint32_t e01 = __byte_perm(qv, 0x00006464u, 0x5140u);
                        const uint32_t e23 = __byte_perm(qv, 0x00006464u, 0x5342u);
                        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1056);
                        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1056);
                        const __half2 w01 = __hmul2(q01, ds2), w23 = __hmul2(q23, ds2);
                        out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                        out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                    }
                    tmem_st8(trow + static_cast<uint32_t>(kTileN + s * kACols + 16 * h + 8 * qq), out);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        // the first dequant warp also waits for the chunk's B box, so the
                        // MMA thread needs one barrier per chunk (Q6_K, whose dequant is
                        // the slower side, leaves that wait to the MMA thread)
                        if (kOneWait && dw == 0) mbar_wait(&b_full[s], (q / kStages) & 1, 3u, poisoned);
                        mbar_arrive(&a_full[s]);
                        if (p == 3) mbar_arrive(&raw_free[rs]);
                    }
                }
            } else if constexpr (TYPE == kTypeIQ4_XS) {
                // IQ4_XS (136 B: f16 d, u16 scales_h, 4 B of 4-bit scales_l, 128 B of
                // level indices): element 64p + 32h + 16qq + l of the block is sub-block
                // j = 2p + h, nibble qq of index byte 8 + 16j + l; w = d (ls_j - 32)
                // level. The block starts o = 136 kb mod 16 (0 or 8) bytes into its
                // 144-byte box row. The level enters as f16 1024 + (level + 128)
                // (an unsigned byte), minus 1152: the level exactly, times the f16
                // d (ls - 32).
                const uint8_t* rowp = raw + rs * kRawBytes + byte_row_slot<TYPE>(P, r) * 144;
                const int o = byte_row_off<TYPE>(P, kb0 + kb, r);
                const float d = __half2float(*reinterpret_cast<const __half*>(rowp + o));
                const uint32_t shb = *reinterpret_cast<const uint16_t*>(rowp + o + 2);
                const uint32_t slb = *reinterpret_cast<const uint32_t*>(rowp + o + 4);
                const int c8 = (o + 8) & 16, q48 = ((o + 8) & 15) >> 2;  // the indices start o + 8 bytes in
                const __half2 k1152 = __float2half2_rn(1152.f);
#pragma unroll
                for (int p = 0; p < 4; ++p, ++q) {
                    const int s = q % kStages;
                    if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    const int j = 2 * p + h;
                    const __half2 ds2 = __float2half2_rn(d * static_cast<float>(iq4xs_scale(shb, slb, j)));
                    const uint4 v = q6_load16(rowp, 16 * j + c8, q48, 0u);
                    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                    uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t u = iq4_lut4((wv[i] >> (4 * qq)) & 0x0F0F0F0Fu) ^ 0x80808080u;  // level + 128
                        const uint32_t e01 = __byte_perm(u, 0x00006464u, 0x5140u);
                        const uint32_t e23 = __byte_perm(u, 0x00006464u, 0x5342u);
                        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1152);
                        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1152);
                        const __half2 w01 = __hmul2(q01, ds2), w23 = __hmul2(q23, ds2);
                        out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                        out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                    }
                    tmem_st8(trow + static_cast<uint32_t>(kTileN + s * kACols + 16 * h + 8 * qq), out);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&a_full[s]);
                        if (p == 3) mbar_arrive(&raw_free[rs]);
                    }
                }
            } else if constexpr (TYPE == kTypeQ4_0) {
                // Q4_0: 8 blocks of 18 B (f16 d, 16 bytes of nibbles: elements
                // 0..15 low, 16..31 high) per 256 elements; this thread's 16
                // quants of chunk p are the low (qq = 0) or high nibbles of block
                // 2p + h, w = d (q - 8). The 16 bytes start 2 (2p + h) + 2 bytes
                // past a 16-byte boundary (warp-uniform)
                const uint8_t* rowp = raw + rs * kRawBytes + r * 144;
                const __half2 k1032 = __float2half2_rn(1032.f);
#pragma unroll
                for (int p = 0; p < 4; ++p, ++q) {
                    const int s = q % kStages;
                    if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    const int bo = 18 * (2 * p + h), a = bo + 2, o = a & 15;
                    const __half2 d2 = __half2half2(*reinterpret_cast<const __half*>(rowp + bo));
                    const uint4 v0 = q6_load16(rowp, a & ~15, o >> 2, 8u * static_cast<uint32_t>(o & 3));
                    const uint32_t wv[4] = {v0.x, v0.y, v0.z, v0.w};
                    uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        // f16 1024 + q (exact), minus 1032: q - 8 exactly
                        const uint32_t nib = (wv[i] >> (4 * qq)) & 0x0F0F0F0Fu;
                        const uint32_t e01 = __byte_perm(nib, 0x00006464u, 0x5140u);
                        const uint32_t e23 = __byte_perm(nib, 0x00006464u, 0x5342u);
                        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1032);
                        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1032);
                        const __half2 w01 = __hmul2(q01, d2), w23 = __hmul2(q23, d2);
                        out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                        out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                    }
                    tmem_st8(trow + static_cast<uint32_t>(kTileN + s * kACols + 16 * h + 8 * qq), out);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        // the first dequant warp also waits for the chunk's B box, so the
                        // MMA thread needs one barrier per chunk (Q6_K, whose dequant is
                        // the slower side, leaves that wait to the MMA thread)
                        if (kOneWait && dw == 0) mbar_wait(&b_full[s], (q / kStages) & 1, 3u, poisoned);
                        mbar_arrive(&a_full[s]);
                        if (p == 3) mbar_arrive(&raw_free[rs]);
                    }
                }
            } else if constexpr (TYPE == kTypeQ8_0) {
                // Q8_0: 8 blocks of 34 B (f16 d, 32 int8) per 256 elements; this
                // thread's 16 quants of chunk p are bytes 16qq .. +15 of block
                // 2p + h, w = d q. Their start is 2 (2p + h) + 2 bytes past a
                // 16-byte boundary (warp-uniform)
                const uint8_t* rowp = raw + rs * kRawBytes + r * 272;
                const __half2 k1152 = __float2half2_rn(1152.f);
#pragma unroll
                for (int p = 0; p < 4; ++p, ++q) {
                    const int s = q % kStages;
                    if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    const int bo = 34 * (2 * p + h), a = bo + 2 + 16 * qq, o = a & 15;
                    const __half2 d2 = __half2half2(*reinterpret_cast<const __half*>(rowp + bo));
                    const uint4 v0 = q6_load16(rowp, a & ~15, o >> 2, 8u * static_cast<uint32_t>(o & 3));
                    const uint32_t wv[4] = {v0.x, v0.y, v0.z, v0.w};
                    uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        // f16 1024 + (q + 128) (exact), minus 1152: q exactly
                        const uint32_t u = wv[i] ^ 0x80808080u;
                        const uint32_t e01 = __byte_perm(u, 0x00006464u, 0x5140u);
                        const uint32_t e23 = __byte_perm(u, 0x00006464u, 0x5342u);
                        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1152);
                        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1152);
                        const __half2 w01 = __hmul2(q01, d2), w23 = __hmul2(q23, d2);
                        out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                        out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                    }
                    tmem_st8(trow + static_cast<uint32_t>(kTileN + s * kACols + 16 * h + 8 * qq), out);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        // the first dequant warp also waits for the chunk's B box, so the
                        // MMA thread needs one barrier per chunk (Q6_K, whose dequant is
                        // the slower side, leaves that wait to the MMA thread)
                        if (kOneWait && dw == 0) mbar_wait(&b_full[s], (q / kStages) & 1, 3u, poisoned);
                        mbar_arrive(&a_full[s]);
                        if (p == 3) mbar_arrive(&raw_free[rs]);
                    }
                }
            } else {
                // Q4_K, and Q5_K (the same header; qh[32] @16, qs[128] @48; bit
                // 2p + h of qh byte 16qq + l is the fifth bit of the element)
                const uint8_t* blk = raw + rs * kRawBytes + r * raw_row_bytes<TYPE>();
                // scales of this thread's sub-blocks j = 2p + h (p = 0..3), get_scale_min_k4
                // (src/inference/jsep/ops/matmul.ts:408-424) on the bytes of the three scale words
                const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
                const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
                const uint32_t w1a = __byte_perm(hdr.y, 0u, sel_a), w1b = __byte_perm(hdr.y, 0u, sel_b);
                const uint32_t w2a = __byte_perm(hdr.z, 0u, sel_a), w2b = __byte_perm(hdr.z, 0u, sel_b);
                const uint32_t w3a = __byte_perm(hdr.w, 0u, sel_a), w3b = __byte_perm(hdr.w, 0u, sel_b);
                const uint32_t scv[4] = {w1a & 63u, w1b & 63u, (w3a & 15u) | ((w1a >> 6) << 4), (w3b & 15u) | ((w1b >> 6) << 4)};
                const uint32_t mv[4] = {w2a & 63u, w2b & 63u, (w3a >> 4) | ((w2a >> 6) << 4), (w3b >> 4) | ((w2b >> 6) << 4)};
                const uint4* qs = reinterpret_cast<const uint4*>(blk + (TYPE == kTypeQ5_K ? 48 : 16));
                uint4 qh = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (TYPE == kTypeQ5_K) qh = *reinterpret_cast<const uint4*>(blk + 16 + 16 * qq);
                const uint32_t hv[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
                for (int p = 0; p < 4; ++p, ++q) {
                    const int s = q % kStages;
                    if (q >= kStages && !mbar_wait(&st_free[s], ((q / kStages) - 1) & 1, 3u, poisoned)) {
                        stop = true;
                        break;
                    }
                    const __half2 sc2 = __float2half2_rn(d * static_cast<float>(scv[p]));
                    const __half2 mn2 = __float2half2_rn(-dmin * static_cast<float>(mv[p]));
                    // bytes 16 qq .. 16 qq + 15 of pair p; this thread's quants are their low
                    // (h = 0) or high (h = 1) nibbles: elements 64p + 32h + 16qq + l, l = 0..15
                    const uint4 v0 = qs[2 * p + qq];
                    const uint32_t wv[4] = {v0.x, v0.y, v0.z, v0.w};
                    uint32_t out[8];  // 16 f16, element order l = 0..15
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t nib = (wv[i] >> (4 * h)) & 0x0F0F0F0Fu;
                        if constexpr (TYPE == kTypeQ5_K) nib |= ((hv[i] >> (2 * p + h)) & 0x01010101u) << 4;
                        // f16 1024 + q (exact) for bytes (0, 1) and (2, 3): 0x64 in each high byte
                        const uint32_t e01 = __byte_perm(nib, 0x00006464u, 0x5140u);
                        const uint32_t e23 = __byte_perm(nib, 0x00006464u, 0x5342u);
                        const __half2 q01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1024);
                        const __half2 q23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1024);
                        const __half2 w01 = __hfma2(q01, sc2, mn2), w23 = __hfma2(q23, sc2, mn2);
                        out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                        out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                    }
                    // k = 32h + 16qq + l of this chunk: TMEM columns 16h + 8qq .. +7 of A stage s
                    tmem_st8(trow + static_cast<uint32_t>(kTileN + s * kACols + 16 * h + 8 * qq), out);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        // the first dequant warp also waits for the chunk's B box, so the
                        // MMA thread needs one barrier per chunk (Q6_K, whose dequant is
                        // the slower side, leaves that wait to the MMA thread)
                        if (kOneWait && dw == 0) mbar_wait(&b_full[s], (q / kStages) & 1, 3u, poisoned);
                        mbar_arrive(&a_full[s]);
                        if (p == 3) mbar_arrive(&raw_free[rs]);
                    }
                }
            }
        }
        // ---------------- epilogue ----------------
        const bool ok = mbar_wait(acc_full, 0, 4u, poisoned);
        tc_fence_after();
        const int col0 = part * (kTileN / 4);  // the 4 warps of a lane quarter split the columns
        const int tr = 32 * quarter + lane, row = m0 + tr;
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        float* ptile = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kTileM * kTileN);
        if (ok) {
#pragma unroll 1
            for (int cc = 0; cc < kTileN / 4; cc += 16) {
                float v[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(32 * quarter) << 16) + static_cast<uint32_t>(col0 + cc), v);
                if (P.splits > 1) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) ptile[(col0 + cc + i) * kTileM + tr] = v[i];  // [col][row]
                } else if (row < P.M) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int n = n0 + col0 + cc + i;
                        if (n < P.N)
                            *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * row) = v[i];
                    }
                }
            }
        }
        // a split that gave up waiting did not write its partial tile: it marks
        // the tile (the marks are zeroed by the pre-pass), and nobody sums it
        if (P.splits > 1 && dw == 0 && lane == 0 && *poisoned) atomicOr(P.counters + blockIdx.y * gridDim.x + blockIdx.x, 1u);
    }
    tc_fence_before();
    __syncthreads();
    if (P.splits > 1) {
        // The S splits of a tile are one cluster (grid z): after the cluster
        // barrier every partial tile is written, and each split sums its own
        // slice of the tile's columns over the S partial tiles, in split order
        // (deterministic), so the reduction runs on S SMs at once.
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (warp >= 2 && __ldcg(P.counters + tile) == 0u) {
            // thread t sums rows 4 (t % 32) .. +3 of slice columns t / 32 + 16 j
            const int t = threadIdx.x - 64, r4 = 4 * (t & 31), cb = t >> 5;
            const int w = (kTileN + P.splits - 1) / P.splits, c0 = blockIdx.z * w, c1 = min(kTileN, c0 + w);
            const float4* base =
                reinterpret_cast<const float4*>(P.partial + static_cast<int64_t>(tile) * P.splits * (kTileM * kTileN));
            constexpr int kJ = kTileN / 2 / 16;  // slice columns per thread at S >= 2
            float4 acc[kJ];
#pragma unroll
            for (int j = 0; j < kJ; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int z = 0; z < P.splits; ++z) {
                float4 v[kJ];
#pragma unroll
                for (int j = 0; j < kJ; ++j) {
                    const int col = c0 + cb + 16 * j;
                    v[j] = col < c1 ? __ldcg(base + (z * kTileN + col) * (kTileM / 4) + (r4 >> 2))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < kJ; ++j) {
                    acc[j].x += v[j].x;
                    acc[j].y += v[j].y;
                    acc[j].z += v[j].z;
                    acc[j].w += v[j].w;
                }
            }
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int col = c0 + cb + 16 * j, n = n0 + col, r = m0 + r4;
                if (col >= c1 || n >= P.N) continue;
                float* yn = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1);
                const float av[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (r + i < P.M) yn[r + i] = av[i];
            }
        }
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// f32 activations [N][K] (vector stride x_nb1 bytes) -> contiguous f16 [N][K].
// Vectors blockIdx.y, blockIdx.y + gridDim.y, ..., elements 4 (blockIdx.x
// blockDim.x + t) .. +3 (and their grid-stride successors); a thread loads
// eight vectors' float4s before it converts and stores them, so enough loads
// are in flight to stream at the HBM rate (one at a time it ran at about half
// of it). CTA (0, 0) also zeroes the split-K tile counters. The GEMM that
// follows may start at once: its prologue and first weight boxes overlap this
// kernel, and it waits for the f16 image with griddepcontrol.wait.
__global__ void x_to_f16_kernel(const float* __restrict__ x, int64_t x_nb1, __half* __restrict__ x16, int K, int N,
                                unsigned* __restrict__ counters, int ncounters) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int t = threadIdx.x; t < ncounters; t += blockDim.x) counters[t] = 0u;
    constexpr int kRows = 8;
    const int k4n = K / 4;
    for (int k4 = blockIdx.x * blockDim.x + threadIdx.x; k4 < k4n; k4 += gridDim.x * blockDim.x) {
        for (int n0 = blockIdx.y; n0 < N; n0 += kRows * gridDim.y) {
            float4 v[kRows];
#pragma unroll
            for (int i = 0; i < kRows; ++i) {
                const int n = n0 + i * gridDim.y;
                if (n < N)
                    v[i] = reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(x) + n * x_nb1)[k4];
            }
#pragma unroll
            for (int i = 0; i < kRows; ++i) {
                const int n = n0 + i * gridDim.y;
                if (n < N) {
                    __half2* orow = reinterpret_cast<__half2*>(x16 + static_cast<int64_t>(n) * K);
                    orow[2 * k4] = __floats2half2_rn(v[i].x, v[i].y);
                    orow[2 * k4 + 1] = __floats2half2_rn(v[i].z, v[i].w);
                }
            }
        }
    }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
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

template <int TYPE>
constexpr size_t smem_bytes() {
    return 1024 /* alignment */ + kStages * kBBytes + kRawSlots * raw_bytes<TYPE>() + 8 * (3 * kStages + 2 * kRawSlots + 1) +
           16;
}
static_assert(smem_bytes<kTypeQ8_0>() <= 227 * 1024 && smem_bytes<kTypeQ6_K>() <= 227 * 1024, "shared memory");
constexpr int kSlots = 148;  // CTAs resident at once (one per SM)
constexpr int kMaxSplits = 8;

// K splits per tile, only while the grid stays within one wave of resident
// CTAs (a split grid past that adds partial-tile traffic without adding
// parallelism): minimises the K blocks per CTA plus the final reduction
// (about 0.65 K blocks' time per split summed).
int plan_splits(const MulMatOp& o) {
    const int tiles = ((o.M + kTileM - 1) / kTileM) * ((o.N + kTileN - 1) / kTileN);
    const int nblk = o.K / 256;
    int best = 1;
    double best_cost = 1e30;
    for (int S = 1; S <= kMaxSplits && S <= nblk && (S == 1 || tiles * S <= kSlots); ++S) {
        const int kb = (nblk + S - 1) / S;
        if (S > 1 && (nblk + kb - 1) / kb < S) continue;  // a split would be empty
        const int waves = (tiles * S + kSlots - 1) / kSlots;
        // a split costs its partial tile's write and its slice's reduction, and
        // clusters of many splits place less freely (S = 8 measured slower than
        // S = 4 at 1024 x 4096 with this term at 1.3)
        const double cost = static_cast<double>(waves) * kb + (S > 1 ? 0.65 * S : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = S;
        }
    }
    return best;
}

// log2 of the row group a byte-mapped op's rows are copied in: 0 for rows a
// multiple of 16 bytes apart; Q6_K / IQ4_XS rows 8 mod 16 bytes apart in
// pairs; Q6_K rows 4 or 12 mod 16 apart in fours, 2 mod 4 in eights (G w_nb1
// a multiple of 16); M a multiple of G; -1 where no group fits. (An IQ4_XS
// block must start at most 8 bytes into its 144-byte box row.)
int row_group_lg(const MulMatOp& o) {
    const int m = static_cast<int>(o.w_nb1 & 15);
    if (m == 0) return 0;
    if (o.w_nb1 >= (int64_t(1) << 26)) return -1;
    int lg = -1;
    if (o.type == kTypeQ6_K && !(m & 1)) lg = m == 8 ? 1 : ((m & 3) == 0 ? 2 : 3);
    if (o.type == kTypeIQ4_XS && m == 8) lg = 1;
    return lg > 0 && o.M % (1 << lg) == 0 ? lg : -1;
}

// Bytes of 256 elements of a row: Q4_K 144, Q5_K 176, Q6_K 210, Q8_0 272, Q4_0 144.
int block_group_bytes(int type) {
    return type == kTypeQ6_K ? 210
                             : (type == kTypeQ5_K ? 176 : (type == kTypeQ8_0 ? 272 : (type == kTypeIQ4_XS ? 136 : 144)));
}

size_t x16_bytes(const MulMatOp& o) { return (static_cast<size_t>(o.N) * o.K * 2 + 255) & ~size_t(255); }
size_t split_bytes(const MulMatOp& o, int splits) {
    if (splits <= 1) return 0;
    const size_t tiles = static_cast<size_t>((o.M + kTileM - 1) / kTileM) * ((o.N + kTileN - 1) / kTileN);
    return tiles * splits * kTileM * kTileN * 4 + tiles * 4;
}

}  // namespace

bool prefill_supported(const MulMatOp& o) {
    if ((o.type != kTypeQ4_K && o.type != kTypeQ5_K && o.type != kTypeQ6_K && o.type != kTypeQ8_0 &&
         o.type != kTypeQ4_0 && o.type != kTypeIQ4_XS) ||
        o.N < kPrefillMinN || o.ne2 != 1 || o.ne3 != 1)
        return false;
    if (o.K % 256 != 0 || o.M < 1) return false;
    const int64_t row_bytes = static_cast<int64_t>(o.K / 256) * block_group_bytes(o.type);
    // TMA rows: 16-byte aligned base and row stride, or (Q6_K, IQ4_XS) rows of
    // an even stride in groups of 2, 4 or 8 (Q6_K K = 1024 (mod 2048) in pairs,
    // K = 256 (mod 512) in eights, unpadded) when M is a multiple of the group
    if ((reinterpret_cast<uintptr_t>(o.w) & 15) || row_group_lg(o) < 0) return false;
    if (o.w_nb1 < row_bytes) return false;
    if (o.type == kTypeQ6_K && row_bytes < kQ6Box) return false;  // the box stays within a row's width
    if (o.type == kTypeIQ4_XS && row_bytes < 144) return false;
    if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;  // float4 reads
    return encoder() != nullptr;
}

size_t prefill_workspace_bytes(const MulMatOp& o) { return x16_bytes(o) + split_bytes(o, plan_splits(o)) + 256; }
size_t prefill_min_workspace_bytes(const MulMatOp& o) { return x16_bytes(o) + 256; }

int launch_prefill(const MulMatOp& o, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!prefill_supported(o)) return -static_cast<int>(cudaErrorInvalidValue);
    if (!workspace || workspace_bytes < prefill_min_workspace_bytes(o) || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return -static_cast<int>(cudaErrorInvalidValue);
    // split K when the workspace holds the partial tiles (else one split)
    int splits = plan_splits(o);
    if (x16_bytes(o) + split_bytes(o, splits) > workspace_bytes) splits = 1;
    const int nblk = o.K / 256, kb_split = (nblk + splits - 1) / splits;
    __half* x16 = static_cast<__half*>(workspace);
    PrefillArgs P{};
    const EncodeFn enc = encoder();
    const bool q6 = o.type == kTypeQ6_K, iq4 = o.type == kTypeIQ4_XS, bytemap = q6 || iq4;
    {
        // Q4_K / Q5_K / Q8_0 / Q4_0: uint64 words, one 256-element column per
        // box (18 / 22 / 34 / 18 words); Q6_K and IQ4_XS: bytes, a 240- or
        // 144-byte box from the block's 16-byte-rounded start (the box's end may
        // pass the row's last block: zeros, never read)
        const cuuint64_t group = static_cast<cuuint64_t>(block_group_bytes(o.type));
        const int lg = row_group_lg(o);
        // row groups: [M / G][G w_nb1 bytes], row j of a group from j w_nb1 on
        const cuuint64_t dims[2] = {lg ? static_cast<cuuint64_t>(o.w_nb1) << lg
                                       : static_cast<cuuint64_t>(o.K / 256) * (bytemap ? group : group / 8),
                                    static_cast<cuuint64_t>(o.M >> lg)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.w_nb1) << lg};
        const cuuint32_t box[2] = {q6 ? static_cast<cuuint32_t>(kQ6Box) : (iq4 ? 144u : static_cast<cuuint32_t>(group / 8)),
                                   static_cast<cuuint32_t>(kTileM >> lg)};
        P.row_lg = lg;
        P.w_nb1 = static_cast<int32_t>(o.w_nb1);
        const cuuint32_t es[2] = {1, 1};
        if (enc(&P.wmap, bytemap ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(o.w),
                dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(o.K), static_cast<cuuint64_t>(o.N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.K) * 2};
        const cuuint32_t box[2] = {kChunkK, kTileN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    P.y = o.y;
    P.y_nb1 = o.y_nb1;
    P.M = o.M;
    P.K = o.K;
    P.N = o.N;
    P.splits = splits;
    P.kb_split = kb_split;
    int launched = 2;
    size_t tiles = 0;
    if (splits > 1) {
        tiles = static_cast<size_t>((o.M + kTileM - 1) / kTileM) * ((o.N + kTileN - 1) / kTileN);
        P.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + x16_bytes(o));
        P.counters = reinterpret_cast<unsigned*>(P.partial + tiles * splits * kTileM * kTileN);
    }
    {
        // the f16 activation image (and the split counters), then the GEMM
        // at most about four CTAs per SM, so that every CTA of the pre-pass is
        // running (and has released the GEMM) at once: the GEMM's launch waits
        // for all of them to execute griddepcontrol.launch_dependents
        const int threads = 256, per_row = (o.K / 4 + threads - 1) / threads;
        const int rows = std::max(1, std::min(o.N, 4 * kSlots / per_row));
        x_to_f16_kernel<<<dim3(per_row, rows), threads, 0, stream>>>(o.x, o.x_nb1, x16, o.K, o.N, P.counters,
                                                                    static_cast<int>(tiles));
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return -static_cast<int>(e);
    }
    // the attribute is per device: one flag per device ordinal and kernel
    static bool configured[kMaxDevices][6] = {};
    int dev = 0;
    if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return -static_cast<int>(e);
    if (dev < 0 || dev >= kMaxDevices) return -static_cast<int>(cudaErrorInvalidDevice);
    const int ti = o.type == kTypeQ4_K    ? 0
                   : o.type == kTypeQ5_K  ? 1
                   : q6                   ? 2
                   : o.type == kTypeQ8_0  ? 3
                   : o.type == kTypeQ4_0  ? 4
                                          : 5;
    void (*const kernels[6])(PrefillArgs) = {prefill_kernel<kTypeQ4_K>, prefill_kernel<kTypeQ5_K>,
                                             prefill_kernel<kTypeQ6_K>, prefill_kernel<kTypeQ8_0>,
                                             prefill_kernel<kTypeQ4_0>, prefill_kernel<kTypeIQ4_XS>};
    const size_t smems[6] = {smem_bytes<kTypeQ4_K>(), smem_bytes<kTypeQ5_K>(), smem_bytes<kTypeQ6_K>(),
                             smem_bytes<kTypeQ8_0>(), smem_bytes<kTypeQ4_0>(), smem_bytes<kTypeIQ4_XS>()};
    void (*const kernel)(PrefillArgs) = kernels[ti];
    const size_t smem = smems[ti];
    if (!configured[dev][ti]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return -static_cast<int>(e);
        configured[dev][ti] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((o.M + kTileM - 1) / kTileM, (o.N + kTileN - 1) / kTileN, splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    // a tile's splits are one cluster, for the barrier before their reduction
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = static_cast<unsigned>(splits);
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, P);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? launched : -static_cast<int>(e);
}

// Fixed device workspace for wllm_mul_mat_prefill_static: the f16 copy of the
// activations (N x K x 2 bytes) lives in this file-scope array instead of
// runtime-allocated memory. Nothing in it needs to start at zero: the
// activation pre-pass writes every byte the GEMM reads. Calls that use it at
// the same time (several streams or host threads) race on it.
static __device__ __align__(256) unsigned char g_prefill_static_ws[kPrefillStaticWorkspaceBytes];

void* prefill_static_workspace(const char** err) {
    // the array's device address, looked up once per device (the lookup must
    // not happen while a stream is being captured)
    static void* addr[kMaxDevices] = {};
    static bool looked_up[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        *err = "cannot query the current device";
        return nullptr;
    }
    if (!looked_up[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_prefill_static_ws);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            *err = "cudaGetSymbolAddress of the static workspace failed";
            return nullptr;
        }
        addr[dev] = p;
        looked_up[dev] = true;
    }
    return addr[dev];
}

unsigned read_and_clear_prefill_error() {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_prefill_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_prefill_error, &z, sizeof(z));
    }
    return v;
}

}  // namespace wllm
