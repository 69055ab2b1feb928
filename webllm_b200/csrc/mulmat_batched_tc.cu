// Small-batch quantized MUL_MAT on tcgen05 tensor cores for Q4_K and Q5_K
// weights (several sequences decoding together: N up to 64 vectors), exact to
// about 2^-22 of every activation element, like the integer decode kernels.
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
//  - activations: per vector a power-of-two scale 2^e (its maximum lands in
//    [2^14, 2^15)) and two f16 parts, hi = f16(x 2^-e), lo = f16(x 2^-e - hi),
//    about 22 bits of each element whatever its neighbours (an outlier channel
//    costs nothing); hi and lo are stacked along K, so the main MMA sums
//    A (hi + lo) into one accumulator column per vector;
//  - the mins: A_min = (m_0 .. m_7, m_0 .. m_7) (K = 16) against the sub-block
//    sums split the same way (scale 2^(e + 5)), one MMA per block.
// A pre-pass (btc_prep_kernel) writes the activation image [hi | lo][np][K],
// the sums image [block][np][64] and the per-vector scales into workspace.
//
// CTA: 128 rows x np vectors (np = N rounded up to 16, at most 64).
//  - warp 0 (TMA): per block, one 2D box of the 128 rows' raw blocks and the
//    block's sums box into a raw slot; per 64-element chunk, the hi and lo
//    boxes of the activations (128-byte swizzle) into a B stage;
//  - warp 1: TMEM allocation; one thread issues per chunk 8 MMAs (4 K-steps x
//    hi, lo; A from TMEM) into the block's accumulator, per block the mins MMA,
//    and commits them;
//  - warps 2..17: dequantize A = sc q straight into TMEM (tcgen05.st), as the
//    prefill GEMM does, write A_min, and run the previous block's epilogue
//    (tcgen05.ld of its two accumulators, y += d s_n main - dmin s'_n mins).
// Accumulators are double-buffered by block parity, so the MMAs of block b
// overlap the epilogue of block b - 1. Split K as in the prefill GEMM.
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

constexpr int kTM = 128;                  // rows of W per CTA (TMEM lanes)
constexpr int kMaxNP = 64;                // vectors per CTA
constexpr int kChunk = 64;                // K per stage (one 128-byte swizzle atom of f16)
constexpr int kSt = 4;                    // A (TMEM) and B (shared) stages
constexpr int kRaw = 4;                   // raw blocks in flight
constexpr int kDq = 16;                   // dequant / epilogue warps
constexpr int kThr = 32 * (2 + kDq);
constexpr int kACol0 = 256, kACols = 32;  // A stage s: TMEM columns 256 + 32 s (two f16 per column)
constexpr int kMinCol0 = 384;             // A_min of block parity p: columns 384 + 8 p
constexpr int kTmemCols = 512;            // accumulators: block parity p at columns 2 np p (main) and + np (mins)
constexpr uint32_t kSpin = 1u << 26;
constexpr int kMaxSplits = 16;

struct BtcArgs {
    CUtensorMap wmap;     // weights [M][row bytes / 8] uint64, box (block bytes / 8) x 128
    CUtensorMap xmap;     // activations [2 np][K] f16 (rows 0..np-1 hi, np.. lo), box 64 x np, 128-byte swizzle
    CUtensorMap smap;     // sub-block sums [blocks x np][64] f16 (k 0..7 hi, 8..15 lo, rest 0), box 64 x np
    const float* vscale;  // [2][np]: 2^e_n (activations), 2^(e_n + 5) (sums)
    float* y;
    int64_t y_nb1;        // bytes between output vectors
    int32_t M, K, N, np;
    int32_t splits, kb_split;
    float* partial;       // [tile][split][np][128] (split K)
    unsigned* counters;   // [tile] (split K, zero at launch)
};

template <int TYPE>
__host__ __device__ constexpr int blk_bytes() {
    return TYPE == kTypeQ5_K ? 176 : 144;
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
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned) {
    for (uint32_t i = 0; i < kSpin; ++i) {
        if (mbar_try(bar, parity)) return true;
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
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
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
// 8 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
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

// Shared-memory layout (from a 1024-byte aligned base): B stages, sums slots,
// raw slots, barriers.
struct Smem {
    uint32_t b_bytes, s_bytes, raw_bytes;
    __host__ __device__ Smem(int np, int bb) {
        b_bytes = static_cast<uint32_t>(2 * np * 128);  // hi + lo boxes of one chunk
        s_bytes = static_cast<uint32_t>(np * 128);
        raw_bytes = static_cast<uint32_t>(kTM * bb);
    }
    __host__ __device__ uint32_t b_off(int s) const { return s * b_bytes; }
    __host__ __device__ uint32_t s_off(int r) const { return kSt * b_bytes + r * s_bytes; }
    __host__ __device__ uint32_t raw_off(int r) const { return kSt * b_bytes + kRaw * s_bytes + r * raw_bytes; }
    __host__ __device__ uint32_t bar_off() const { return (kSt * b_bytes + kRaw * s_bytes + kRaw * raw_bytes + 7) & ~7u; }
    // barriers: b_full[kSt], a_full[kSt], st_free[kSt], raw_full[kRaw], raw_free[kRaw], amin_full[2],
    // acc_full[2], acc_free[2]; then the TMEM base address word, the poison flag and 2 np scales
    __host__ __device__ uint32_t total(int np) const {
        return bar_off() + 8 * (3 * kSt + 2 * kRaw + 6) + 16 + 8 * np + 1024;  // + alignment slack
    }
};

template <int TYPE>
__global__ void __launch_bounds__(kThr, 1) btc_kernel(const __grid_constant__ BtcArgs P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int BB = blk_bytes<TYPE>();
    const int np = P.np;
    const Smem L(np, BB);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off());
    uint64_t* b_full = bars;
    uint64_t* a_full = b_full + kSt;
    uint64_t* st_free = a_full + kSt;
    uint64_t* raw_full = st_free + kSt;
    uint64_t* raw_free = raw_full + kRaw;
    uint64_t* amin_full = raw_free + kRaw;
    uint64_t* acc_full = amin_full + 2;
    uint64_t* acc_free = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_free + 2);
    volatile int* poisoned = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* vs = reinterpret_cast<float*>(tmem_slot + 4);  // [2][np]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTM;
    const int kb0 = blockIdx.z * P.kb_split;  // first K block of this split
    const int nblk = min(P.K / 256 - kb0, P.kb_split);
    const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(np >> 3) << 17) | (static_cast<uint32_t>(kTM >> 4) << 24);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSt; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&a_full[s], kDq);
            mbar_init(&st_free[s], 1);
        }
        for (int r = 0; r < kRaw; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_free[r], kDq + 1);  // the dequant warps and the mins MMA's commit
        }
        for (int p = 0; p < 2; ++p) {
            mbar_init(&amin_full[p], 4);  // one warp per TMEM lane quarter
            mbar_init(&acc_full[p], 1);
            mbar_init(&acc_free[p], kDq);
        }
        *poisoned = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < 2 * np; i += kThr) vs[i] = P.vscale[i];
    if (warp == 1) {
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
            asm volatile("prefetch.tensormap [%0];" ::"l"(&P.smap) : "memory");
            int raw_issued = 0, b_issued = 0;
            bool stop = false;
            for (int b = 0; b < nblk && !stop; ++b) {
                const int r = b % kRaw;
                if (b >= kRaw && !mbar_wait(&raw_free[r], ((b / kRaw) - 1) & 1, 1u, poisoned)) break;
                mbar_expect_tx(&raw_full[r], L.raw_bytes + L.s_bytes);
                tma_2d(smem + L.raw_off(r), &P.wmap, (kb0 + b) * (BB / 8), m0, &raw_full[r]);
                tma_2d(smem + L.s_off(r), &P.smap, 0, (kb0 + b) * np, &raw_full[r]);
                raw_issued = b + 1;
                for (int c = 0; c < 4; ++c) {
                    const int q = 4 * b + c, s = q % kSt;
                    if (q >= kSt && !mbar_wait(&st_free[s], ((q / kSt) - 1) & 1, 1u, poisoned)) {
                        stop = true;
                        break;
                    }
                    mbar_expect_tx(&b_full[s], L.b_bytes);
                    const int kx = (kb0 + b) * 256 + kChunk * c;
                    tma_2d(smem + L.b_off(s), &P.xmap, kx, 0, &b_full[s]);
                    tma_2d(smem + L.b_off(s) + L.b_bytes / 2, &P.xmap, kx, np, &b_full[s]);
                    b_issued = q + 1;
                }
            }
            // before the CTA exits, the last copy into every slot and stage has
            // landed (bounded, whatever the poison flag says)
            for (int b = max(0, raw_issued - kRaw); b < raw_issued; ++b)
                if (!mbar_wait_drain(&raw_full[b % kRaw], (b / kRaw) & 1)) atomicOr(&g_btc_error, 16u);
            for (int q = max(0, b_issued - kSt); q < b_issued; ++q)
                if (!mbar_wait_drain(&b_full[q % kSt], (q / kSt) & 1)) atomicOr(&g_btc_error, 16u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int committed = 0;  // chunks committed (for the drain after a time-out)
        bool stop = false;
        for (int b = 0; b < nblk && !stop; ++b) {
            const int buf = b & 1;
            const uint32_t dmain = tmem + static_cast<uint32_t>(2 * np * buf), dmin = dmain + static_cast<uint32_t>(np);
            int ok = 1;
            if (lane == 0 && b >= 2) ok = mbar_wait(&acc_free[buf], ((b / 2) - 1) & 1, 2u, poisoned);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            for (int c = 0; c < 4; ++c) {
                const int q = 4 * b + c, s = q % kSt;
                const uint32_t par = (q / kSt) & 1;
                ok = 1;
                if (lane == 0) ok = mbar_wait(&b_full[s], par, 2u, poisoned) && mbar_wait(&a_full[s], par, 2u, poisoned);
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    stop = true;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a0 = tmem + static_cast<uint32_t>(kACol0 + s * kACols);
                    const uint32_t bhi = smem_u32(smem + L.b_off(s)), blo = bhi + L.b_bytes / 2;
#pragma unroll
                    for (int ks = 0; ks < kChunk / 16; ++ks) {  // K = 16 per MMA: 8 A columns, 32 bytes of B rows
                        umma_f16_ts(dmain, a0 + 8 * ks, umma_desc_sw128(bhi + 32 * ks), idesc, (c | ks) ? 1u : 0u);
                        umma_f16_ts(dmain, a0 + 8 * ks, umma_desc_sw128(blo + 32 * ks), idesc, 1u);
                    }
                    umma_commit(&st_free[s]);  // A and B stage s are free once these have read them
                }
                committed = q + 1;
                __syncwarp();
            }
            if (stop) break;
            // the mins: A_min (K = 16) against the block's sums box
            const int r = b % kRaw;
            ok = 1;
            if (lane == 0)
                ok = mbar_wait(&raw_full[r], (b / kRaw) & 1, 2u, poisoned) &&
                     mbar_wait(&amin_full[buf], (b / 2) & 1, 2u, poisoned);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            if (lane == 0) {
                umma_f16_ts(dmin, tmem + static_cast<uint32_t>(kMinCol0 + 8 * buf), umma_desc_sw128(smem_u32(smem + L.s_off(r))),
                            idesc, 0u);
                umma_commit(&raw_free[r]);  // the sums box is read
                umma_commit(&acc_full[buf]);
            }
            __syncwarp();
        }
        if (*poisoned) {
            // a time-out: the MMAs already issued still write TMEM, which is freed
            // at the end; wait (bounded) for the last commit, which tracks them all
            if (lane == 0 && committed > 0 &&
                !mbar_wait_drain(&st_free[(committed - 1) % kSt], ((committed - 1) / kSt) & 1))
                atomicOr(&g_btc_error, 16u);
            __syncwarp();
        }
    } else {
        // ---------------- dequant, A_min and epilogue ----------------
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int dw = warp - 2;
        const int part = dw >> 2;      // quarter of each chunk's K; quarter of the vectors in the epilogue
        const int r = 32 * quarter + lane, h = part >> 1, qq = part & 1;  // row; sub-block 2p + h, its half qq
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
        const uint32_t sel_a = 0x4440u + static_cast<uint32_t>(h);      // byte h, zero-extended
        const uint32_t sel_b = 0x4440u + 2u + static_cast<uint32_t>(h);  // byte 2 + h
        const int nq = np / 4, n0 = part * nq;  // this warp's vectors in the epilogue
        float yacc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) yacc[i] = 0.f;
        float dprev = 0.f, dminprev = 0.f;
        bool stop = false;
        // the epilogue of block pb: y += d s_n main - dmin s'_n mins
        auto epilogue = [&](int pb, float d, float dm) {
            const int pbuf = pb & 1;
            const bool ok = mbar_wait(&acc_full[pbuf], (pb / 2) & 1, 4u, poisoned);
            tc_fence_after();
            if (ok) {
                float mv[16], nv[16];
                tmem_ld16(trow + static_cast<uint32_t>(2 * np * pbuf + n0), mv);
                tmem_ld16(trow + static_cast<uint32_t>(2 * np * pbuf + np + n0), nv);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    if (i < nq)
                        yacc[i] = fmaf(mv[i], d * vs[n0 + i], fmaf(-nv[i], dm * vs[np + n0 + i], yacc[i]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[pbuf]);
            return ok;
        };
        int q = 0;
        for (int b = 0; b < nblk && !stop; ++b) {
            const int rs = b % kRaw, buf = b & 1;
            if (!mbar_wait(&raw_full[rs], (b / kRaw) & 1, 3u, poisoned)) break;
            const uint8_t* blk = smem + L.raw_off(rs) + r * BB;
            // scales of this thread's sub-blocks j = 2p + h (p = 0..3), get_scale_min_k4
            // (src/inference/jsep/ops/matmul.ts:408-424) on the bytes of the three scale words
            const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
            const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
            const uint32_t w1a = __byte_perm(hdr.y, 0u, sel_a), w1b = __byte_perm(hdr.y, 0u, sel_b);
            const uint32_t w3a = __byte_perm(hdr.w, 0u, sel_a), w3b = __byte_perm(hdr.w, 0u, sel_b);
            const uint32_t scv[4] = {w1a & 63u, w1b & 63u, (w3a & 15u) | ((w1a >> 6) << 4),
                                     (w3b & 15u) | ((w1b >> 6) << 4)};
            const uint4* qs = reinterpret_cast<const uint4*>(blk + (TYPE == kTypeQ5_K ? 48 : 16));
            uint4 qh = make_uint4(0u, 0u, 0u, 0u);
            if constexpr (TYPE == kTypeQ5_K) qh = *reinterpret_cast<const uint4*>(blk + 16 + 16 * qq);
            const uint32_t hv[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
            for (int p = 0; p < 4; ++p, ++q) {
                const int s = q % kSt;
                if (q >= kSt && !mbar_wait(&st_free[s], ((q / kSt) - 1) & 1, 3u, poisoned)) {
                    stop = true;
                    break;
                }
                // A = sc q exactly: (1024 + q) sc - 1024 sc in one f16 FMA (the
                // exact result, at most 1953, is an f16 integer)
                const float scf = static_cast<float>(scv[p]);
                const __half2 sc2 = __float2half2_rn(scf), mn2 = __float2half2_rn(-1024.f * scf);
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
                    const __half2 w01 = __hfma2(*reinterpret_cast<const __half2*>(&e01), sc2, mn2);
                    const __half2 w23 = __hfma2(*reinterpret_cast<const __half2*>(&e23), sc2, mn2);
                    out[2 * i] = *reinterpret_cast<const uint32_t*>(&w01);
                    out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&w23);
                }
                // k = 32h + 16qq + l of this chunk: TMEM columns 16h + 8qq .. +7 of A stage s
                tmem_st8(trow + static_cast<uint32_t>(kACol0 + s * kACols + 16 * h + 8 * qq), out);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[s]);
            }
            if (stop) break;
            if (part == 0) {
                // A_min of this block: the eight 6-bit mins (get_scale_min_k4), twice,
                // as f16 pairs (k 0..7 meet the sums' hi parts, 8..15 their lo parts).
                // Block b - 2's mins MMA, which read these columns, is complete: this
                // warp waited for its accumulator in the previous epilogue.
                const uint32_t mv0 = hdr.z & 0x3F3F3F3Fu;  // m_0..m_3 (bytes 8..11, low 6 bits)
                uint32_t mm[4];
                const uint32_t mhi = (((hdr.w >> 4) & 0x0F0F0F0Fu)) | (((hdr.z >> 6) & 0x03030303u) << 4);  // m_4..m_7
                const uint32_t mq[2] = {mv0, mhi};
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const uint32_t e01 = __byte_perm(mq[t], 0x00006464u, 0x5140u);
                    const uint32_t e23 = __byte_perm(mq[t], 0x00006464u, 0x5342u);
                    const __half2 k1024 = __float2half2_rn(1024.f);
                    const __half2 m01 = __hsub2(*reinterpret_cast<const __half2*>(&e01), k1024);
                    const __half2 m23 = __hsub2(*reinterpret_cast<const __half2*>(&e23), k1024);
                    mm[2 * t] = *reinterpret_cast<const uint32_t*>(&m01);
                    mm[2 * t + 1] = *reinterpret_cast<const uint32_t*>(&m23);
                }
                const uint32_t amin[8] = {mm[0], mm[1], mm[2], mm[3], mm[0], mm[1], mm[2], mm[3]};
                tmem_st8(trow + static_cast<uint32_t>(kMinCol0 + 8 * buf), amin);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&amin_full[buf]);
            }
            if (lane == 0) mbar_arrive(&raw_free[rs]);
            if (b >= 1 && !epilogue(b - 1, dprev, dminprev)) {
                stop = true;
                break;
            }
            dprev = d;
            dminprev = dmin;
        }
        if (!stop && nblk > 0) epilogue(nblk - 1, dprev, dminprev);
        // ---------------- outputs ----------------
        const int row = m0 + r;
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (P.splits == 1) {
            if (row < P.M) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = n0 + i;
                    if (i < nq && n < P.N)
                        *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * row) = yacc[i];
                }
            }
        } else {
            float* ptile = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kMaxNP * kTM);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < nq) ptile[(n0 + i) * kTM + r] = yacc[i];
            // the tile's last split sums all of them in split order (deterministic);
            // a split that gave up waiting counts in the high half and nobody sums
            __shared__ int last;
            asm volatile("bar.sync 1, %0;" ::"n"(kDq * 32) : "memory");
            if (threadIdx.x == 64) {
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
            asm volatile("bar.sync 1, %0;" ::"n"(kDq * 32) : "memory");
            if (last) {
                const float* base = P.partial + static_cast<int64_t>(tile) * P.splits * (kMaxNP * kTM);
                for (int i = threadIdx.x - 64; i < np * kTM; i += kDq * 32) {
                    const int n = i / kTM, rr = i - n * kTM;
                    float acc = 0.f;
                    for (int z = 0; z < P.splits; ++z) acc += __ldcg(base + z * (kMaxNP * kTM) + i);
                    if (n < P.N && m0 + rr < P.M)
                        *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1 + 4LL * (m0 + rr)) = acc;
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

// The activation image of vector blockIdx.x: its power-of-two scale 2^e (the
// maximum |x| in [2^14, 2^15) after scaling), hi / lo f16 parts, and the f16
// hi / lo parts of its 32-element sums at scale 2^(e + 5); zeros past N.
__global__ void btc_prep_kernel(const float* __restrict__ x, int64_t x_nb1, __half* __restrict__ ximg,
                                __half* __restrict__ simg, float* __restrict__ vscale, int K, int N, int np) {
    const int n = blockIdx.x;
    const float* xn = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(x) + n * x_nb1);
    __shared__ float red[32];
    __shared__ int e_sh;
    float mx = 0.f;
    if (n < N)
        for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(xn[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.f;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
        int E = 0;
        frexpf(m, &E);  // m < 2^E
        e_sh = (m > 0.f && isfinite(m)) ? E - 15 : 0;
    }
    __syncthreads();
    const int e = e_sh;
    __half* hi = ximg + static_cast<int64_t>(n) * K;
    __half* lo = ximg + static_cast<int64_t>(np + n) * K;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = n < N ? ldexpf(xn[k], -e) : 0.f;
        const __half h = __float2half_rn(v);
        hi[k] = h;
        lo[k] = __float2half_rn(v - __half2float(h));
    }
    // the sums: one 32-element sub-block per thread and round, in order, in double
    const int nsub = K / 32;
    for (int sb = threadIdx.x; sb < nsub; sb += blockDim.x) {
        double acc = 0.0;
        if (n < N)
            for (int i = 0; i < 32; ++i) acc += static_cast<double>(xn[32 * sb + i]);
        const double v = ldexp(acc, -(e + 5));
        const __half h = __double2half(v);
        const __half l = __double2half(v - static_cast<double>(__half2float(h)));
        __half* row = simg + (static_cast<int64_t>(sb / 8) * np + n) * 64;
        row[sb % 8] = h;
        row[8 + sb % 8] = l;
        if (sb % 8 == 0)
            for (int i = 16; i < 64; ++i) row[i] = __float2half_rn(0.f);
    }
    if (threadIdx.x == 0) {
        vscale[n] = ldexpf(1.f, e);
        vscale[np + n] = ldexpf(1.f, e + 5);
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

int np_of(const MulMatOp& o) { return (o.N + 15) / 16 * 16; }
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
size_t ximg_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(2) * np_of(o) * o.K * 2); }
size_t simg_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(o.K / 256) * np_of(o) * 128); }
size_t vscale_bytes(const MulMatOp& o) { return align256(static_cast<size_t>(2) * np_of(o) * 4); }

// K splits: about one wave of CTAs (one per SM), at least two blocks per split.
int plan_splits(const MulMatOp& o, int num_sms) {
    const int tiles = (o.M + kTM - 1) / kTM, nblk = o.K / 256;
    int s = num_sms / tiles;
    s = s < kMaxSplits ? s : kMaxSplits;
    s = s < nblk / 2 ? s : nblk / 2;
    return s > 1 ? s : 1;
}
size_t split_bytes(const MulMatOp& o, int splits) {
    if (splits <= 1) return 0;
    const size_t tiles = static_cast<size_t>((o.M + kTM - 1) / kTM);
    return align256(tiles * splits * kMaxNP * kTM * 4) + align256(tiles * 4);
}

}  // namespace

bool batched_tc_supported(const MulMatOp& o) {
    if (o.type != kTypeQ4_K && o.type != kTypeQ5_K) return false;
    if (o.N < 1 || o.N > kMaxNP || o.ne2 != 1 || o.ne3 != 1) return false;
    if (o.K % 256 != 0 || o.M < 1) return false;
    // TMA rows: 16-byte aligned base and row stride
    if ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15) return false;
    if (o.w_nb1 < static_cast<int64_t>(o.K / 256) * (o.type == kTypeQ5_K ? 176 : 144)) return false;
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
    const int np = np_of(o), nblk = o.K / 256, kb_split = (nblk + splits - 1) / splits;
    splits = (nblk + kb_split - 1) / kb_split;  // no empty split
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* ximg = reinterpret_cast<__half*>(ws);
    __half* simg = reinterpret_cast<__half*>(ws + ximg_bytes(o));
    float* vscale = reinterpret_cast<float*>(ws + ximg_bytes(o) + simg_bytes(o));
    btc_prep_kernel<<<np, 256, 0, stream>>>(o.x, o.x_nb1, ximg, simg, vscale, o.K, o.N, np);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return -static_cast<int>(e);
    BtcArgs P{};
    const EncodeFn enc = btc_encoder();
    const int bb = o.type == kTypeQ5_K ? 176 : 144;
    const cuuint32_t es[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(nblk) * (bb / 8), static_cast<cuuint64_t>(o.M)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.w_nb1)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(bb / 8), static_cast<cuuint32_t>(kTM)};
        if (enc(&P.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(o.w), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(o.K), static_cast<cuuint64_t>(2 * np)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.K) * 2};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), static_cast<cuuint32_t>(np)};
        if (enc(&P.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ximg, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    {
        const cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(nblk) * np};
        const cuuint64_t strides[1] = {128};
        const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(np)};
        if (enc(&P.smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, simg, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -static_cast<int>(cudaErrorInvalidValue);
    }
    P.vscale = vscale;
    P.y = o.y;
    P.y_nb1 = o.y_nb1;
    P.M = o.M;
    P.K = o.K;
    P.N = o.N;
    P.np = np;
    P.splits = splits;
    P.kb_split = kb_split;
    const int tiles = (o.M + kTM - 1) / kTM;
    int launched = 2;
    if (splits > 1) {
        P.partial = reinterpret_cast<float*>(ws + base);
        P.counters = reinterpret_cast<unsigned*>(ws + base + align256(static_cast<size_t>(tiles) * splits * kMaxNP * kTM * 4));
        e = cudaMemsetAsync(P.counters, 0, static_cast<size_t>(tiles) * 4, stream);
        if (e != cudaSuccess) return -static_cast<int>(e);
    }
    const size_t smem = Smem(np, bb).total(np);
    static size_t configured[kMaxDevices][2] = {};
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return -static_cast<int>(e);
    if (dev < 0 || dev >= kMaxDevices) return -static_cast<int>(cudaErrorInvalidDevice);
    const int ti = o.type == kTypeQ5_K ? 1 : 0;
    void (*const kernel)(BtcArgs) = ti ? btc_kernel<kTypeQ5_K> : btc_kernel<kTypeQ4_K>;
    if (configured[dev][ti] < smem) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return -static_cast<int>(e);
        configured[dev][ti] = smem;
    }
    kernel<<<dim3(tiles, 1, splits), kThr, smem, stream>>>(P);
    e = cudaGetLastError();
    return e == cudaSuccess ? launched : -static_cast<int>(e);
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
