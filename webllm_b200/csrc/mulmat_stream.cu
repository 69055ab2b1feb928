// Decode-regime quantized MUL_MAT (N = 1 to 4 activation vectors): a
// persistent, warp-specialised streaming GEMV over raw GGUF blocks.
//
// Data movement. The weight matrix is cut into units of 16 rows (one MMA
// tile); each unit's rows into segments of at most 14 Q4_K / 11 Q5_K / 9 Q6_K
// / 32 Q8_0 / 64 Q4_0 blocks. Warp 0 (copy warp, lane 0) moves each (unit, segment) into a ring
// of shared-memory stages with ONE 2D tensor-map TMA copy (16 rows x the
// segment, rounded out to 16-byte columns; evict-first L2 policy, each
// weight byte is read once). Row layouts whose stride is not a multiple of 16
// bytes fall back to one bulk copy per row. A launch's first kPreStages boxes
// go out at once; the rest wait until the activation image is staged.
//
// Work split. The 8 consumer warps take work items (one block of a unit, all
// 16 rows; at N = 1 two blocks at a time) round-robin from the CTA's item
// sequence without CTA-wide barriers. Every warp writes its partial sums of a
// unit to shared memory and arrives on the unit's barrier; the unit's owner
// warp sums the 8 partials in a fixed order (results are deterministic)
// kRedDelay units later, when the others are normally done, and writes the
// rows.
//
// Every type runs on integer tensor cores (mma.sync m16n8k32, u8 / s8 x s8 ->
// s32):
//  - activations: per 256-element block and vector, x = (l0 + l1/128 +
//    l2/16384) / s with s = 127 / max|x| and int8 limbs l0 = rint(x s),
//    l1 = rint(128 (x s - l0)), l2 = rint(128 (128 (x s - l0) - l1))
//    (|error| <= max|x| / 4161536, about 22 bits of the block maximum: two
//    limbs, 15 bits, left elements next to a 100x outlier channel with a few
//    percent error); the MMA's eight B columns are two (slot, vector) pairs of
//    four columns each, limbs 0, 1, 2 and a zero column, so a lane's two
//    accumulator columns always belong to one pair (even lanes: limbs 0 and
//    1, odd lanes: limb 2). Sub-blocks in different slots share one
//    accumulator without mixing, since a sub-block's MMA reads real B rows
//    only in its own slot's columns. Four vectors take two passes over each
//    weight fragment, one per vector pair;
//  - Q4_K weights: ldmatrix hands each lane the bytes of its fragment; the
//    low nibbles (v & 0x0F0F0F0F) and the high nibbles kept in place
//    (v & 0xF0F0F0F0 = 16 q) are the A operands; 6-bit scales are applied in
//    integer (16 sc for the low-nibble sub-blocks), the mins through exact
//    f32 sums of x over 32-element sub-blocks;
//  - Q6_K weights (210-byte blocks, 2-byte aligned in shared memory): A
//    fragments come from aligned 32-bit loads and a funnel shift; one LOP3
//    per group assembles the 6-bit quants from ql and qh; int8 scales are
//    applied in integer, the -32 offset through exact sums of x over
//    16-element sub-blocks.
//  - Q8_0 weights (34-byte blocks): the signed quants are the A operands as
//    they are (aligned 32-bit loads and a funnel shift); each block's s32
//    result is scaled by its rows' f16 d in f32.
//  - Q5_K weights (176-byte blocks): as Q4_K, with the high-bit plane as a
//    fifth ldmatrix per item; each sub-block's 5-bit quants (u8 0..31) enter
//    the MMA and are scaled by sc.
//  - Q4_0 weights (18-byte blocks): as Q8_0, the nibbles entering as s8
//    q - 8.
//
// Launch: programmatic dependent launch. CTAs trigger their dependents at
// entry; the copy warp streams weights (never written by a preceding kernel)
// at once; consumers execute griddepcontrol.wait before reading activations or
// writing outputs. Every mbarrier wait is bounded; on timeout the CTA records
// an error code for the host and stops waiting, so it still ends.
#include <cuda.h>  // CUtensorMap types only; the encoder is fetched with cudaGetDriverEntryPoint
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_stream_error = 0;

namespace {

constexpr int kCW = 8;                        // consumer warps
constexpr int kThreads = 32 * (kCW + 1);      // + copy warp
constexpr int kRows = 16;                     // rows per unit (one MMA m-tile)
constexpr int kQ4kSegBlocks = 14;             // <= 2016 B per row and stage (a TMA box row is <= 2048 B)
constexpr int kQ6kSegBlocks = 9;              // <= 1890 B (+ 16-byte window slack: a 1936 B box row)
constexpr int kQ80SegBlocks = 32;             // 1088 B, whole 8-block groups
constexpr int kQ5kSegBlocks = 11;             // <= 1936 B
constexpr int kQ40SegBlocks = 64;             // 1152 B, whole 8-block groups
constexpr int kIq4SegBlocks = 14;             // 1904 B (+ 16-byte window slack: a 1936 B box row)
constexpr int kMaxStages = 8;
constexpr int kRedDelay = 2;                  // a unit's partials are summed this many units later
// Unit slots in flight: consumer warps drift apart by at most kMaxStages
// stages (a stage is refilled only after every warp released it), so a slot
// is summed before any warp writes it again.
constexpr int kUnitSlots = kMaxStages + kRedDelay + 2;
constexpr int kXPad = 16;                     // bytes after each int8 activation column (ldmatrix banks)
constexpr int kMaxNT = 4;
constexpr int kMaxK34 = 8192;                 // K limit for 3 or 4 vectors (their activation image)
// Boxes the copy warp issues before the consumers have staged the first
// activation image: the activation loads wait behind whatever weight requests
// are queued in the memory system, so a launch's first boxes are held back
// until the image is built.
constexpr int kPreStages = 2;
static_assert((kCW & (kCW - 1)) == 0, "unit ownership rotates with a mask");
constexpr int kMaxK = 16384;                  // activation image in shared memory
// Polls before a bounded wait gives up (well over a second), unless the host
// set another limit (wllm_set_wait_limit). The limit travels in the launch
// parameters and sits in shared memory beside the CTA's poison flag.
constexpr uint32_t kSpinLimit = 1u << 26;
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
    float* y_peer[kMaxRanks];     // row-sharded launch: this op's rows on rank r (own rank unused)
};

// Fused prologue of the activations, applied before the limb split:
// - kProNorm: RMS_NORM (+ gain MUL), x / sqrt(mean(x^2) + eps) * gain
//   (src/inference/jsep/ops/rms-norm.ts:14-15,61-67; the gain is the separate
//   MUL of src/inference/model-inference.ts:2281,2478-2481);
// - kProSwiglu: silu(x) * up, x the gate projection's output
//   (model-inference.ts:2484-2489, op_swiglu_split of
//   src/wasm/webgpu-bridge.cpp:272-275);
// - kProGelu: gelu(x) * up, the Gemma form (model-inference.ts:2486-2487).
struct ProArgs {
    const float* gain;  // kProNorm: K floats, or null (no gain)
    const float* up;    // kProSwiglu / kProGelu: the up projection's output, laid out like x
    int64_t up_nb1;     // bytes between its vectors
    float eps;          // kProNorm
    int32_t kind;
};

// Row-sharded launch: sig[r] is rank r's signal array, state this rank's
// counters ([0] CTAs done with the launch, [1] launches done).
struct TpSig {
    int32_t world, rank;  // world 1: not row-sharded
    uint32_t* sig[kMaxRanks];
    uint32_t* state;
    uint32_t spin_limit;  // polls of the peer wait before it gives up
};

struct SList {
    SOp op[kMaxOpsPerLaunch];
    int32_t n_ops;
    int32_t total_units;
    int32_t stages;
    int32_t stage_bytes;  // 16 rows x the largest wbox
    int32_t x_bytes;      // shared-memory bytes reserved for the activation image
    int32_t all_tma;      // every op is copied with its tensor map
    TpSig tp;             // world > 1: every output row also goes to the other ranks
    ProArgs pro;          // prologue applied to every op's activations (kind kProNone: none)
    uint32_t spin_limit;  // polls before a bounded wait gives up
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

// Non-blocking test of a phase (cheaper than a potentially blocking try_wait
// when the phase has already completed).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait. If the phase does not complete in time the CTA is poisoned:
// an error code is recorded for the host and every later wait of the CTA
// returns at once, so all threads run to the end (results are garbage, the
// error is reported by wllm_sync). The poison flag is read once per 256
// polls: every poll is a shared-memory operation, and polls of many warps
// were measured to slow the copy warp's own barrier and TMA operations.
// The CTA's wait limit: the word after its poison flag.
__device__ __forceinline__ uint32_t spin_limit_of(volatile int* poisoned) {
    return reinterpret_cast<volatile uint32_t*>(poisoned)[1];
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint32_t lim = spin_limit_of(poisoned);
    for (uint32_t i = 0; i < lim; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *poisoned) return false;
    }
    *poisoned = 1;
    atomicOr(&g_stream_error, code);
    return false;
}

// Warp-wide wait of a consumer warp: lane 0 polls, backing off with a short
// sleep between polls; then every lane observes the completed phase itself
// (one poll that succeeds at once), which orders the landed copy's bytes
// before its reads.
__device__ __forceinline__ void mbar_wait_warp(uint64_t* bar, uint32_t parity, unsigned code, volatile int* poisoned,
                                               int lane) {
    int ok = 1;
    if (lane == 0) {
        ok = 0;
        const uint32_t lim = spin_limit_of(poisoned);
        for (uint32_t i = 0; i < lim; ++i) {
            if (mbar_try_wait(bar, parity)) {
                ok = 1;
                break;
            }
            if ((i & 255u) == 255u && *poisoned) break;
            __nanosleep(32);
        }
        if (!ok && !*poisoned) {
            *poisoned = 1;
            atomicOr(&g_stream_error, code);
        }
    }
    if (__shfl_sync(0xffffffffu, ok, 0)) (void)mbar_try_wait(bar, parity);
}

// Before the copy warp leaves: waits (bounded, whatever the poison flag
// says) until the last copy issued into each stage has landed, so that no
// bulk copy still writes into this CTA's shared memory after it exits. In a
// healthy launch the consumers have waited for all of them already; after a
// time-out they may not have. Bit s of `issued` marks a stage that received
// a copy, bit s of `par` the parity of its last full phase.
__device__ __forceinline__ void drain_copies(uint64_t* full, int S, uint32_t issued, uint32_t par,
                                             volatile int* poisoned) {
    const uint32_t lim = spin_limit_of(poisoned);
    for (int st = 0; st < S; ++st) {
        if (!((issued >> st) & 1u)) continue;
        uint32_t i = 0;
        while (i < lim && !mbar_try_wait(&full[st], (par >> st) & 1u)) ++i;
        if (i == lim) atomicOr(&g_stream_error, 8u);
    }
}

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
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

// Four 8x8 b16 matrices from shared memory; lane l supplies the row address
// for row l%8 of matrix l/8 and receives, of each matrix, bytes 4(l%4)..+3 of
// row l/4.
__device__ __forceinline__ void ldmatrix_x4_at(uint32_t (&r)[4], uint32_t smem_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr));
}

// D += A (16x32 u8, row) * B (32x8 s8, col), s32.
__device__ __forceinline__ void imma_u8s8_acc(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D += A (16x32 s8, row) * B (32x8 s8, col), s32.
__device__ __forceinline__ void imma_s8s8_acc(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__host__ __device__ __forceinline__ int seg_cap(int type) {
    switch (type) {
        case kTypeQ4_K: return kQ4kSegBlocks;
        case kTypeQ5_K: return kQ5kSegBlocks;
        case kTypeQ6_K: return kQ6kSegBlocks;
        case kTypeQ4_0: return kQ40SegBlocks;
        case kTypeIQ4_XS: return kIq4SegBlocks;
        default: return kQ80SegBlocks;
    }
}
__device__ __forceinline__ int block_elems_of(int type) {
    return (type == kTypeQ8_0 || type == kTypeQ4_0) ? 32 : 256;
}
__device__ __forceinline__ int block_bytes_of(int type) {
    switch (type) {
        case kTypeQ4_K: return 144;
        case kTypeQ5_K: return 176;
        case kTypeQ6_K: return 210;
        case kTypeQ4_0: return 18;
        case kTypeIQ4_XS: return 136;
        default: return 34;
    }
}

// Four 4-bit quants q (0..15, one per byte) -> the int8 bytes q - 8: q ^ 8 is
// q - 8 as a 4-bit two's-complement number; copy its sign bit (bit 3) into
// bits 4..7 (0x08 * 0x1E = 0xF0 stays inside each byte).
__device__ __forceinline__ uint32_t q4_signed(uint32_t q) {
    const uint32_t t = q ^ 0x08080808u;
    return t | ((t & 0x08080808u) * 0x1Eu);
}

// Byte layout of the shared-memory activation image.
//  Every type (one shared image): int8 limb columns [3N][K + kXPad]
//        (column 3t + l = limb l of vector t), then f32 d-factors [N][K/256]
//        (max|x| / (127 * 16) per block), then exact f32 sums of x over
//        32-element sub-blocks [N][K/32] (Q4_K, Q5_K) and over 16-element
//        sub-blocks [N][K/16] (Q6_K). Q8_0 and Q4_0 use the limbs and
//        d-factors.
__host__ __device__ __forceinline__ int img_col_bytes(int K) { return K + kXPad; }
constexpr int kLimbs = 3;  // int8 limbs per activation element
__host__ __device__ __forceinline__ int img_inv_off(int K, int N) { return kLimbs * N * img_col_bytes(K); }
// (16-byte aligned: the sums are read as float2)
__host__ __device__ __forceinline__ int img_sum_off(int K, int N) {
    return (img_inv_off(K, N) + 4 * N * (K / 256) + 15) & ~15;
}
__host__ __device__ __forceinline__ int img_sum16_off(int K, int N) { return img_sum_off(K, N) + 4 * N * (K / 32); }
__host__ __device__ __forceinline__ int img_bytes(int K, int N) { return img_sum16_off(K, N) + 4 * N * (K / 16); }

// 4 bytes at any 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);
    return __funnelshift_r(q[0], q[1], mis * 8);
}
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// Scales of the sub-blocks j = q NS + sl (q = 0 .. NCH-1) of one Q4_K block
// header h (get_scale_min_k4 semantics, src/inference/jsep/ops/matmul.ts:408-424:
// for j < 4 sc = s[j]&63, m = s[j+4]&63; for j >= 4 sc = (s[j+4]&15) |
// (s[j-4]>>6)<<4, m = (s[j+4]>>4) | (s[j]>>6)<<4). sc comes out as an int,
// times 16 for even (low-nibble) sub-blocks, whose quants enter the MMA
// unscaled (RAW, for Q5_K: sc for every sub-block); m as dmin*m, exactly
// rounded: (2^23 + m) dmin - 2^23 dmin in one FMA (both products exact: dmin
// has at most 11 significant bits).
template <int NS, int NCH, bool RAW = false>
__device__ __forceinline__ void q4k_slot_scales(const uint4 h, int sl, int (&sc)[NCH], float (&mdm)[NCH], float& d) {
    d = f16_bits_to_f32(h.x);
    const float dmin = f16_bits_to_f32(h.x >> 16);
    const float dm23 = dmin * 8388608.f;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int jj = q * NS + sl;
        const uint32_t sel = 0x4440u + static_cast<uint32_t>(jj & 3);  // byte jj%4, zero-extended
        uint32_t scv, mv;
        if (q * NS < 4) {  // j < 4 (NS divides 4 and sl < NS)
            scv = __byte_perm(h.y, 0u, sel) & 63u;
            mv = __byte_perm(h.z, 0u, sel) & 63u;
        } else {
            const uint32_t b1 = __byte_perm(h.y, 0u, sel), b2 = __byte_perm(h.z, 0u, sel), b3 = __byte_perm(h.w, 0u, sel);
            scv = (b3 & 15u) | ((b1 >> 2) & 0x30u);
            mv = (b3 >> 4) | ((b2 >> 2) & 0x30u);
        }
        sc[q] = static_cast<int>(scv << (((jj & 1) || RAW) ? 0 : 4));
        mdm[q] = fmaf(__uint_as_float(0x4B000000u | mv), dmin, -dm23);
    }
}

// One Q4_K item: 16 rows x one 256-element block, for NP = 1 or 2 vectors
// (four vectors run this twice, once per vector pair). The MMA's 8 columns
// are two (slot, vector) pairs of limbs 0, 1, 2 and a zero column: NS = 2
// sub-block slots of one vector, or one slot of two vectors (column
// 4 u + l). A sub-block's MMA reads the activation rows of its own slot;
// every other B row is the zero row, so the NS sub-blocks of a chain
// accumulate into one fragment without mixing, and lane (g, c) ends up with
// pair u = c / 2 of rows g and g+8: limbs 0 and 1 (hl = c & 1 = 0) or limb 2
// (hl = 1). It scales only its slot's sub-blocks, NCH = 8 / NS per row; the
// mins are added by the hl = 0 lane of each pair.
template <int NP, int NI>
__device__ __forceinline__ void q4k_items(const uint8_t* blk, int wbox, uint32_t wl, uint32_t xaddr, uint32_t xzero,
                                          bool xv0, bool xv1, const float* df, const float* xs, int g, int sl, int hl,
                                          float& yg, float& yh) {
    // NI items of one unit at once (blocks kCW apart): independent chains the
    // scheduler interleaves
    static_assert(NP == 1 || NP == 2, "vector pairs");
    constexpr int NS = NP == 1 ? 2 : 1, NCH = 8 / NS;
    constexpr int BS = kCW * 144;  // stage bytes between the items
    constexpr int XS = kCW * 256;  // activation bytes between the items
    int scg[NI][NCH], sch[NI][NCH];
    float mg[NI][NCH], mh[NI][NCH], dg[NI], dh[NI];
#pragma unroll
    for (int k = 0; k < NI; ++k) {
        const uint4 hg = *reinterpret_cast<const uint4*>(blk + k * BS + g * wbox);
        const uint4 hh = *reinterpret_cast<const uint4*>(blk + k * BS + (g + 8) * wbox);
        q4k_slot_scales<NS, NCH>(hg, sl, scg[k], mg[k], dg[k]);
        q4k_slot_scales<NS, NCH>(hh, sl, sch[k], mh[k], dh[k]);
    }
    int D[NI][NCH][4];
#pragma unroll
    for (int k = 0; k < NI; ++k)
#pragma unroll
        for (int q = 0; q < NCH; ++q) D[k][q][0] = D[k][q][1] = D[k][q][2] = D[k][q][3] = 0;
    const uint32_t wbase = smem_u32(blk) + wl;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int k = 0; k < NI; ++k) {
            uint32_t w[4], x[4];
            ldmatrix_x4_at(w, wbase + k * BS + 32 * p);
            ldmatrix_x4_at(x, ((p & 1) ? xv1 : xv0) ? xaddr + k * XS + 64 * p : xzero);
            imma_u8s8_acc(D[k][(2 * p) / NS], w[0] & 0x0F0F0F0Fu, w[1] & 0x0F0F0F0Fu, w[2] & 0x0F0F0F0Fu,
                          w[3] & 0x0F0F0F0Fu, x[0], x[1]);
            imma_u8s8_acc(D[k][(2 * p + 1) / NS], w[0] & 0xF0F0F0F0u, w[1] & 0xF0F0F0F0u, w[2] & 0xF0F0F0F0u,
                          w[3] & 0xF0F0F0F0u, x[2], x[3]);
        }
    }
    // limb weights of the lane's two columns: (1, 1/128) or (1/16384, 0)
    const float lf = hl ? 6.103515625e-05f : 1.f;
#pragma unroll
    for (int k = 0; k < NI; ++k) {
        int a0 = 0, a1 = 0, a2 = 0, a3 = 0;  // (g, col 0), (g, col 1), (g+8, col 0), (g+8, col 1)
#pragma unroll
        for (int q = 0; q < NCH; ++q) {
            a0 += scg[k][q] * D[k][q][0];
            a1 += scg[k][q] * D[k][q][1];
            a2 += sch[k][q] * D[k][q][2];
            a3 += sch[k][q] * D[k][q][3];
        }
        const float xf = df[k * kCW];
        yg = fmaf(fmaf(static_cast<float>(a1), 0.0078125f, static_cast<float>(a0) * lf), dg[k] * xf, yg);
        yh = fmaf(fmaf(static_cast<float>(a3), 0.0078125f, static_cast<float>(a2) * lf), dh[k] * xf, yh);
        if (!hl) {
#pragma unroll
            for (int q = 0; q < NCH; ++q) {
                const float X = xs[k * kCW * 8 + q * NS + sl];
                yg = fmaf(-mg[k][q], X, yg);
                yh = fmaf(-mh[k][q], X, yh);
            }
        }
    }
}

// One Q5_K item (176-byte blocks, 16-byte aligned like Q4_K): as q4k_items,
// with the high-bit plane qh[32] at +16 (one more ldmatrix per item, same
// lane layout as a quant pair) and the quants at +48. Sub-block j's 5-bit
// quants are its nibbles (the high ones shifted down) with bit j of qh as
// bit 4, u8 0..31; the scales are sc for every sub-block and the x factor
// is 1/s (16 dfac).
template <int NP, int NI>
__device__ __forceinline__ void q5k_items(const uint8_t* blk, int wbox, uint32_t wl, uint32_t xaddr, uint32_t xzero,
                                          bool xv0, bool xv1, const float* df, const float* xs, int g, int sl, int hl,
                                          float& yg, float& yh) {
    static_assert(NP == 1 || NP == 2, "vector pairs");
    constexpr int NS = NP == 1 ? 2 : 1, NCH = 8 / NS;
    constexpr int BS = kCW * 176;  // stage bytes between the items
    constexpr int XS = kCW * 256;  // activation bytes between the items
    int scg[NI][NCH], sch[NI][NCH];
    float mg[NI][NCH], mh[NI][NCH], dg[NI], dh[NI];
#pragma unroll
    for (int k = 0; k < NI; ++k) {
        const uint4 hg = *reinterpret_cast<const uint4*>(blk + k * BS + g * wbox);
        const uint4 hh = *reinterpret_cast<const uint4*>(blk + k * BS + (g + 8) * wbox);
        q4k_slot_scales<NS, NCH, true>(hg, sl, scg[k], mg[k], dg[k]);
        q4k_slot_scales<NS, NCH, true>(hh, sl, sch[k], mh[k], dh[k]);
    }
    int D[NI][NCH][4];
#pragma unroll
    for (int k = 0; k < NI; ++k)
#pragma unroll
        for (int q = 0; q < NCH; ++q) D[k][q][0] = D[k][q][1] = D[k][q][2] = D[k][q][3] = 0;
    const uint32_t wbase = smem_u32(blk) + wl;  // wl points at +16: qh, then the quant pairs at +48
    uint32_t hq[NI][4];
#pragma unroll
    for (int k = 0; k < NI; ++k) ldmatrix_x4_at(hq[k], wbase + k * BS);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int k = 0; k < NI; ++k) {
            uint32_t w[4], x[4], lo[4], hi[4];
            ldmatrix_x4_at(w, wbase + k * BS + 32 + 32 * p);
            ldmatrix_x4_at(x, ((p & 1) ? xv1 : xv0) ? xaddr + k * XS + 64 * p : xzero);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                lo[r] = (w[r] & 0x0F0F0F0Fu) | (((hq[k][r] >> (2 * p)) & 0x01010101u) << 4);
                hi[r] = ((w[r] >> 4) & 0x0F0F0F0Fu) | (((hq[k][r] >> (2 * p + 1)) & 0x01010101u) << 4);
            }
            imma_u8s8_acc(D[k][(2 * p) / NS], lo[0], lo[1], lo[2], lo[3], x[0], x[1]);
            imma_u8s8_acc(D[k][(2 * p + 1) / NS], hi[0], hi[1], hi[2], hi[3], x[2], x[3]);
        }
    }
    const float lf = hl ? 6.103515625e-05f : 1.f;  // limb weights (see q4k_items)
#pragma unroll
    for (int k = 0; k < NI; ++k) {
        int a0 = 0, a1 = 0, a2 = 0, a3 = 0;  // (g, col 0), (g, col 1), (g+8, col 0), (g+8, col 1)
#pragma unroll
        for (int q = 0; q < NCH; ++q) {
            a0 += scg[k][q] * D[k][q][0];
            a1 += scg[k][q] * D[k][q][1];
            a2 += sch[k][q] * D[k][q][2];
            a3 += sch[k][q] * D[k][q][3];
        }
        const float xf = 16.f * df[k * kCW];
        yg = fmaf(fmaf(static_cast<float>(a1), 0.0078125f, static_cast<float>(a0) * lf), dg[k] * xf, yg);
        yh = fmaf(fmaf(static_cast<float>(a3), 0.0078125f, static_cast<float>(a2) * lf), dh[k] * xf, yh);
        if (!hl) {
#pragma unroll
            for (int q = 0; q < NCH; ++q) {
                const float X = xs[k * kCW * 8 + q * NS + sl];
                yg = fmaf(-mg[k][q], X, yg);
                yh = fmaf(-mh[k][q], X, yh);
            }
        }
    }
}

// rint(v) for |v| < 2^22 without the conversion pipe: adding 1.5 * 2^23
// rounds v to an integer (round to nearest even), and the sum's bit pattern
// is 0x4B400000 + rint(v), so its low byte is the low byte of rint(v) in
// two's complement; `r` gets rint(v) as a float (exact).
__device__ __forceinline__ int round_low_byte(float v, float& r) {
    constexpr float kRound = 12582912.f;  // 1.5 * 2^23
    const float t = __fadd_rn(v, kRound);
    r = __fsub_rn(t, kRound);
    return __float_as_int(t);
}

// Low bytes of four ints -> one word.
__device__ __forceinline__ uint32_t pack_b4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x0040u),
                       __byte_perm(static_cast<uint32_t>(c), static_cast<uint32_t>(d), 0x0040u), 0x5410u);
}

// A operands of the four 32-element groups of one Q6_K half-block at one
// fragment position: ql0 / ql1 hold four bytes of the half's low-quant
// chunks 0 / 1 (ql[64h + l], ql[64h + 32 + l]), qh the four matching high-bit
// bytes (qh[32h + l]). Group t holds the 6-bit quants (0..63) of elements
// 128h + 32t + l: low nibble of chunk t&1 for t < 2, high nibble for t >= 2,
// and bits 2t, 2t+1 of qh as bits 4, 5 (src/inference/jsep/ops/matmul.ts
// leaves Q6_K to ggml; the layout is ggml's dequantize_row_q6_K). Each group
// is one LOP3 (a & 0x0F) | (b & 0xF0) whose b carries nothing but the two
// wanted bits in the high half of every byte.
__device__ __forceinline__ void q6k_groups(uint32_t ql0, uint32_t ql1, uint32_t qh, uint32_t (&a)[4]) {
    const uint32_t m = 0x0F0F0F0Fu;
    const uint32_t qa = qh & 0x33333333u, qb = qh & 0xCCCCCCCCu;  // groups 0, 2 / 1, 3
    a[0] = (ql0 & m) | ((qa << 4) & ~m);
    a[1] = (ql1 & m) | ((qb << 2) & ~m);
    a[2] = ((ql0 >> 4) & m) | (qa & ~m);
    a[3] = ((ql1 >> 4) & m) | ((qb >> 2) & ~m);
}

// One Q6_K item: 16 rows x one 256-element block on integer tensor cores,
// for NP = N rounded up to a power of two. Blocks are 210 bytes, so a block
// sits at any even offset in shared memory: the A fragments come from aligned
// 32-bit loads and a funnel shift (ldmatrix needs 16-byte rows). MMA i covers
// elements 32i .. 32i+31, i.e. the 16-element sub-blocks 2i (k 0..15) and
// 2i+1 (k 16..31). As for Q4_K (NP = 1 or 2), the 8 B columns are two
// (slot, vector) pairs of limbs 0..2 and a zero column, NS = 2 / NP slots;
// sub-block j uses slot j % NS of chain j / NS, its B rows are real only in
// its slot's columns, so NS sub-blocks share one fragment without mixing.
// Lane (g, c) scales the chains' slot sl: the sub-blocks j = q NS + sl of
// rows g and g + 8, with their int8 scales in integer. The -32 offset of
// every quant is applied through the exact 16-element sums of x:
// sum sc (q - 32) x = sum sc q x - 32 sum sc X (by the hl = 0 lane of a pair).
template <int NP>
__device__ __forceinline__ void q6k_item(const uint8_t* pg, const uint8_t* ph, uint32_t xaddr, uint32_t xzero,
                                         bool xv, float xf, const float* xs, int c, int sl, int hl, float& yg,
                                         float& yh) {
    static_assert(NP == 1 || NP == 2, "vector pairs");
    constexpr int NS = NP == 1 ? 2 : 1, NCH = 16 / NS, NCHH = NCH / 2;  // chains per half-block
    // |D| <= 16 * 63 * 127 per sub-block; times |sc| <= 128, summed over the
    // lane's 4, 8 or 16 sub-blocks: well inside int32
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    float sg = 0.f, sh = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int D[NCHH][4];
#pragma unroll
        for (int q = 0; q < NCHH; ++q) D[q][0] = D[q][1] = D[q][2] = D[q][3] = 0;
        // fragment positions: 0 = row g k 4c.., 1 = row g+8 k 4c.., 2 = row g
        // k 16+4c.., 3 = row g+8 k 16+4c..
        uint32_t A[4][4];  // [position][group]
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint8_t* b = ((r & 1) ? ph : pg) + 4 * c + 16 * (r >> 1);
            q6k_groups(lds_u32_any(b + 64 * h), lds_u32_any(b + 64 * h + 32), lds_u32_any(b + 128 + 32 * h), A[r]);
        }
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
            const int p = 2 * h + pp;  // MMAs 2p, 2p+1 = groups 2pp, 2pp+1 of half h
            uint32_t x[4];
            ldmatrix_x4_at(x, xv ? xaddr + 64 * p : xzero);
            if constexpr (NS == 1) {
                // one slot (a vector pair): the two 16-element sub-blocks of an MMA
                // step cannot share its columns, so each gets its own MMA with
                // the other half of the A fragment zero
                imma_u8s8_acc(D[4 * pp], A[0][2 * pp], A[1][2 * pp], 0u, 0u, x[0], x[1]);
                imma_u8s8_acc(D[4 * pp + 1], 0u, 0u, A[2][2 * pp], A[3][2 * pp], x[0], x[1]);
                imma_u8s8_acc(D[4 * pp + 2], A[0][2 * pp + 1], A[1][2 * pp + 1], 0u, 0u, x[2], x[3]);
                imma_u8s8_acc(D[4 * pp + 3], 0u, 0u, A[2][2 * pp + 1], A[3][2 * pp + 1], x[2], x[3]);
            } else {
                imma_u8s8_acc(D[(4 * pp) / NS], A[0][2 * pp], A[1][2 * pp], A[2][2 * pp], A[3][2 * pp], x[0], x[1]);
                imma_u8s8_acc(D[(4 * pp + 2) / NS], A[0][2 * pp + 1], A[1][2 * pp + 1], A[2][2 * pp + 1],
                              A[3][2 * pp + 1], x[2], x[3]);
            }
        }
        // chain q of this half holds sub-blocks (h NCHH + q) NS + slot
#pragma unroll
        for (int q = 0; q < NCHH; ++q) {
            const int j = (h * NCHH + q) * NS + sl;
            const int scg = static_cast<int>(*reinterpret_cast<const int8_t*>(pg + 192 + j));
            const int sch = static_cast<int>(*reinterpret_cast<const int8_t*>(ph + 192 + j));
            a0 += scg * D[q][0];
            a1 += scg * D[q][1];
            a2 += sch * D[q][2];
            a3 += sch * D[q][3];
            const float X = xs[j];
            sg = fmaf(static_cast<float>(scg), X, sg);
            sh = fmaf(static_cast<float>(sch), X, sh);
        }
    }
    const float dg = f16_bits_to_f32(lds_u16(pg + 208)), dh = f16_bits_to_f32(lds_u16(ph + 208));
    const float lf = hl ? 6.103515625e-05f : 1.f;  // limb weights (see q4k_items)
    const float mf = hl ? 0.f : -32.f;             // the offset once per pair
    yg = fmaf(dg, fmaf(fmaf(static_cast<float>(a1), 0.0078125f, static_cast<float>(a0) * lf), xf, mf * sg), yg);
    yh = fmaf(dh, fmaf(fmaf(static_cast<float>(a3), 0.0078125f, static_cast<float>(a2) * lf), xf, mf * sh), yh);
}

// One IQ4_XS item: 16 rows x one 136-byte block (256 elements), for NP = 1 or
// 2 vectors. Sub-block j (32 elements) is one MMA on the int8 levels: lane
// (g, c)'s A fragment for rows g / g+8 is the low nibbles of qs[16j + 4c ..
// + 3] (k = 4c ..) and their high nibbles (k = 16 + 4c ..), looked up in the
// level table. As for Q4_K, NS = 2/NP sub-blocks share an accumulator through
// the B-column slots (sub-block j: slot j % NS, chain j / NS); lane (g, c)
// scales its slot's sub-blocks by ls - 32 in integer, then by the rows' f16 d.
// Blocks sit 8-byte aligned in shared memory.
template <int NP>
__device__ __forceinline__ void iq4xs_item(const uint8_t* pg, const uint8_t* ph, uint32_t xaddr, uint32_t xzero,
                                           bool xv0, bool xv1, float xf, int c, int sl, int hl, float& yg,
                                           float& yh) {
    static_assert(NP == 1 || NP == 2, "vector pairs");
    constexpr int NS = NP == 1 ? 2 : 1, NCH = 8 / NS;
    int D[NCH][4];
#pragma unroll
    for (int q = 0; q < NCH; ++q) D[q][0] = D[q][1] = D[q][2] = D[q][3] = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {  // sub-blocks 2p, 2p+1: one ldmatrix of activations
        uint32_t x[4];
        ldmatrix_x4_at(x, ((p & 1) ? xv1 : xv0) ? xaddr + 64 * p : xzero);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * p + h;
            const uint32_t wg = lds_u32_any(pg + 8 + 16 * j + 4 * c), wh = lds_u32_any(ph + 8 + 16 * j + 4 * c);
            uint32_t gl, gh, hl, hh;  // levels: rows g / g+8, low / high nibbles
            iq4_lut8(wg, gl, gh);
            iq4_lut8(wh, hl, hh);
            imma_s8s8_acc(D[j / NS], gl, hl, gh, hh, x[2 * h],
                          x[2 * h + 1]);
        }
    }
    // |D| <= 32 * 127 * 127 per sub-block, times |ls - 32| <= 32, over 8: inside int32
    const uint32_t shg = lds_u16(pg + 2), slg = lds_u32_any(pg + 4);
    const uint32_t shh = lds_u16(ph + 2), slh = lds_u32_any(ph + 4);
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int j = q * NS + sl;
        const int scg = iq4xs_scale(shg, slg, j), sch = iq4xs_scale(shh, slh, j);
        a0 += scg * D[q][0];
        a1 += scg * D[q][1];
        a2 += sch * D[q][2];
        a3 += sch * D[q][3];
    }
    const float lf = hl ? 6.103515625e-05f : 1.f;  // limb weights (see q4k_items)
    const float dg = f16_bits_to_f32(lds_u16(pg)), dh = f16_bits_to_f32(lds_u16(ph));
    yg = fmaf(fmaf(static_cast<float>(a1), 0.0078125f, static_cast<float>(a0) * lf), dg * xf, yg);
    yh = fmaf(fmaf(static_cast<float>(a3), 0.0078125f, static_cast<float>(a2) * lf), dh * xf, yh);
}

// One Q8_0 / Q4_0 item: 16 rows x one group of 8 blocks (256 elements, one x
// scale), for NP = 1 or 2 vectors. Each 32-element block is one MMA on the
// signed quants as they are; as for Q4_K, NS = 2/NP blocks share an
// accumulator through the B-column slots (block j: slot j % NS, chain j / NS),
// and lane (g, c) scales its slot's blocks j = q NS + sl of rows g and g + 8
// by their f16 d in f32. Blocks are 34 (18) bytes, so they
// sit 2-byte aligned in shared memory: aligned 32-bit loads and a funnel
// shift. Q4_0's nibbles enter as s8 q - 8 (a 4-bit sign extension).
template <int NP, int TYPE>
__device__ __forceinline__ void q8_item(const uint8_t* pg, const uint8_t* ph, uint32_t xaddr, uint32_t xzero,
                                        bool xv0, bool xv1, float xf, int c, int sl, int hl, float& yg, float& yh) {
    static_assert(NP == 1 || NP == 2, "vector pairs");
    constexpr int NS = NP == 1 ? 2 : 1, NCH = 8 / NS;
    constexpr int BB = TYPE == kTypeQ4_0 ? 18 : 34;  // block bytes
    int D[NCH][4];
#pragma unroll
    for (int q = 0; q < NCH; ++q) D[q][0] = D[q][1] = D[q][2] = D[q][3] = 0;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {  // blocks 2pp, 2pp+1: one ldmatrix of activations
        uint32_t x[4];
        ldmatrix_x4_at(x, ((pp & 1) ? xv1 : xv0) ? xaddr + 64 * pp : xzero);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * pp + h;
            const uint8_t* bg = pg + BB * j + 2 + 4 * c;
            const uint8_t* bh = ph + BB * j + 2 + 4 * c;
            if (TYPE == kTypeQ4_0) {
                // elements 4c.. are the low nibbles of qs[4c..], 16+4c.. the high ones
                const uint32_t wg = lds_u32_any(bg), wh = lds_u32_any(bh);
                imma_s8s8_acc(D[j / NS], q4_signed(wg & 0x0F0F0F0Fu), q4_signed(wh & 0x0F0F0F0Fu),
                              q4_signed((wg >> 4) & 0x0F0F0F0Fu), q4_signed((wh >> 4) & 0x0F0F0F0Fu), x[2 * h],
                              x[2 * h + 1]);
            } else {
                imma_s8s8_acc(D[j / NS], lds_u32_any(bg), lds_u32_any(bh), lds_u32_any(bg + 16), lds_u32_any(bh + 16),
                              x[2 * h], x[2 * h + 1]);
            }
        }
    }
    // |D| <= 32 * 127 * 127 per block
    const float lf = hl ? 6.103515625e-05f : 1.f;  // limb weights (see q4k_items)
    float ag = 0.f, ah = 0.f;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int j = q * NS + sl;
        const float dg = f16_bits_to_f32(lds_u16(pg + BB * j)), dh = f16_bits_to_f32(lds_u16(ph + BB * j));
        ag = fmaf(fmaf(static_cast<float>(D[q][1]), 0.0078125f, static_cast<float>(D[q][0]) * lf), dg, ag);
        ah = fmaf(fmaf(static_cast<float>(D[q][3]), 0.0078125f, static_cast<float>(D[q][2]) * lf), dh, ah);
    }
    yg = fmaf(ag, xf, yg);
    yh = fmaf(ah, xf, yh);
}


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
    float* y_peer[kMaxRanks];
};

// The current op's fields, held in registers by the consumer warps (the
// shared-memory table is read only when the op changes).
struct OpRegs {
    const uint8_t* w;
    float* y;
    int64_t w_nb1, y_nb1;
    int32_t type, M, K, N, unit_begin, seg_blocks, nseg, wbox;
};

__device__ __forceinline__ OpRegs op_regs(const OpInfo& o) {
    OpRegs r;
    r.w = o.w;
    r.y = o.y;
    r.w_nb1 = o.w_nb1;
    r.y_nb1 = o.y_nb1;
    r.type = o.type;
    r.M = o.M;
    r.K = o.K;
    r.N = o.N;
    r.unit_begin = o.unit_begin;
    r.seg_blocks = o.seg_blocks;
    r.nseg = o.nseg;
    r.wbox = o.wbox;
    return r;
}

struct OpTable {
    OpInfo op[kMaxOpsPerLaunch];
    int32_t n_ops, total_units;
    ProArgs pro;
};


// x * sigmoid(z) = x / (1 + e^-z) with the SFU exponential and reciprocal
// (__expf, __fdividef: a few f32 ulps from the correctly rounded forms,
// below the activation's 14-bit limb split). e^-z = inf gives x / inf = 0.
__device__ __forceinline__ float x_sigmoid(float x, float z) { return __fdividef(x, 1.f + __expf(-z)); }

// silu(g) * u: ggml's scalar CPU kernel, g / (1 + e^-g) times u
// (ggml_vec_swiglu_f32).
__device__ __forceinline__ float swiglu1(float g, float u) { return __fmul_rn(x_sigmoid(g, g), u); }

// gelu(g) * u as ggml's CPU GELU computes it (its GGML_GELU_FP16 table): g
// rounded to f16, the tanh form 0.5 f (1 + tanh(s)), s = sqrt(2/pi) f (1 +
// 0.044715 f^2), rounded to f16; 0 at g <= -10 and g itself at g >= 10. The
// tanh form is evaluated as f * sigmoid(2 s), the same function. The MUL by
// u is a separate f32 op in the reference.
__device__ __forceinline__ float gelu1(float g, float u) {
    float y;
    if (g <= -10.f) {
        y = 0.f;
    } else if (g >= 10.f) {
        y = g;
    } else {
        const float f = __half2float(__float2half_rn(g));
        const float s = (0.7978845608028654f * f) * (1.f + (0.044715f * f) * f);
        y = __half2float(__float2half_rn(x_sigmoid(f, 2.f * s)));
    }
    return __fmul_rn(y, u);
}

template <int PRO>
__device__ __forceinline__ float4 glu4(float4 g, float4 u) {
    if constexpr (PRO == kProSwiglu)
        return make_float4(swiglu1(g.x, u.x), swiglu1(g.y, u.y), swiglu1(g.z, u.z), swiglu1(g.w, u.w));
    else
        return make_float4(gelu1(g.x, u.x), gelu1(g.y, u.y), gelu1(g.z, u.z), gelu1(g.w, u.w));
}

// Builds the activation image of `op` in shared memory (all consumer warps;
// one L2 round trip).
// With a fused RMS_NORM, a first pass over the same elements sums x^2 per
// vector: per warp, then over the 8 warps in warp order (deterministic); it
// keeps each half-warp's first (vector, block) pair and its gains in
// registers for the second pass (at batch 1 and K <= 4096 that is every pair;
// the others come from L1). Every element is then scaled by
// 1 / sqrt(mean(x^2) + eps) and then by its gain. With a fused GLU the up
// projection's values are loaded beside the gate's and combined with them.
template <int PRO>
__device__ __forceinline__ void stage_activations(const OpInfo& op, uint8_t* xsm, int lane, int cw, const ProArgs& nrm,
                                                  float (*nred)[kMaxNT]) {
    constexpr bool NORM = PRO == kProNorm;
    constexpr bool GLU = PRO == kProSwiglu || PRO == kProGelu;
    const int K = op.K, N = op.N;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(op.x);
    const int nblk = K / 256, XS = img_col_bytes(K);
    float* dfac = reinterpret_cast<float*>(xsm + img_inv_off(K, N));
    float* Xs = reinterpret_cast<float*>(xsm + img_sum_off(K, N));
    float* X16 = reinterpret_cast<float*>(xsm + img_sum16_off(K, N));
    float inv[kMaxNT] = {1.f, 1.f, 1.f, 1.f};
    float4 keep_x[4], keep_g[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) keep_g[k] = keep_x[k] = make_float4(1.f, 1.f, 1.f, 1.f);
    if constexpr (NORM) {
        float ssl[kMaxNT] = {0.f, 0.f, 0.f, 0.f};
        for (int tb = 2 * cw + (lane >> 4); tb < N * nblk; tb += 2 * kCW) {
            const int t = tb / nblk, b = tb - t * nblk;
            const float4* xv = reinterpret_cast<const float4*>(xb + t * op.x_nb1) + b * 64 + 4 * (lane & 15);
            const bool first = tb == 2 * cw + (lane >> 4);
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 e = __ldg(xv + k);
                if (first) {  // the second pass's first pair: kept in registers with its gains
                    keep_x[k] = e;
                    if (nrm.gain) keep_g[k] = __ldg(reinterpret_cast<const float4*>(nrm.gain) + b * 64 + 4 * (lane & 15) + k);
                }
                a = fmaf(e.x, e.x, a);
                a = fmaf(e.y, e.y, a);
                a = fmaf(e.z, e.z, a);
                a = fmaf(e.w, e.w, a);
            }
#pragma unroll
            for (int q = 0; q < kMaxNT; ++q) ssl[q] += q == t ? a : 0.f;
        }
#pragma unroll
        for (int q = 0; q < kMaxNT; ++q) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ssl[q] += __shfl_xor_sync(0xffffffffu, ssl[q], o);
        }
        if (lane == 0)
#pragma unroll
            for (int q = 0; q < kMaxNT; ++q) nred[cw][q] = ssl[q];
        consumers_sync();
#pragma unroll
        for (int q = 0; q < kMaxNT; ++q) {
            float ss = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kCW; ++w2) ss += nred[w2][q];
            inv[q] = 1.f / sqrtf(ss / static_cast<float>(K) + nrm.eps);
        }
    }
    // one (vector, block) per half-warp and round: lane h = lane%16 covers
    // elements 16h .. 16h+15. Two rounds' loads are issued before any
    // arithmetic (K = 8192 at N = 1 is two rounds: one L2 round trip)
    const int hw = lane >> 4, h = lane & 15, total = N * nblk;
    for (int tb0 = 2 * cw + hw; tb0 - hw < total; tb0 += 4 * kCW) {  // warp-uniform
        float4 v[2][4], uq[2][4];
        bool act[2];
        int t[2], b[2];
        // the second round only where the warp has one (warp-uniform)
        const int rounds = tb0 - hw + 2 * kCW < total ? 2 : 1;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int tb = tb0 + 2 * kCW * r;
            act[r] = tb < total;
            t[r] = act[r] ? tb / nblk : 0;
            b[r] = act[r] ? tb - t[r] * nblk : 0;
            const float4* xv = reinterpret_cast<const float4*>(xb + t[r] * op.x_nb1) + b[r] * 64 + 4 * h;
            if (r < rounds) {
                const bool kept = NORM && r == 0 && tb0 == 2 * cw + hw;  // loaded by the first pass
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    v[r][k] = !act[r] ? make_float4(0.f, 0.f, 0.f, 0.f) : (kept ? keep_x[k] : __ldg(xv + k));
                if constexpr (GLU) {
                    const float4* uv = reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(nrm.up) +
                                                                       t[r] * nrm.up_nb1) + b[r] * 64 + 4 * h;
#pragma unroll
                    for (int k = 0; k < 4; ++k) uq[r][k] = act[r] ? __ldg(uv + k) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        if constexpr (GLU) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r >= rounds) continue;
#pragma unroll
                for (int k = 0; k < 4; ++k) v[r][k] = glu4<PRO>(v[r][k], uq[r][k]);
            }
        }
        if constexpr (NORM) {
            // (x * inv_rms) * gain: the reference's two ops, in order (after
            // both rounds' loads are issued)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r >= rounds || !act[r]) continue;
                const float sc = t[r] == 0 ? inv[0] : (t[r] == 1 ? inv[1] : (t[r] == 2 ? inv[2] : inv[3]));
                const float4* gv = reinterpret_cast<const float4*>(nrm.gain) + b[r] * 64 + 4 * h;
                const bool kept = r == 0 && tb0 == 2 * cw + hw;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 gk = !nrm.gain ? make_float4(1.f, 1.f, 1.f, 1.f) : (kept ? keep_g[k] : __ldg(gv + k));
                    v[r][k] = make_float4(__fmul_rn(__fmul_rn(v[r][k].x, sc), gk.x),
                                          __fmul_rn(__fmul_rn(v[r][k].y, sc), gk.y),
                                          __fmul_rn(__fmul_rn(v[r][k].z, sc), gk.z),
                                          __fmul_rn(__fmul_rn(v[r][k].w, sc), gk.w));
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            if (r >= rounds) break;
            float mx = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[r][k].x), fabsf(v[r][k].y)),
                                     fmaxf(fabsf(v[r][k].z), fabsf(v[r][k].w))));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));  // within the half
            const float sc = mx > 0.f ? 127.f / mx : 0.f;
            // l0 = rint(x s) (|l0| <= 127), l1 = rint(r1) with r1 = 128 (x s - l0)
            // (|l1| <= 65), l2 = rint(128 (r1 - l1)) (|l2| <= 64). fmaf takes the
            // exact product x s; r1 - l1 and the scalings by 128 are exact.
            uint32_t p0[4], p1[4], p2[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float e[4] = {v[r][k].x, v[r][k].y, v[r][k].z, v[r][k].w};
                int b0[4], b1[4], b2[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float l0, l1, l2;
                    b0[j] = round_low_byte(__fmul_rn(e[j], sc), l0);
                    const float r1 = fmaf(e[j], sc, -l0) * 128.f;
                    b1[j] = round_low_byte(r1, l1);
                    b2[j] = round_low_byte(__fsub_rn(r1, l1) * 128.f, l2);
                }
                p0[k] = pack_b4(b0[0], b0[1], b0[2], b0[3]);
                p1[k] = pack_b4(b1[0], b1[1], b1[2], b1[3]);
                p2[k] = pack_b4(b2[0], b2[1], b2[2], b2[3]);
            }
            float a16 = 0.f;  // a lane's 16 elements: one Q6_K sub-block
#pragma unroll
            for (int k = 0; k < 4; ++k) a16 += (v[r][k].x + v[r][k].y) + (v[r][k].z + v[r][k].w);
            const float a = a16 + __shfl_xor_sync(0xffffffffu, a16, 1);  // a Q4_K sub-block is two lanes
            if (act[r]) {
                const int tt = t[r], bb = b[r];
                uint8_t* c0 = xsm + (kLimbs * tt) * XS + bb * 256 + 16 * h;
                *reinterpret_cast<uint4*>(c0) = make_uint4(p0[0], p0[1], p0[2], p0[3]);
                *reinterpret_cast<uint4*>(c0 + XS) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
                *reinterpret_cast<uint4*>(c0 + 2 * XS) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
                X16[tt * (K / 16) + bb * 16 + h] = a16;
                if ((h & 1) == 0) Xs[tt * (K / 32) + bb * 8 + (h >> 1)] = a;
                if (h == 0) dfac[tt * nblk + bb] = mx * (1.f / 2032.f);  // 1 / (16 s)
            }
        }
    }
    consumers_sync();
}

// Where a unit's rows go; written and read by the unit's owner warp only.
struct UnitMeta {
    float* y;        // first output row of the unit, vector 0
    int64_t y_nb1;   // bytes between vectors
    int32_t rows;    // valid rows (<= 16)
    int32_t n;       // vectors
    int32_t op;      // the unit's op (for the other ranks' copies)
    int32_t r0;      // the unit's first row
};

// Stage-ring position of the consumer warps.
struct Ring {
    uint8_t* stages;
    uint64_t* full;
    uint64_t* empty;
    volatile int* poisoned;
    int SB, S;
    int slot;
    uint32_t phase;
    uint32_t item_base;  // items of the CTA's sequence before the current segment
    __device__ __forceinline__ void advance() {
        if (++slot == S) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

// Per-op constants of a consumer lane on the Q4_K path (see q4k_items), for
// one vector pair: NP = 1 (one vector) or 2 (vectors 2G, 2G + 1).
struct Q4Lane {
    uint32_t wl;        // weights ldmatrix row offset in a stage
    uint32_t xcol;      // activations ldmatrix row address (block 0, pair 0)
    bool xv0, xv1;      // that row is real (not the zero row) for even / odd pairs
    const float* dfac;  // d-factors of vector tk
    const float* Xs;    // sub-block sums of vector tk
    int sl, tk, hl;     // slot, vector and limb half of the lane's accumulator columns
};

// B column rr of an MMA (0..7) is limb rr & 3 (3: the zero column) of pair
// rr >> 2: slot rr >> 2 of vector 2G at NP = 1, vector 2G + (rr >> 2) at NP = 2.
template <int NP>
__device__ __forceinline__ Q4Lane q4k_lane(const OpInfo& op, const uint8_t* xsm, int lane, int G) {
    constexpr int NS = NP == 1 ? 2 : 1;
    const int K = op.K, N = op.N, XS = img_col_bytes(K), nblocks = K / 256;
    const int c = lane & 3;
    Q4Lane q;
    q.sl = NP == 1 ? c >> 1 : 0;
    q.tk = (NP == 1 ? 0 : c >> 1) + 2 * G;
    q.hl = c & 1;
    // weights ldmatrix: matrix lane/8 = rows 0-7 / 8-15 of the pair's 16-byte chunk 0 / 1
    q.wl = static_cast<uint32_t>(((lane & 7) + 8 * ((lane >> 3) & 1)) * op.wbox + 16 + 16 * (lane >> 4));
    // activations ldmatrix: matrix mi = lane/8 (0, 1: b0, b1 of the low-nibble
    // sub-block of a pair; 2, 3: of the high one), row rr = lane%8 = B column
    const int mi = lane >> 3, rr = lane & 7;
    const int u_r = rr >> 2, l_r = rr & 3;
    const int slot_r = NP == 1 ? u_r : 0, t_r = (NP == 1 ? 0 : u_r) + 2 * G;
    const bool real = l_r < kLimbs && t_r < N;
    q.xv0 = real && slot_r == (mi >> 1) % NS;        // even pairs
    q.xv1 = real && slot_r == (2 + (mi >> 1)) % NS;  // odd pairs
    q.xcol = smem_u32(xsm) + static_cast<uint32_t>((kLimbs * (real ? t_r : 0) + (real ? l_r : 0)) * XS + 16 * mi);
    const int tkc = q.tk < N ? q.tk : 0;
    q.dfac = reinterpret_cast<const float*>(xsm + img_inv_off(K, N)) + tkc * nblocks;
    q.Xs = reinterpret_cast<const float*>(xsm + img_sum_off(K, N)) + tkc * (K / 32);
    return q;
}

// Per-op constants of a consumer lane on the Q6_K path (see q6k_item), for
// one vector pair as in q4k_lane.
struct Q6Lane {
    uint32_t xcol;      // activations ldmatrix row address (block 0, pair 0)
    bool xv;            // that row is real (not the zero row)
    const float* dfac;  // d-factors of vector tk
    const float* X16;   // 16-element sub-block sums of vector tk
    int sl, tk, hl;     // slot, vector and limb half of the lane's accumulator columns
};

template <int NP>
__device__ __forceinline__ Q6Lane q6k_lane(const OpInfo& op, const uint8_t* xsm, int lane, int G) {
    constexpr int NS = NP == 1 ? 2 : 1;
    const int K = op.K, N = op.N, XS = img_col_bytes(K);
    const int c = lane & 3;
    Q6Lane q;
    q.sl = NP == 1 ? c >> 1 : 0;
    q.tk = (NP == 1 ? 0 : c >> 1) + 2 * G;
    q.hl = c & 1;
    // matrix mi = lane/8 of a pair's ldmatrix is sub-block 4p + mi (k half
    // mi&1 of MMA 2p + mi/2), slot mi % NS; row rr = lane%8 = B column
    const int mi = lane >> 3, rr = lane & 7;
    const int u_r = rr >> 2, l_r = rr & 3;
    const int slot_r = NP == 1 ? u_r : 0, t_r = (NP == 1 ? 0 : u_r) + 2 * G;
    const bool real = l_r < kLimbs && t_r < N;
    q.xv = real && slot_r == mi % NS;
    q.xcol = smem_u32(xsm) + static_cast<uint32_t>((kLimbs * (real ? t_r : 0) + (real ? l_r : 0)) * XS + 16 * mi);
    const int tkc = q.tk < N ? q.tk : 0;
    q.dfac = reinterpret_cast<const float*>(xsm + img_inv_off(K, N)) + tkc * (K / 256);
    q.X16 = reinterpret_cast<const float*>(xsm + img_sum16_off(K, N)) + tkc * (K / 16);
    return q;
}

// Warp-wide bounded wait on an mbarrier phase (see ring_wait).
__device__ __forceinline__ void ring_barrier_wait(uint64_t* bar, uint32_t parity, volatile int* poisoned, int lane) {
    if (mbar_test_wait(bar, parity)) return;
    mbar_wait_warp(bar, parity, 4u, poisoned, lane);
}

// Waits for the current stage of the ring (warp-wide): a non-blocking test
// first, then lane 0 polls with a short back-off, then every lane observes
// the completed phase itself (ordering the landed copy's bytes before its
// reads).
__device__ __forceinline__ void ring_wait(Ring& R, int lane) {
    if (mbar_test_wait(&R.full[R.slot], R.phase)) return;
    mbar_wait_warp(&R.full[R.slot], R.phase, 2u, R.poisoned, lane);
}

// Sums a lane's partial rows over the lanes of its vector and writes them to
// the warp's unit buffer: at one vector all four lanes of a row group hold
// parts of it (two slots x two limb halves), at two or four the lane pair
// 2u, 2u + 1 (two limb halves).
template <int NP, int NT, int NG>
__device__ __forceinline__ void write_partials(float (&yg)[NG], float (&yh)[NG], const int (&tk)[NG], int N, int lane,
                                               float* ub) {
    const int g = lane >> 2;
#pragma unroll
    for (int G = 0; G < NG; ++G) {
        yg[G] += __shfl_xor_sync(0xffffffffu, yg[G], 1);
        yh[G] += __shfl_xor_sync(0xffffffffu, yh[G], 1);
        if (NP == 1) {
            yg[G] += __shfl_xor_sync(0xffffffffu, yg[G], 2);
            yh[G] += __shfl_xor_sync(0xffffffffu, yh[G], 2);
        }
        const bool writer = NP == 1 ? (lane & 3) == 0 : (lane & 1) == 0;
        if (writer && tk[G] < N) {
            ub[g * NT + tk[G]] = yg[G];
            ub[(g + 8) * NT + tk[G]] = yh[G];
        }
    }
}

// All segments of one Q4_K (Q5_K with Q5 = true) unit for this consumer
// warp; writes the warp's partial sums of the unit's 16 rows (zeros where it
// had no item) to ub. Four vectors take two passes over each item, one per
// vector pair (qa, qb).
template <int NP, int NT, bool Q5>
__device__ __forceinline__ void q4k_unit(const OpRegs& op, const Q4Lane& qa, const Q4Lane& qb, Ring& R,
                                         uint32_t xzero, int lane, int cw, float* ub) {
    constexpr int NPI = NP == 1 ? 1 : 2;  // vectors per pass
    constexpr int NG = NP == 4 ? 2 : 1;   // passes
    constexpr int BB = Q5 ? 176 : 144;
    const int N = op.N, nblocks = op.K / 256;
    const int g = lane >> 2;
    const Q4Lane qs[2] = {qa, qb};
    float yg[NG], yh[NG];  // the lane's columns of rows g and g + 8, per pass
#pragma unroll
    for (int G = 0; G < NG; ++G) yg[G] = yh[G] = 0.f;
    for (int sg = 0; sg < op.nseg; ++sg) {
        const int b0 = sg * op.seg_blocks;
        const int nb = min(op.seg_blocks, nblocks - b0);
        // this warp's first item of the segment; a warp without one neither
        // waits for nor releases the stage (the warp with item 0 releases it
        // for them)
        const int i0 = (cw - static_cast<int>(R.item_base % kCW) + kCW) % kCW;
        if (i0 < nb) {
            ring_wait(R, lane);
            const uint8_t* stage = R.stages + R.slot * R.SB;
            int i = i0;
            // item pairs at N = 1 (at N = 2 the doubled accumulators would spill)
            for (; NP == 1 && i + kCW < nb; i += 2 * kCW) {
                const int bg = b0 + i;
                const Q4Lane& q = qs[0];
                if (Q5)
                    q5k_items<1, 2>(stage + i * BB, op.wbox, q.wl, q.xcol + bg * 256, xzero, q.xv0, q.xv1,
                                    q.dfac + bg, q.Xs + bg * 8, g, q.sl, q.hl, yg[0], yh[0]);
                else
                    q4k_items<1, 2>(stage + i * BB, op.wbox, q.wl, q.xcol + bg * 256, xzero, q.xv0, q.xv1,
                                    q.dfac + bg, q.Xs + bg * 8, g, q.sl, q.hl, yg[0], yh[0]);
            }
            for (; i < nb; i += kCW) {
                const int bg = b0 + i;
#pragma unroll
                for (int G = 0; G < NG; ++G) {
                    const Q4Lane& q = qs[G];
                    if (Q5)
                        q5k_items<NPI, 1>(stage + i * BB, op.wbox, q.wl, q.xcol + bg * 256, xzero, q.xv0, q.xv1,
                                          q.dfac + bg, q.Xs + bg * 8, g, q.sl, q.hl, yg[G], yh[G]);
                    else
                        q4k_items<NPI, 1>(stage + i * BB, op.wbox, q.wl, q.xcol + bg * 256, xzero, q.xv0, q.xv1,
                                          q.dfac + bg, q.Xs + bg * 8, g, q.sl, q.hl, yg[G], yh[G]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&R.empty[R.slot], i0 == 0 ? 1u + kCW - min(nb, kCW) : 1u);
        }
        R.item_base += nb;
        R.advance();
    }
    int tk[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) tk[G] = qs[G].tk;
    write_partials<NP, NT, NG>(yg, yh, tk, N, lane, ub);
}

// All segments of one Q6_K unit for this consumer warp (see q4k_unit). Each
// row's copy window starts at its segment start rounded down to 16 bytes;
// glo is the low word of the unit's first row address.
template <int NP, int NT>
__device__ __forceinline__ void q6k_unit(const OpRegs& op, const Q6Lane& qa, const Q6Lane& qb, Ring& R,
                                         uint32_t xzero, uint32_t glo, int lane, int cw, float* ub) {
    constexpr int NPI = NP == 1 ? 1 : 2;  // vectors per pass
    constexpr int NG = NP == 4 ? 2 : 1;   // passes
    const int N = op.N, nblocks = op.K / 256;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t nb1 = static_cast<uint32_t>(op.w_nb1);
    const Q6Lane qs[2] = {qa, qb};
    float yg[NG], yh[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) yg[G] = yh[G] = 0.f;
    for (int sg = 0; sg < op.nseg; ++sg) {
        const int b0 = sg * op.seg_blocks;
        const int nb = min(op.seg_blocks, nblocks - b0);
        const int i0 = (cw - static_cast<int>(R.item_base % kCW) + kCW) % kCW;
        if (i0 < nb) {
            ring_wait(R, lane);
            const uint8_t* stage = R.stages + R.slot * R.SB;
            const uint32_t gl = glo + static_cast<uint32_t>(b0 * 210);
            const uint8_t* pg = stage + g * op.wbox + ((gl + static_cast<uint32_t>(g) * nb1) & 15u);
            const uint8_t* ph = stage + (g + 8) * op.wbox + ((gl + static_cast<uint32_t>(g + 8) * nb1) & 15u);
            for (int i = i0; i < nb; i += kCW) {
                const int bg = b0 + i;
#pragma unroll
                for (int G = 0; G < NG; ++G) {
                    const Q6Lane& q = qs[G];
                    q6k_item<NPI>(pg + i * 210, ph + i * 210, q.xcol + bg * 256, xzero, q.xv, 16.f * q.dfac[bg],
                                  q.X16 + bg * 16, c, q.sl, q.hl, yg[G], yh[G]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&R.empty[R.slot], i0 == 0 ? 1u + kCW - min(nb, kCW) : 1u);
        }
        R.item_base += nb;
        R.advance();
    }
    int tk[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) tk[G] = qs[G].tk;
    write_partials<NP, NT, NG>(yg, yh, tk, N, lane, ub);
}

// One thread: every other rank's count of this rank's sync points goes up by
// one with a system-scope release reduction, which orders before it all that
// this rank wrote earlier (all earlier kernels' row stores into other ranks'
// memory, ordered before this thread by the stream or the dependency wait).
__device__ void tp_signal_peers(uint32_t* const* sig, int world, int rank) {
    for (int p = 0; p < world; ++p)
        if (p != rank) asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(sig[p] + rank) : "memory");
}

// Bounded wait (one thread) until every other rank has signalled `seq`
// sync points to this rank; false (and an error code) on time-out.
__device__ bool tp_wait_peers(const uint32_t* const* sig, int world, int rank, uint32_t seq, volatile int* poisoned,
                              uint32_t lim) {
    for (int src = 0; src < world; ++src) {
        if (src == rank) continue;
        const uint32_t* f = sig[rank] + src;
        uint32_t v;
        uint32_t i = 0;
        for (;; ++i) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (static_cast<int32_t>(v - seq) >= 0) break;
            if (i == lim || (poisoned && *poisoned)) {
                if (poisoned) *poisoned = 1;
                atomicOr(&g_stream_error, 4u);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

// All segments of one Q8_0 / Q4_0 unit for this consumer warp (see
// q6k_unit); an item is a group of 8 blocks (segments hold whole groups).
template <int NP, int NT, int TYPE>
__device__ __forceinline__ void q8_unit(const OpRegs& op, const Q4Lane& qa, const Q4Lane& qb, Ring& R,
                                        uint32_t xzero, uint32_t glo, int lane, int cw, float* ub) {
    constexpr int NPI = NP == 1 ? 1 : 2;  // vectors per pass
    constexpr int NG = NP == 4 ? 2 : 1;   // passes
    constexpr int BB = TYPE == kTypeQ4_0 ? 18 : 34;  // block bytes
    const int N = op.N, nblocks = op.K / 32;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t nb1 = static_cast<uint32_t>(op.w_nb1);
    const Q4Lane qs[2] = {qa, qb};
    float yg[NG], yh[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) yg[G] = yh[G] = 0.f;
    for (int sg = 0; sg < op.nseg; ++sg) {
        const int b0 = sg * op.seg_blocks;
        const int ng = (min(op.seg_blocks, nblocks - b0) + 7) / 8;  // groups of this segment
        const int i0 = (cw - static_cast<int>(R.item_base % kCW) + kCW) % kCW;
        if (i0 < ng) {
            ring_wait(R, lane);
            const uint8_t* stage = R.stages + R.slot * R.SB;
            const uint32_t gl = glo + static_cast<uint32_t>(b0 * BB);
            const uint8_t* pg = stage + g * op.wbox + ((gl + static_cast<uint32_t>(g) * nb1) & 15u);
            const uint8_t* ph = stage + (g + 8) * op.wbox + ((gl + static_cast<uint32_t>(g + 8) * nb1) & 15u);
            for (int i = i0; i < ng; i += kCW) {
                const int gg = b0 / 8 + i;  // 256-element group
#pragma unroll
                for (int G = 0; G < NG; ++G) {
                    const Q4Lane& q = qs[G];
                    q8_item<NPI, TYPE>(pg + i * 8 * BB, ph + i * 8 * BB, q.xcol + gg * 256, xzero, q.xv0, q.xv1,
                                       16.f * q.dfac[gg], c, q.sl, q.hl, yg[G], yh[G]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&R.empty[R.slot], i0 == 0 ? 1u + kCW - min(ng, kCW) : 1u);
        }
        R.item_base += ng;
        R.advance();
    }
    int tk[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) tk[G] = qs[G].tk;
    write_partials<NP, NT, NG>(yg, yh, tk, N, lane, ub);
}

// All segments of one IQ4_XS unit for this consumer warp (see q6k_unit): an
// item is one block.
template <int NP, int NT>
__device__ __forceinline__ void iq4xs_unit(const OpRegs& op, const Q4Lane& qa, const Q4Lane& qb, Ring& R,
                                           uint32_t xzero, uint32_t glo, int lane, int cw, float* ub) {
    constexpr int NPI = NP == 1 ? 1 : 2;  // vectors per pass
    constexpr int NG = NP == 4 ? 2 : 1;   // passes
    const int N = op.N, nblocks = op.K / 256;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t nb1 = static_cast<uint32_t>(op.w_nb1);
    const Q4Lane qs[2] = {qa, qb};
    float yg[NG], yh[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) yg[G] = yh[G] = 0.f;
    for (int sg = 0; sg < op.nseg; ++sg) {
        const int b0 = sg * op.seg_blocks;
        const int nb = min(op.seg_blocks, nblocks - b0);
        const int i0 = (cw - static_cast<int>(R.item_base % kCW) + kCW) % kCW;
        if (i0 < nb) {
            ring_wait(R, lane);
            const uint8_t* stage = R.stages + R.slot * R.SB;
            const uint32_t gl = glo + static_cast<uint32_t>(b0 * 136);
            const uint8_t* pg = stage + g * op.wbox + ((gl + static_cast<uint32_t>(g) * nb1) & 15u);
            const uint8_t* ph = stage + (g + 8) * op.wbox + ((gl + static_cast<uint32_t>(g + 8) * nb1) & 15u);
            for (int i = i0; i < nb; i += kCW) {
                const int bg = b0 + i;
#pragma unroll
                for (int G = 0; G < NG; ++G) {
                    const Q4Lane& q = qs[G];
                    iq4xs_item<NPI>(pg + i * 136, ph + i * 136, q.xcol + bg * 256, xzero, q.xv0, q.xv1,
                                    16.f * q.dfac[bg], c, q.sl, q.hl, yg[G], yh[G]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cnt(&R.empty[R.slot], i0 == 0 ? 1u + kCW - min(nb, kCW) : 1u);
        }
        R.item_base += nb;
        R.advance();
    }
    int tk[NG];
#pragma unroll
    for (int G = 0; G < NG; ++G) tk[G] = qs[G].tk;
    write_partials<NP, NT, NG>(yg, yh, tk, N, lane, ub);
}

// PRO: the fused activation prologue (kProNone for the plain GEMV; each kind
// is a separate instantiation, so the plain GEMV carries none of their code).
template <int NT, int PRO>
__global__ void __launch_bounds__(kThreads, 1) stream_gemv_kernel(const __grid_constant__ SList L) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = L.stages;
    const int SB = L.stage_bytes;
    uint8_t* stages = smem;
    uint8_t* xsm = smem + S * SB;
    uint8_t* zrow = xsm + L.x_bytes;                                     // 16 zero bytes: the Q4_K MMA's empty B rows
    float* ubuf = reinterpret_cast<float*>(zrow + 16);                   // [kUnitSlots][kCW][16][NT]
    UnitMeta* umeta = reinterpret_cast<UnitMeta*>(ubuf + kUnitSlots * kCW * kRows * NT);  // [kUnitSlots]
    uint64_t* ubar = reinterpret_cast<uint64_t*>(umeta + kUnitSlots);    // [kUnitSlots]: all warps' partials written
    uint64_t* full = ubar + kUnitSlots;
    uint64_t* empty = full + kMaxStages;
    uint64_t* xready = empty + kMaxStages;  // the first activation image is staged
    volatile int* poisoned = reinterpret_cast<volatile int*>(xready + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(zrow)[threadIdx.x] = 0u;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        for (int s = 0; s < kUnitSlots; ++s) mbar_init(&ubar[s], kCW);
        mbar_init(xready, 1);
        *poisoned = 0;
        reinterpret_cast<volatile uint32_t*>(poisoned)[1] = L.spin_limit;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __shared__ OpTable T;
    __shared__ float nred[kCW][kMaxNT];  // fused RMS_NORM: per-warp sums of x^2
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
        for (int r = 0; r < kMaxRanks; ++r) d.y_peer[r] = o.y_peer[r];
        if (o.use_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&o.tmap) : "memory");
    }
    if (threadIdx.x == 0) {
        T.n_ops = L.n_ops;
        T.pro = L.pro;
        T.total_units = L.total_units;
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // Boxes issued before the first activation image is staged. A fused GLU's
    // staging is SFU-bound after its loads, so the whole ring may go first
    // (measured 0.2 us faster on a Q6_K 3072 x 8192 down projection; the
    // RMS_NORM's two load passes were 0.8 us slower with it).
    constexpr int pre = PRO == kProSwiglu || PRO == kProGelu ? kMaxStages : kPreStages;
    if (warp == 0 && L.all_tma) {
        // ---------------- copy warp, tensor-map path: lane 0 alone ----------------
        // One thread issues every box: a warp-wide loop (shuffles, reconvergence)
        // was measured to double the time between two issues.
        if (lane != 0) return;
        const uint64_t policy = evict_first_policy();
        const int n_ops = T.n_ops, total = T.total_units;
        int u = blockIdx.x, oi = 0;
        while (oi + 1 < n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
        int s = 0, issued = 0;
        uint32_t phase = 1;  // the first pass finds every slot free
        uint32_t issued_mask = 0, par_mask = 0;  // for drain_copies
        bool stop = false;
        for (; u < total && !stop; u += gridDim.x) {
            while (oi + 1 < n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
            const OpInfo& op = T.op[oi];
            const int bb = block_bytes_of(op.type), nseg = op.nseg, step = op.seg_blocks * bb;
            const uint32_t box = static_cast<uint32_t>(kRows * op.wbox);
            const int r0 = (u - op.unit_begin) * kRows;
            const CUtensorMap* tm = &L.op[oi].tmap;
            for (int sg = 0, col = 0; sg < nseg; ++sg, col += step) {
                if (!mbar_wait(&empty[s], phase, 1u, poisoned) ||
                    (issued++ == pre && !mbar_wait(xready, 0u, 3u, poisoned))) {
                    stop = true;
                    break;
                }
                // one box: 16 rows x wbox bytes from the 16-byte-aligned column at or
                // below the segment start (rows past M and columns past the row end
                // read as zeros)
                mbar_arrive_expect_tx(&full[s], box);
                tma_2d_g2s(stages + s * SB, tm, (col & ~15) / 8, r0, &full[s], policy);
                issued_mask |= 1u << s;
                par_mask = (par_mask & ~(1u << s)) | (((phase ^ 1u) & 1u) << s);
                if (++s == S) {
                    s = 0;
                    phase ^= 1u;
                }
            }
        }
        drain_copies(full, S, issued_mask, par_mask, poisoned);
        return;
    }
    if (warp == 0) {
        // ---------------- copy warp, any op copied row by row ----------------
        // The op's fields live in registers and are reloaded only when the op
        // changes: every shared-memory access here competes with the
        // consumers' traffic.
        const uint64_t policy = evict_first_policy();
        const int n_ops = T.n_ops, total = T.total_units;
        int u = blockIdx.x, oi = 0;
        while (oi + 1 < n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
        int s = 0, issued = 0;
        uint32_t phase = 1;  // the first pass finds every slot free
        uint32_t issued_mask = 0, par_mask = 0;  // for drain_copies
        for (; u < total; u += gridDim.x) {
            while (oi + 1 < n_ops && u >= T.op[oi + 1].unit_begin) ++oi;
            const OpInfo& op = T.op[oi];
            const int bb = block_bytes_of(op.type), nseg = op.nseg, seg_blocks = op.seg_blocks, wbox = op.wbox;
            const int r0 = (u - op.unit_begin) * kRows;
            const bool tma = op.use_tma != 0;
            const CUtensorMap* tm = &L.op[oi].tmap;
            const int nblocks = op.K / block_elems_of(op.type), nrows = min(kRows, op.M - r0);
            const uint8_t* wrow = op.w + static_cast<int64_t>(r0 + (lane < nrows ? lane : 0)) * op.w_nb1;
            bool stop = false;
            for (int sg = 0; sg < nseg; ++sg) {
                int ok = 0;
                if (lane == 0) {
                    ok = mbar_wait(&empty[s], phase, 1u, poisoned);
                    if (ok && issued == pre) ok = mbar_wait(xready, 0u, 3u, poisoned);
                }
                ++issued;
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    stop = true;
                    break;
                }
                const int b0 = sg * seg_blocks;
                uint8_t* dst = stages + s * SB;
                if (tma) {
                    // one box: 16 rows x wbox bytes from the 16-byte-aligned column at
                    // or below the segment start (rows past M and columns past the row
                    // end read as zeros)
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(kRows * wbox));
                        tma_2d_g2s(dst, tm, ((b0 * bb) & ~15) / 8, r0, &full[s], policy);
                    }
                } else {
                    // one bulk copy per row: the row's segment rounded out to 16 bytes
                    const bool active = lane < nrows;
                    const int nbytes = min(seg_blocks, nblocks - b0) * bb;
                    const uintptr_t g = reinterpret_cast<uintptr_t>(wrow + b0 * bb);
                    const uintptr_t ga = g & ~uintptr_t(15);
                    const uint32_t bytes = active ? static_cast<uint32_t>(((g + nbytes + 15) & ~uintptr_t(15)) - ga) : 0u;
                    const uint32_t sum = __reduce_add_sync(0xffffffffu, bytes);
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], sum);
                    __syncwarp();
                    if (active) bulk_g2s(dst + lane * wbox, reinterpret_cast<const void*>(ga), bytes, &full[s], policy);
                }
                issued_mask |= 1u << s;
                par_mask = (par_mask & ~(1u << s)) | (((phase ^ 1u) & 1u) << s);
                if (++s == S) {
                    s = 0;
                    phase ^= 1u;
                }
            }
            if (stop) break;
        }
        if (lane == 0) drain_copies(full, S, issued_mask, par_mask, poisoned);
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ct = threadIdx.x - 32;  // 0 .. 32 kCW - 1
    const int cw = warp - 1;          // 0 .. kCW - 1
    // Row-sharded: this launch is sync point `tp_seq` of the rank. CTA 0
    // tells the other ranks that the rank's earlier launches are complete (the
    // dependency wait above covers them), and every CTA waits until all ranks
    // have reached this sync point, so their earlier rows have landed here
    // before any activation is read (the first staging's barrier makes every
    // consumer thread wait for thread 0).
    uint32_t tp_seq = 0;
    if (L.tp.world > 1 && ct == 0) {
        tp_seq = *reinterpret_cast<volatile uint32_t*>(L.tp.state + 1);
        if (blockIdx.x == 0) tp_signal_peers(L.tp.sig, L.tp.world, L.tp.rank);
        tp_wait_peers(L.tp.sig, L.tp.world, L.tp.rank, tp_seq + 1u, poisoned, L.spin_limit);
    }
    Ring R{stages, full, empty, poisoned, SB, S, 0, 0u, 0u};
    const int n_ops = T.n_ops, total = T.total_units;
    int staged = -1, oi = -1, useq = 0;
    int next_begin = -1;     // first unit of the next op
    int uslot = 0, own = 0;  // useq % kUnitSlots, useq % kCW
    OpRegs op{};
    Q4Lane q4{}, q4b{};  // vector pairs 0 and 1 (the second only at 3 or 4 vectors)
    Q6Lane q6{}, q6b{};
    // Sums the 8 warps' partials of this CTA's unit number j (fixed order:
    // deterministic) and writes its rows; done by the unit's owner warp
    // kRedDelay units later, when the other warps are normally long done.
    auto reduce_unit = [&](int j) {
        const int slot = j % kUnitSlots;
        ring_barrier_wait(&ubar[slot], static_cast<uint32_t>(j / kUnitSlots) & 1u, poisoned, lane);
        const UnitMeta m = umeta[slot];
        for (int e = lane; e < kRows * m.n; e += 32) {  // (two rounds at 3 or 4 vectors)
            const int r = e / m.n, n = e - r * m.n;
            const float* vb = ubuf + slot * kCW * kRows * NT + r * NT + n;
            float v = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < kCW; ++w2) v += vb[w2 * kRows * NT];
            if (r < m.rows) {
                *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(m.y) + n * m.y_nb1 + 4 * r) = v;
                // row-sharded: the same row into every other rank's copy (NVLink stores)
                for (int p = 0; p < L.tp.world; ++p) {
                    float* yp = T.op[m.op].y_peer[p];
                    if (p != L.tp.rank && yp)
                        *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(yp) + n * m.y_nb1 + 4LL * (m.r0 + r)) = v;
                }
            }
        }
    };
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++useq) {
        if (u >= next_begin) {
            // ---- next op: activation image (re)built when x or its layout changes ----
            do {
                ++oi;
            } while (oi + 1 < n_ops && u >= T.op[oi + 1].unit_begin);
            const OpInfo& oo = T.op[oi];
            if (staged < 0 || T.op[staged].x != oo.x || T.op[staged].K != oo.K || T.op[staged].N != oo.N ||
                T.op[staged].x_nb1 != oo.x_nb1) {
                consumers_sync();  // nobody still reads the previous image
                stage_activations<PRO>(oo, xsm, lane, cw, T.pro, nred);
                if (ct == 0 && useq == 0) mbar_arrive_cnt(xready, 1u);  // the copy warp may go on
                staged = oi;
            }
            const bool one = NT == 1 || oo.N == 1;
            if (oo.type != kTypeQ6_K) {
                q4 = one ? q4k_lane<1>(oo, xsm, lane, 0) : q4k_lane<2>(oo, xsm, lane, 0);
                if (NT == 4 && oo.N > 2) q4b = q4k_lane<2>(oo, xsm, lane, 1);
            } else {
                q6 = one ? q6k_lane<1>(oo, xsm, lane, 0) : q6k_lane<2>(oo, xsm, lane, 0);
                if (NT == 4 && oo.N > 2) q6b = q6k_lane<2>(oo, xsm, lane, 1);
            }
            op = op_regs(oo);
            next_begin = oi + 1 < n_ops ? T.op[oi + 1].unit_begin : total;
        }
        const int N = op.N, K = op.K;
        const int bb = block_bytes_of(op.type);
        const int nblocks = K / block_elems_of(op.type);
        const int r0 = (u - op.unit_begin) * kRows;
        // this warp's partial sums of the unit: every warp writes all 16 rows
        float* ub = ubuf + (uslot * kCW + cw) * kRows * NT;

        if (op.type == kTypeQ4_K) {
            // ================= Q4_K, integer tensor cores =================
            if (NT == 1 || N == 1)
                q4k_unit<1, NT, false>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
            else if (NT == 2 || N == 2)
                q4k_unit<2, NT, false>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
            else if constexpr (NT == 4)
                q4k_unit<4, NT, false>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
        } else if (op.type == kTypeQ5_K) {
            // ================= Q5_K, integer tensor cores =================
            if (NT == 1 || N == 1)
                q4k_unit<1, NT, true>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
            else if (NT == 2 || N == 2)
                q4k_unit<2, NT, true>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
            else if constexpr (NT == 4)
                q4k_unit<4, NT, true>(op, q4, q4b, R, smem_u32(zrow), lane, cw, ub);
        } else if (op.type == kTypeQ6_K) {
            // ================= Q6_K, integer tensor cores =================
            const uint32_t glo =
                static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0) * op.w_nb1));
            if (NT == 1 || N == 1)
                q6k_unit<1, NT>(op, q6, q6b, R, smem_u32(zrow), glo, lane, cw, ub);
            else if (NT == 2 || N == 2)
                q6k_unit<2, NT>(op, q6, q6b, R, smem_u32(zrow), glo, lane, cw, ub);
            else if constexpr (NT == 4)
                q6k_unit<4, NT>(op, q6, q6b, R, smem_u32(zrow), glo, lane, cw, ub);
        } else if (op.type == kTypeIQ4_XS) {
            // ================= IQ4_XS, integer tensor cores =================
            const uint32_t glo =
                static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0) * op.w_nb1));
            if (NT == 1 || N == 1)
                iq4xs_unit<1, NT>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
            else if (NT == 2 || N == 2)
                iq4xs_unit<2, NT>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
            else if constexpr (NT == 4)
                iq4xs_unit<4, NT>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
        } else {
            // ============= Q8_0 / Q4_0, integer tensor cores =============
            const uint32_t glo =
                static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0) * op.w_nb1));
            if (op.type == kTypeQ4_0) {
                if (NT == 1 || N == 1)
                    q8_unit<1, NT, kTypeQ4_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
                else if (NT == 2 || N == 2)
                    q8_unit<2, NT, kTypeQ4_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
                else if constexpr (NT == 4)
                    q8_unit<4, NT, kTypeQ4_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
            } else {
                if (NT == 1 || N == 1)
                    q8_unit<1, NT, kTypeQ8_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
                else if (NT == 2 || N == 2)
                    q8_unit<2, NT, kTypeQ8_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
                else if constexpr (NT == 4)
                    q8_unit<4, NT, kTypeQ8_0>(op, q4, q4b, R, smem_u32(zrow), glo, lane, cw, ub);
            }
        }
        // ---- unit hand-off: publish this warp's partials; the owner sums them later ----
        if (own == cw && lane == 0) {
            UnitMeta m;
            m.y = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(op.y) + 4LL * r0);
            m.y_nb1 = op.y_nb1;
            m.rows = min(kRows, op.M - r0);
            m.n = N;
            m.op = oi;
            m.r0 = r0;
            umeta[uslot] = m;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(&ubar[uslot], 1u);  // release: the warp's partial writes precede it
        if (useq >= kRedDelay && ((own - kRedDelay) & (kCW - 1)) == cw) reduce_unit(useq - kRedDelay);
        if (++uslot == kUnitSlots) uslot = 0;
        own = (own + 1) & (kCW - 1);
    }
    // the last kRedDelay units of the CTA
    for (int j = useq - kRedDelay; j < useq; ++j)
        if (j >= 0 && j % kCW == cw) reduce_unit(j);
    if (L.tp.world > 1 && ct == 0) {
        // Row-sharded: the last CTA to finish counts the sync point (every CTA
        // read the count at its start, before this).
        const unsigned prev = atomicAdd(L.tp.state, 1u);
        if (prev == gridDim.x - 1) {
            L.tp.state[0] = 0u;
            L.tp.state[1] = tp_seq + 1u;
        }
    }
}

// A sync point on its own: the rank's earlier row-sharded launches are
// complete (stream order); after it every rank's rows are in place here.
__global__ void tp_wait_kernel(const __grid_constant__ TpSig t) {
    if (threadIdx.x == 0) {
        const uint32_t seq = t.state[1];
        tp_signal_peers(t.sig, t.world, t.rank);
        tp_wait_peers(t.sig, t.world, t.rank, seq + 1u, nullptr, t.spin_limit);
        t.state[1] = seq + 1u;
    }
}

size_t smem_bytes(int stages, int stage_bytes, int x_bytes, int nt) {
    return static_cast<size_t>(stages) * static_cast<size_t>(stage_bytes) + static_cast<size_t>(x_bytes) +
           16ull + 4ull * kUnitSlots * kCW * kRows * nt + sizeof(UnitMeta) * kUnitSlots + 8ull * kUnitSlots +
           8ull * (2 * kMaxStages + 1) + 16;
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
        if (o.type != kTypeQ4_K && o.type != kTypeQ5_K && o.type != kTypeQ6_K && o.type != kTypeQ4_0 &&
            o.type != kTypeQ8_0 && o.type != kTypeIQ4_XS)
            return false;
        if (o.ne2 != 1 || o.ne3 != 1) return false;
        if (o.N < 1 || o.N > kMaxNT) return false;
        if (o.N > 2 && o.K > kMaxK34) return false;  // the 3- or 4-vector image with a two-stage ring
        if (o.K % 256 != 0) return false;  // whole 256-element groups (Q8_0 too)
        if (o.K > kMaxK) return false;
        if ((o.type == kTypeQ4_K || o.type == kTypeQ5_K) &&
            ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15))
            return false;  // 16-byte header loads and ldmatrix rows from shared memory
        if ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 1)
            return false;  // 2-byte f16 and word-pair loads from shared memory
        if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;
    }
    return true;
}

namespace {
std::atomic<uint32_t> g_wait_limit{kSpinLimit};
}

void set_stream_wait_limit(uint32_t polls) { g_wait_limit.store(polls ? polls : kSpinLimit); }

int launch_stream(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms, const TpLaunch* tp,
                  const ProLaunch* pro) {
    SList L{};
    L.n_ops = n_ops;
    L.spin_limit = g_wait_limit.load();
    L.tp.spin_limit = L.spin_limit;
    const int kind = pro ? pro->kind : kProNone;
    if (kind < kProNone || kind > kProGelu) return -static_cast<int>(cudaErrorInvalidValue);
    if (pro) {
        L.pro.gain = pro->gain;
        L.pro.up = pro->up;
        L.pro.up_nb1 = pro->up_nb1;
        L.pro.eps = pro->eps;
        L.pro.kind = kind;
    }
    L.tp.world = 1;
    if (tp) {
        L.tp.world = tp->world;
        L.tp.rank = tp->rank;
        for (int r = 0; r < kMaxRanks; ++r) L.tp.sig[r] = tp->sig[r];
        L.tp.state = tp->state;
        for (int i = 0; i < n_ops; ++i)
            for (int r = 0; r < kMaxRanks; ++r) L.op[i].y_peer[r] = r < tp->world ? tp->y_peer[i][r] : nullptr;
    }
    int units = 0, max_n = 1, x_bytes = 0, wmax = 0;
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
        if (o.type == kTypeQ8_0 || o.type == kTypeQ4_0) seg = (seg + 7) / 8 * 8;
        s.seg_blocks = seg;
        s.nseg = (nblocks + seg - 1) / seg;
        // stage row width: the segment plus room for the 16-byte window rounding,
        // made == 16 mod 32 so the 8 rows a warp reads hit 8 different bank groups
        const int bb = block_bytes(o.type);
        const bool aligned_rows = o.type == kTypeQ4_K || o.type == kTypeQ5_K;  // 16-byte blocks
        int wbox = aligned_rows ? seg * bb : (seg * bb + 30 + 15) / 16 * 16;
        if (wbox % 32 == 0) wbox += 16;
        s.wbox = wbox;
        s.use_tma = encode_weight_map(s, nblocks * bb) ? 1 : 0;
        wmax = wbox > wmax ? wbox : wmax;
        units += (o.M + kRows - 1) / kRows;
        max_n = o.N > max_n ? o.N : max_n;
        const int xb = (img_bytes(o.K, o.N) + 15) / 16 * 16;
        x_bytes = xb > x_bytes ? xb : x_bytes;
    }
    L.total_units = units;
    L.all_tma = 1;
    for (int i = 0; i < n_ops; ++i) L.all_tma &= L.op[i].use_tma;
    L.x_bytes = x_bytes;
    L.stage_bytes = kRows * wmax;
    const int nt = max_n <= 1 ? 1 : (max_n <= 2 ? 2 : 4);
    const size_t fixed = smem_bytes(0, L.stage_bytes, x_bytes, nt);
    const size_t per_stage = smem_bytes(1, L.stage_bytes, x_bytes, nt) - fixed;
    int stages = fixed >= static_cast<size_t>(kSmemBudget)
                     ? 0
                     : static_cast<int>((static_cast<size_t>(kSmemBudget) - fixed) / per_stage);
    stages = stages > kMaxStages ? kMaxStages : stages;
    if (stages < 2) stages = 2;
    L.stages = stages;
    const size_t smem = smem_bytes(stages, L.stage_bytes, x_bytes, nt);
    if (smem > 227 * 1024) return -static_cast<int>(cudaErrorInvalidValue);
    // one CTA per SM: the ring needs most of its shared memory
    const int grid = units < num_sms ? units : num_sms;

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
    // (the attribute is per device: one size per device ordinal and kernel)
    static size_t configured[kMaxDevices][12] = {};
    int dev = 0;
    if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return -static_cast<int>(e);
    if (dev < 0 || dev >= kMaxDevices) return -static_cast<int>(cudaErrorInvalidDevice);
    const int ti = (nt == 1 ? 0 : (nt == 2 ? 1 : 2)) + 3 * kind;
    void (*const kernels[12])(SList) = {
        stream_gemv_kernel<1, kProNone>,   stream_gemv_kernel<2, kProNone>,   stream_gemv_kernel<4, kProNone>,
        stream_gemv_kernel<1, kProNorm>,   stream_gemv_kernel<2, kProNorm>,   stream_gemv_kernel<4, kProNorm>,
        stream_gemv_kernel<1, kProSwiglu>, stream_gemv_kernel<2, kProSwiglu>, stream_gemv_kernel<4, kProSwiglu>,
        stream_gemv_kernel<1, kProGelu>,   stream_gemv_kernel<2, kProGelu>,   stream_gemv_kernel<4, kProGelu>};
    void (*const kernel)(SList) = kernels[ti];
    cudaError_t e;
    if (configured[dev][ti] < smem) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return -static_cast<int>(e);
        configured[dev][ti] = smem;
    }
    e = cudaLaunchKernelEx(&cfg, kernel, L);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -static_cast<int>(e);
}

int launch_tp_wait(const TpLaunch& tp, cudaStream_t stream) {
    TpSig t{};
    t.spin_limit = g_wait_limit.load();
    t.world = tp.world;
    t.rank = tp.rank;
    for (int r = 0; r < kMaxRanks; ++r) t.sig[r] = tp.sig[r];
    t.state = tp.state;
    tp_wait_kernel<<<1, 32, 0, stream>>>(t);
    const cudaError_t e = cudaGetLastError();
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

