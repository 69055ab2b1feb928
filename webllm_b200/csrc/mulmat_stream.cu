// Decode-regime quantized MUL_MAT (N = 1 or 2 activation vectors): a
// persistent, warp-specialised streaming GEMV over raw GGUF blocks.
//
// Data movement. The weight matrix is cut into units of 16 rows; each
// unit's rows are cut into segments of at most 8 Q4_K / 5 Q6_K / 32 Q8_0
// blocks. One producer warp moves every (row, segment) piece HBM -> shared
// memory with one bulk async copy (cp.async.bulk, completion counted on an
// mbarrier) through a ring of stages, with an evict-first L2 policy (each
// weight byte is read exactly once). The copy window is the piece rounded
// out to 16-byte boundaries, so Q6_K (210 B) and Q8_0 (34 B) blocks, which
// are not 16-byte aligned, stream exactly like Q4_K. Eight consumer warps
// compute from shared memory.
//
// Q4_K on tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate). A unit
// is one 16-row MMA tile. A 4-bit quant enters the MMA as the exact f16
// subnormal q * 2^-24 (one LOP3 per two quants: low nibble pairs are
// (v & 0x000F000F), high nibbles (v & 0x00F000F0) = 16 q * 2^-24). The
// activations are the B operand, split into two f16 limbs hi = f16(x s),
// lo = f16(x s - hi) (s a power of two per vector keeps x s inside f16
// range), so 22 bits of x take part and every product is exact; the MMA
// sums them in f32. Each 32-element sub-block is its own accumulator chain
// of two k16 MMAs; the chain result is scaled in f32 by d*sc (decoded once
// per stage into a shared table) and the min term dmin*m*sum(x) is
// subtracted in f32. The k order inside an MMA is a fixed permutation
// shared by A and B: lane group c holds quant bytes 4c..4c+3.
//
// Q6_K and Q8_0 on CUDA cores. Lanes 8j..8j+7 work on row 4q+j (q = 0..3);
// lane chunk c = lane%8 owns 32 elements of a 256-element block (Q6_K) or
// one 32-element block (Q8_0); the lane's activation chunk stays in
// registers for the unit's four quads. A 6-bit quant becomes the float
// 1 + q/128 with one byte permute (0x80|q placed in bits 16..23 of
// 0x3F800000), S = sum (1 + q/128) x runs on packed FFMA2, and the quant
// sum is recovered as 128 (S - X) with X = sum x over the same elements.
//
// Launch. Programmatic dependent launch: CTAs trigger their dependents at
// entry; the producer streams weights (never written by a preceding kernel)
// immediately; consumers execute griddepcontrol.wait before reading
// activations or writing outputs. Every mbarrier wait is bounded; on timeout
// the CTA records an error code and drains without further waiting.
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_stream_error = 0;

namespace {

constexpr int kCW = 8;                        // consumer warps
constexpr int kThreads = 32 * (kCW + 1);      // + one producer warp
constexpr int kRows = 16;                     // rows per unit (one MMA m-tile)
constexpr int kPieceStride = 1296;            // bytes per row piece (== 16 mod 128: conflict-free rows)
constexpr int kStageBytes = kRows * kPieceStride;
constexpr int kMaxStages = 8;
constexpr int kMaxNT = 2;
constexpr int kQ4kSegBlocks = 8;              // 1152 B
constexpr int kQ6kSegBlocks = 5;              // 1050 B (+ window slack)
constexpr int kQ80SegBlocks = 32;             // 1088 B, whole 8-block groups
constexpr int kTabBytes = kRows * kQ4kSegBlocks * 4 * 16;  // Q4_K scale table, one buffer
constexpr uint32_t kSpinLimit = 1u << 16;    // polls of up to ~0.1 ms each
constexpr int kSmemBudget = 112 * 1024;       // two CTAs per SM: this launch and the next (PDL)

struct SOp {
    const uint8_t* w;
    const float* x;
    float* y;
    int64_t w_nb1, x_nb1, y_nb1;  // bytes
    int32_t type, M, K, N;
    int32_t unit_begin;           // first unit of this op
    int32_t seg_blocks;           // blocks per segment (last may be shorter)
    int32_t nseg;
};

struct SList {
    SOp op[kMaxOpsPerLaunch];
    int32_t n_ops;
    int32_t total_units;
    int32_t stages;
    int32_t x_bytes;  // shared-memory bytes reserved for staged activations
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// try_wait with a suspend-time hint: the thread sleeps (up to ~0.1 ms) until
// the phase completes instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait. If the phase does not complete within kSpinLimit polls the
// CTA is poisoned: an error code is recorded for the host, and every later
// wait of the CTA returns at once, so all threads still reach the same
// barriers and the kernel ends (with garbage results and the error set).
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
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ int block_elems_of(int type) { return type == kTypeQ8_0 ? 32 : 256; }
__device__ __forceinline__ int block_bytes_of(int type) {
    return type == kTypeQ4_K ? 144 : (type == kTypeQ6_K ? 210 : 34);
}

// 1 + q/128 for the byte 0x80|q in byte position k of w.
template <int k>
__device__ __forceinline__ float unit_q(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7044u | (k << 8)));
}

// Element offset (within its 256-element group) of float4 f of lane chunk c,
// for the CUDA-core formats. Activations are staged as xs4[group][f][c] so
// the 8 chunks of one LDS.128 phase are 8 consecutive float4.
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

// ---------------------------------------------------------------- Q4_K (tensor cores)

// Scale table entry for (row, block, pair p): d*sc*2^24 (low sub-block),
// d*sc*2^20 (high sub-block; its quants enter as 16 q), dmin*m low, high.
__device__ __forceinline__ void q4k_decode_scales(const uint8_t* blk, float4* out /* [4] */) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    const uint32_t sc_lo4 = s0 & 0x3F3F3F3Fu, m_lo4 = s1 & 0x3F3F3F3Fu;
    const uint32_t sc_hi4 = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t m_hi4 = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    const float d24 = d * 16777216.f, d20 = d * 1048576.f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t scw = p < 2 ? sc_lo4 : sc_hi4, mw = p < 2 ? m_lo4 : m_hi4;
        const int sh = 16 * (p & 1);
        out[p] = make_float4(d24 * static_cast<float>((scw >> sh) & 0xFFu),
                             d20 * static_cast<float>((scw >> (sh + 8)) & 0xFFu),
                             dmin * static_cast<float>((mw >> sh) & 0xFFu),
                             dmin * static_cast<float>((mw >> (sh + 8)) & 0xFFu));
    }
}

// ---------------------------------------------------------------- Q6_K / Q8_0 (CUDA cores)

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

template <int NT>
__global__ void __maxnreg__(112) stream_gemv_kernel(const __grid_constant__ SList L) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = L.stages;
    uint8_t* stages = smem;
    uint8_t* xsm = smem + S * kStageBytes;                                 // staged activations
    float4* tab = reinterpret_cast<float4*>(xsm + L.x_bytes);              // [2][16 rows][8 blocks][4]
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tab) + 2 * kTabBytes);  // [2][kCW][16][NT]
    float* xscale = red + 2 * kCW * kRows * NT;                            // [NT] 1/s per vector
    uint64_t* full = reinterpret_cast<uint64_t*>(xscale + 2 * kMaxNT);
    uint64_t* empty = full + kMaxStages;
    volatile int* poisoned = reinterpret_cast<volatile int*>(empty + kMaxStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        *poisoned = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ---------------- producer: lane r issues row r's copy ----------------
        const uint64_t policy = evict_first_policy();
        uint32_t it = 0;
        int oi = 0;
        for (int u = blockIdx.x; u < L.total_units; u += gridDim.x) {
            while (oi + 1 < L.n_ops && u >= L.op[oi + 1].unit_begin) ++oi;
            const SOp& op = L.op[oi];
            const int bb = block_bytes_of(op.type);
            const int nblocks = op.K / block_elems_of(op.type);
            const int r0 = (u - op.unit_begin) * kRows;
            const int nrows = min(kRows, op.M - r0);
            const bool active = lane < nrows;
            const uintptr_t grow = reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0 + (active ? lane : 0)) * op.w_nb1);
            for (int sg = 0; sg < op.nseg; ++sg, ++it) {
                const int s = it % S;
                int ok = 1;
                if (lane == 0) ok = mbar_wait(&empty[s], ((it / S) & 1) ^ 1, 1u, poisoned);
                if (!__shfl_sync(0xffffffffu, ok, 0)) return;
                const int b0 = sg * op.seg_blocks;
                const int nbytes = min(op.seg_blocks, nblocks - b0) * bb;
                const uintptr_t g = grow + static_cast<uintptr_t>(b0 * bb);
                const uintptr_t ga = g & ~uintptr_t(15);
                const uint32_t bytes = active ? static_cast<uint32_t>(((g + nbytes + 15) & ~uintptr_t(15)) - ga) : 0u;
                const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
                if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
                __syncwarp();
                if (active)
                    bulk_g2s(stages + s * kStageBytes + lane * kPieceStride, reinterpret_cast<const void*>(ga), bytes,
                             &full[s], policy);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ct = threadIdx.x - 32;  // 0..255
    const int cw = warp - 1;          // 0..7
    uint32_t it = 0;
    int oi = 0, staged = -1;
    int rb = 0, tb = 0;
    for (int u = blockIdx.x; u < L.total_units; u += gridDim.x) {
        while (oi + 1 < L.n_ops && u >= L.op[oi + 1].unit_begin) ++oi;
        const SOp& op = L.op[oi];
        const int N = op.N;
        const int K = op.K;
        const bool tc = op.type == kTypeQ4_K;
        // ---- (re)stage activations when the op's x or layout changes ----
        if (staged < 0 || L.op[staged].x != op.x || L.op[staged].type != op.type || L.op[staged].K != K ||
            L.op[staged].N != N || L.op[staged].x_nb1 != op.x_nb1) {
            consumers_sync();
            const uint8_t* xb = reinterpret_cast<const uint8_t*>(op.x);
            const int per_tok4 = K / 4;           // float4 per vector (a multiple of 64)
            const int total4 = per_tok4 * N;
            constexpr int kBatch = 4;             // float4 loads in flight per thread
            if (tc) {
                // pass 1: per-vector max|x| -> power-of-two scale s (loads batched)
                float mx[kMaxNT] = {0.f, 0.f};
                for (int base = 0; base < total4; base += kBatch * kCW * 32) {
                    float4 v[kBatch];
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4)
                            v[i] = __ldg(reinterpret_cast<const float4*>(xb + (idx / per_tok4) * op.x_nb1) + idx % per_tok4);
                    }
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4) {
                            const float m = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
                            if (idx < per_tok4) mx[0] = fmaxf(mx[0], m);
                            else mx[1] = fmaxf(mx[1], m);
                        }
                    }
                }
#pragma unroll
                for (int n = 0; n < kMaxNT; ++n) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx[n] = fmaxf(mx[n], __shfl_xor_sync(0xffffffffu, mx[n], o));
                    if (lane == 0) red[n * kCW + cw] = mx[n];
                }
                consumers_sync();
                if (ct < N) {
                    float m = 0.f;
#pragma unroll
                    for (int w2 = 0; w2 < kCW; ++w2) m = fmaxf(m, red[ct * kCW + w2]);
                    const float sc = limb_scale(m);
                    xscale[ct] = sc;
                    xscale[kMaxNT + ct] = 1.f / sc;
                }
                consumers_sync();
                // pass 2 (L1-resident reload): f16 limbs in B-fragment order, entry
                // e = ((b*4 + p)*2 + j)*2 + h, lanes 0..8N-1, and the sub-block sums
                // X of the unscaled x for the min term (8 consecutive lanes hold one
                // 32-element sub-block).
                uint2* xB = reinterpret_cast<uint2*>(xsm);
                const int lanes = 8 * N;
                float* Xs = reinterpret_cast<float*>(xsm + (K / 256) * 16 * lanes * 8);
                for (int base = 0; base < total4; base += kBatch * kCW * 32) {
                    float4 v[kBatch];
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4)
                            v[i] = __ldg(reinterpret_cast<const float4*>(xb + (idx / per_tok4) * op.x_nb1) + idx % per_tok4);
                    }
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4) {  // warp-uniform: total4 is a multiple of 64
                            const int t = idx / per_tok4, k = 4 * (idx % per_tok4);
                            const int b = k >> 8, r = k & 255, p = r >> 6, h = (r >> 5) & 1, jj = (r >> 4) & 1;
                            const int cp = (r >> 2) & 3;
                            const int e = ((b * 4 + p) * 2 + jj) * 2 + h;
                            const float sc = xscale[t];
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
            } else {
                float4* xs4 = reinterpret_cast<float4*>(xsm);
                for (int base = 0; base < total4; base += kBatch * kCW * 32) {
                    float4 v[kBatch];
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4) {
                            const int n = idx / per_tok4, r = idx % per_tok4;
                            const int g = r >> 6, f = (r >> 3) & 7, cc = r & 7;
                            v[i] = __ldg(reinterpret_cast<const float4*>(
                                reinterpret_cast<const float*>(xb + n * op.x_nb1) + g * 256 + chunk_elem(op.type, cc, f)));
                        }
                    }
#pragma unroll
                    for (int i = 0; i < kBatch; ++i) {
                        const int idx = base + i * kCW * 32 + ct;
                        if (idx < total4) xs4[idx] = v[i];
                    }
                }
            }
            consumers_sync();
            staged = oi;
        }
        const int bb = block_bytes_of(op.type);
        const int nblocks = K / block_elems_of(op.type);
        const int r0 = (u - op.unit_begin) * kRows;
        const uint32_t wlo = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(op.w + static_cast<int64_t>(r0) * op.w_nb1));
        const uint32_t nb1lo = static_cast<uint32_t>(op.w_nb1);

        if (tc) {
            // ================= Q4_K, tensor cores =================
            const int g = lane >> 2, c = lane & 3;
            const int lanes = 8 * N;
            const uint2* xB = reinterpret_cast<const uint2*>(xsm);
            const float* Xs = reinterpret_cast<const float*>(xsm + (K / 256) * 16 * lanes * 8);
            const int nsub = K / 32;
            float accm_g = 0.f, accm_g8 = 0.f;  // sum A * (D_hi + D_lo), in units of x*s
            float accn_g = 0.f, accn_g8 = 0.f;  // sum dmin*m*X (unscaled)
            for (int sg = 0; sg < op.nseg; ++sg, ++it) {
                const int s = it % S;
                mbar_wait(&full[s], (it / S) & 1, 2u, poisoned);
                const int b0 = sg * op.seg_blocks;
                const int nb = min(op.seg_blocks, nblocks - b0);
                const uint8_t* stage = stages + s * kStageBytes;
                float4* tbuf = tab + tb * (kRows * kQ4kSegBlocks * 4);
                // scale table: one thread per (row, block)
                if (ct < kRows * nb) {
                    const int r = ct & 15, bl = ct >> 4;
                    q4k_decode_scales(stage + r * kPieceStride + bl * 144, tbuf + (r * kQ4kSegBlocks + bl) * 4);
                }
                consumers_sync();
                const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
                for (int item = cw; item < nb * 4; item += kCW) {
                    const int bl = item >> 2, p = item & 3;
                    const int bg = b0 + bl;
                    const uint8_t* rq = stage + g * kPieceStride + bl * 144 + 16 + 32 * p + 4 * c;
                    const uint32_t vg0 = *reinterpret_cast<const uint32_t*>(rq);
                    const uint32_t vg1 = *reinterpret_cast<const uint32_t*>(rq + 16);
                    const uint32_t vh0 = *reinterpret_cast<const uint32_t*>(rq + 8 * kPieceStride);
                    const uint32_t vh1 = *reinterpret_cast<const uint32_t*>(rq + 8 * kPieceStride + 16);
                    const uint2* xe = xB + ((bg * 4 + p) * 4) * lanes;  // entries (j, h) = 0..3
                    uint2 bl0 = make_uint2(0u, 0u), bl1 = bl0, bh0 = bl0, bh1 = bl0;
                    if (lane < lanes) {
                        bl0 = xe[0 * lanes + lane];  // j=0, lo
                        bh0 = xe[1 * lanes + lane];  // j=0, hi
                        bl1 = xe[2 * lanes + lane];  // j=1, lo
                        bh1 = xe[3 * lanes + lane];  // j=1, hi
                    }
                    const uint32_t vg0s = vg0 >> 8, vg1s = vg1 >> 8, vh0s = vh0 >> 8, vh1s = vh1 >> 8;
                    float dlo[4], dhi[4];
                    mma_f16(dlo, vg0 & 0x000F000Fu, vh0 & 0x000F000Fu, vg0s & 0x000F000Fu, vh0s & 0x000F000Fu, bl0.x,
                            bl0.y, zero4);
                    mma_f16(dlo, vg1 & 0x000F000Fu, vh1 & 0x000F000Fu, vg1s & 0x000F000Fu, vh1s & 0x000F000Fu, bl1.x,
                            bl1.y, dlo);
                    mma_f16(dhi, vg0 & 0x00F000F0u, vh0 & 0x00F000F0u, vg0s & 0x00F000F0u, vh0s & 0x00F000F0u, bh0.x,
                            bh0.y, zero4);
                    mma_f16(dhi, vg1 & 0x00F000F0u, vh1 & 0x00F000F0u, vg1s & 0x00F000F0u, vh1s & 0x00F000F0u, bh1.x,
                            bh1.y, dhi);
                    const float4 sg_ = tbuf[(g * kQ4kSegBlocks + bl) * 4 + p];
                    const float4 sg8 = tbuf[((g + 8) * kQ4kSegBlocks + bl) * 4 + p];
                    float xlo = 0.f, xhi = 0.f;
                    if (c < N) {
                        xlo = Xs[c * nsub + bg * 8 + 2 * p];
                        xhi = Xs[c * nsub + bg * 8 + 2 * p + 1];
                    }
                    accm_g += sg_.x * (dlo[0] + dlo[1]) + sg_.y * (dhi[0] + dhi[1]);
                    accm_g8 += sg8.x * (dlo[2] + dlo[3]) + sg8.y * (dhi[2] + dhi[3]);
                    accn_g += sg_.z * xlo + sg_.w * xhi;
                    accn_g8 += sg8.z * xlo + sg8.w * xhi;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                tb ^= 1;
            }
            if (c < N) {
                const float inv = xscale[kMaxNT + c];
                red[((rb * kCW + cw) * kRows + g) * NT + c] = accm_g * inv - accn_g;
                red[((rb * kCW + cw) * kRows + g + 8) * NT + c] = accm_g8 * inv - accn_g8;
            }
        } else {
            // ================= Q6_K / Q8_0, CUDA cores =================
            const int j = lane >> 3, c = lane & 7;
            const int K256 = K / 256;
            const float4* xs4 = reinterpret_cast<const float4*>(xsm);
            float acc[4][NT];
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int n = 0; n < NT; ++n) acc[q][n] = 0.f;
            for (int sg = 0; sg < op.nseg; ++sg, ++it) {
                const int s = it % S;
                mbar_wait(&full[s], (it / S) & 1, 2u, poisoned);
                const int b0 = sg * op.seg_blocks;
                const int nb = min(op.seg_blocks, nblocks - b0);
                const uint8_t* stage = stages + s * kStageBytes;
                const uint32_t glo = wlo + static_cast<uint32_t>(b0 * bb);
                const uint8_t* base[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int r = 4 * q + j;
                    base[q] = stage + r * kPieceStride + ((glo + static_cast<uint32_t>(r) * nb1lo) & 15u);
                }
                const int gpb = op.type == kTypeQ8_0 ? 8 : 1;
                const int g0 = b0 / gpb;
                const int ngroups = (nb + gpb - 1) / gpb;
                for (int gi = cw; gi < ngroups; gi += kCW) {
                    const int g = g0 + gi;
                    float4 xr[NT][8];
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int f = 0; f < 8; ++f) xr[n][f] = xs4[(n * K256 + g) * 64 + f * 8 + c];
                    if (op.type == kTypeQ8_0) {
                        const int blk = g * 8 + c;
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
                        for (int q = 0; q < 4; ++q) item_q6_k<NT>(base[q] + (g - b0) * 210, c, xr, xq, acc[q]);
                    }
                }
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
                    if (c == 0) red[((rb * kCW + cw) * kRows + 4 * q + j) * NT + n] = v;
                }
        }
        consumers_sync();
        if (ct < kRows * N) {
            const int r = ct / N, n = ct % N;
            if (r0 + r < op.M) {
                float v = 0.f;
#pragma unroll
                for (int w2 = 0; w2 < kCW; ++w2) v += red[((rb * kCW + w2) * kRows + r) * NT + n];
                *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(op.y) + n * op.y_nb1 + 4LL * (r0 + r)) = v;
            }
        }
        rb ^= 1;
    }
}

size_t smem_bytes(int stages, int x_bytes) {
    return static_cast<size_t>(stages) * kStageBytes + static_cast<size_t>(x_bytes) + 2ull * kTabBytes +
           4ull * 2 * kCW * kRows * kMaxNT + 4ull * 2 * kMaxNT + 16ull * kMaxStages + 16;
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
        if (o.K > 16384) return false;
        if (o.type == kTypeQ4_K && ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15))
            return false;  // 16-byte header loads from shared memory
        if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;
    }
    return true;
}

int launch_stream(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms) {
    SList L{};
    L.n_ops = n_ops;
    int units = 0, max_n = 1, x_bytes = 0;
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
        const int cap = o.type == kTypeQ4_K ? kQ4kSegBlocks : (o.type == kTypeQ6_K ? kQ6kSegBlocks : kQ80SegBlocks);
        const int nseg = (nblocks + cap - 1) / cap;
        int seg = (nblocks + nseg - 1) / nseg;
        if (o.type == kTypeQ8_0) seg = (seg + 7) / 8 * 8;
        s.seg_blocks = seg;
        s.nseg = (nblocks + seg - 1) / seg;
        units += (o.M + kRows - 1) / kRows;
        max_n = o.N > max_n ? o.N : max_n;
        const int xb = o.type == kTypeQ4_K ? (o.K / 256) * 16 * 8 * o.N * 8 + (o.K / 32) * o.N * 4 : 4 * o.K * o.N;
        x_bytes = xb > x_bytes ? xb : x_bytes;
    }
    x_bytes = (x_bytes + 15) / 16 * 16;
    L.total_units = units;
    L.x_bytes = x_bytes;
    const size_t fixed = smem_bytes(0, x_bytes);
    int stages = fixed >= static_cast<size_t>(kSmemBudget)
                     ? 0
                     : static_cast<int>((static_cast<size_t>(kSmemBudget) - fixed) / kStageBytes);
    stages = stages > kMaxStages ? kMaxStages : stages;
    if (stages < 2) stages = 2;
    L.stages = stages;
    const size_t smem = smem_bytes(stages, x_bytes);
    if (smem > 227 * 1024) return -static_cast<int>(cudaErrorInvalidValue);
    const int grid = units < num_sms ? units : num_sms;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (max_n <= 1) {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(stream_gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            configured = true;
        }
        e = cudaLaunchKernelEx(&cfg, stream_gemv_kernel<1>, L);
    } else {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(stream_gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            configured = true;
        }
        e = cudaLaunchKernelEx(&cfg, stream_gemv_kernel<2>, L);
    }
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
