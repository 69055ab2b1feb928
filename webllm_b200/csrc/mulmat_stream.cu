// Decode-regime quantized MUL_MAT (N = 1 or 2 activation vectors): a
// persistent, warp-specialised streaming GEMV over raw GGUF blocks.
//
// Data movement. The weight matrix is cut into units of 8 rows; each unit's
// rows are cut into segments of at most 2304 bytes. One producer warp moves
// every (row, segment) piece HBM -> shared memory with one bulk async copy
// (cp.async.bulk, completion counted on an mbarrier), through a ring of
// stages, with an evict-first L2 policy because each weight byte is read
// exactly once. The copy window is the piece rounded out to 16-byte
// boundaries, so Q6_K (210 B) and Q8_0 (34 B) blocks, which are not
// 16-byte aligned, stream exactly like Q4_K. Eight consumer warps decode
// from shared memory.
//
// Consumer mapping. Lanes 8j..8j+7 work on row 4q+j of the unit; lane
// chunk c = lane%8 owns 32 elements of a 256-element block (Q4_K, Q6_K) or
// one whole 32-element block (Q8_0). The activation chunk a lane needs is
// the same for the four rows of a quad and for both quads of the unit, so it
// is loaded from shared memory once per block and kept in registers.
//
// Arithmetic. A 4- or 6-bit quant q is turned into the float 1 + q/128 with
// one byte permute (the byte 0x80|q becomes bits 16..23 of 0x3F800000);
// S = sum (1 + q/128) x is accumulated with packed FFMA2 and the quant sum
// is recovered as 128 (S - X), X = sum x over the same elements (computed
// once per block and lane). This keeps the weight unpack at ~1.3 integer
// ops per weight. Scales, mins and d are applied per sub-block in f32.
//
// Launch. Programmatic dependent launch: every CTA triggers its dependents
// at entry, the producer streams weights (never written by a preceding
// kernel) immediately, and the consumers execute griddepcontrol.wait before
// reading activations or writing outputs. So the next MUL_MAT's weight
// stream overlaps this one's tail. Every mbarrier wait is bounded; on
// timeout the kernel records an error code and returns.
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

__device__ unsigned int g_stream_error = 0;

namespace {

constexpr int kCW = 8;                       // consumer warps
constexpr int kThreads = 32 * (kCW + 1);     // + one producer warp
constexpr int kRows = 8;                     // rows per unit
constexpr int kPieceCap = 2304;              // max bytes of one row segment
constexpr int kPieceStride = kPieceCap + 32; // + window rounding slack
constexpr int kStageBytes = kRows * kPieceStride;
constexpr int kMaxStages = 6;
constexpr int kMaxNT = 2;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kSmemBudget = 110 * 1024;      // leaves room for a second CTA per SM

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
    int32_t x_floats;  // shared-memory floats reserved for activations
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

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

__device__ __forceinline__ int block_elems_of(int type) { return type == kTypeQ8_0 ? 32 : 256; }
__device__ __forceinline__ int block_bytes_of(int type) {
    return type == kTypeQ4_K ? 144 : (type == kTypeQ6_K ? 210 : 34);
}

// 1 + q/128 for the byte 0x80|q in byte position k of w.
template <int k>
__device__ __forceinline__ float unit_q(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7044u | (k << 8)));
}

// Element offset (within the block group) of float4 f of lane chunk c.
// Activations are staged as xs4[group][f][c] so that the 8 chunks of one
// LDS.128 phase are 8 consecutive float4 (no bank conflicts).
__device__ __forceinline__ int chunk_elem(int type, int c, int f) {
    if (type == kTypeQ4_K) {
        const int p = c >> 1, h = c & 1;
        return 64 * p + 16 * h + (f < 4 ? 4 * f : 32 + 4 * (f - 4));
    }
    if (type == kTypeQ6_K) {
        const int h = c >> 2, l0 = 8 * (c & 3), t = f >> 1;
        return 128 * h + 32 * t + l0 + 4 * (f & 1);
    }
    return 32 * c + 4 * f;  // Q8_0: lane chunk c is block c of the group
}

// 16-byte (or smaller-aligned) loads from shared memory of raw block bytes.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);  // keeps the shared-space provenance
    return __funnelshift_r(q[0], q[1], mis * 8);
}
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

template <int NT>
struct Acc {
    float v[2][NT];  // [quad][token]
};

// ---- per-format item computations (one lane, one row, one block) ----

template <int NT>
__device__ __forceinline__ void item_q4_k(const uint8_t* blk, int c, const float4 (&xr)[NT][8], const float (&xs)[NT][2],
                                          float (&acc)[NT]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 16 * c);
    const int p = c >> 1;
    // packed 6-bit scales/mins (get_scale_min_k4): words of bytes sc0..3, m0..3, sc4..7, m4..7
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    uint32_t scw, mw;
    if (p < 2) {
        scw = s0 & 0x3F3F3F3Fu;
        mw = s1 & 0x3F3F3F3Fu;
    } else {
        scw = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
        mw = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    }
    const int sh = 16 * (p & 1);  // byte pair (2p, 2p+1) within the word
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    const float sc_lo = static_cast<float>((scw >> sh) & 0xFFu), sc_hi = static_cast<float>((scw >> (sh + 8)) & 0xFFu);
    const float m_lo = static_cast<float>((mw >> sh) & 0xFFu), m_hi = static_cast<float>((mw >> (sh + 8)) & 0xFFu);
    const float a_lo = 128.f * d * sc_lo, a_hi = 128.f * d * sc_hi;
    const float b_lo = a_lo + dmin * m_lo, b_hi = a_hi + dmin * m_hi;
    const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
    float2 slo[NT], shi[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) slo[n] = shi[n] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = (w4[i] & 0x0F0F0F0Fu) | 0x80808080u;
        const uint32_t hi = ((w4[i] >> 4) & 0x0F0F0F0Fu) | 0x80808080u;
        const float2 l01 = make_float2(unit_q<0>(lo), unit_q<1>(lo)), l23 = make_float2(unit_q<2>(lo), unit_q<3>(lo));
        const float2 h01 = make_float2(unit_q<0>(hi), unit_q<1>(hi)), h23 = make_float2(unit_q<2>(hi), unit_q<3>(hi));
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const float4 xl = xr[n][i], xh = xr[n][4 + i];
            slo[n] = __ffma2_rn(l01, make_float2(xl.x, xl.y), slo[n]);
            slo[n] = __ffma2_rn(l23, make_float2(xl.z, xl.w), slo[n]);
            shi[n] = __ffma2_rn(h01, make_float2(xh.x, xh.y), shi[n]);
            shi[n] = __ffma2_rn(h23, make_float2(xh.z, xh.w), shi[n]);
        }
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const float S_lo = slo[n].x + slo[n].y, S_hi = shi[n].x + shi[n].y;
        // sum (d sc q - dmin m) x = a (S - X) - dmin m X = a S - b X
        acc[n] += a_lo * S_lo - b_lo * xs[n][0] + a_hi * S_hi - b_hi * xs[n][1];
    }
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
            // sum d sc (q6 - 32) x = a (S - X) - 32/128 a X = a S - (5/4) a X
            r += a[t] * ((s[t][n].x + s[t][n].y) - 1.25f * xq[n][t]);
        }
        acc[n] += r;
    }
}

template <int NT>
__device__ __forceinline__ void item_q8_0(const uint8_t* blk, const float4 (&xr)[NT][8], float (&acc)[NT]) {
    const float d = f16_bits_to_f32(lds_u16(blk));
    float2 s[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n] = make_float2(0.f, 0.f);
#pragma unroll
    for (int f = 0; f < 8; ++f) {
        const uint32_t w = lds_u32_any(blk + 2 + 4 * f) ^ 0x80808080u;  // biased to u = q + 128
        // 2^23 + u exactly, then subtract 2^23 + 128 -> q
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

template <int NT>
__global__ void __launch_bounds__(kThreads, 2) stream_gemv_kernel(const __grid_constant__ SList L) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = L.stages;
    uint8_t* stages = smem;
    float4* xs4 = reinterpret_cast<float4*>(smem + S * kStageBytes);
    float* red = reinterpret_cast<float*>(smem + S * kStageBytes + 4 * L.x_floats);  // [2][kCW][kRows][NT]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kCW * kRows * NT);
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
        // ---------------- producer ----------------
        if (lane == 0) {
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
                for (int sg = 0; sg < op.nseg; ++sg, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, 1u, poisoned)) return;
                    const int b0 = sg * op.seg_blocks;
                    const int nb = min(op.seg_blocks, nblocks - b0);
                    uint32_t total = 0;
                    for (int r = 0; r < nrows; ++r) {
                        const uintptr_t g = reinterpret_cast<uintptr_t>(op.w + (r0 + r) * op.w_nb1 + b0 * bb);
                        total += static_cast<uint32_t>(((g + nb * bb + 15) & ~uintptr_t(15)) - (g & ~uintptr_t(15)));
                    }
                    mbar_arrive_expect_tx(&full[s], total);
                    for (int r = 0; r < nrows; ++r) {
                        const uintptr_t g = reinterpret_cast<uintptr_t>(op.w + (r0 + r) * op.w_nb1 + b0 * bb);
                        const uintptr_t ga = g & ~uintptr_t(15);
                        const uint32_t bytes = static_cast<uint32_t>(((g + nb * bb + 15) & ~uintptr_t(15)) - ga);
                        bulk_g2s(stages + s * kStageBytes + r * kPieceStride, reinterpret_cast<const void*>(ga), bytes,
                                 &full[s], policy);
                    }
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int ct = threadIdx.x - 32;  // 0..255
    const int cw = warp - 1;          // 0..7
    const int j = lane >> 3, c = lane & 7;
    uint32_t it = 0;
    int oi = 0, staged = -1;
    int rb = 0;  // reduction buffer parity
    for (int u = blockIdx.x; u < L.total_units; u += gridDim.x) {
        while (oi + 1 < L.n_ops && u >= L.op[oi + 1].unit_begin) ++oi;
        const SOp& op = L.op[oi];
        // (re)stage activations when the op's x or layout changes
        if (staged < 0 || L.op[staged].x != op.x || L.op[staged].type != op.type || L.op[staged].K != op.K ||
            L.op[staged].N != op.N || L.op[staged].x_nb1 != op.x_nb1) {
            consumers_sync();
            const int groups = op.K / 256;  // 256-element block groups
            const int per_tok = groups * 64;
            for (int idx = ct; idx < per_tok * op.N; idx += kCW * 32) {
                const int n = idx / per_tok, r = idx % per_tok;
                const int g = r >> 6, f = (r >> 3) & 7, cc = r & 7;
                const float* xp = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(op.x) + n * op.x_nb1);
                xs4[idx] = __ldg(reinterpret_cast<const float4*>(xp + g * 256 + chunk_elem(op.type, cc, f)));
            }
            consumers_sync();
            staged = oi;
        }
        const int bb = block_bytes_of(op.type);
        const int nblocks = op.K / block_elems_of(op.type);
        const int r0 = (u - op.unit_begin) * kRows;
        const int groups_per_tok = op.K / 256;
        float acc[2][NT];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int n = 0; n < NT; ++n) acc[q][n] = 0.f;

        for (int sg = 0; sg < op.nseg; ++sg, ++it) {
            const int s = it % S;
            mbar_wait(&full[s], (it / S) & 1, 2u, poisoned);
            const int b0 = sg * op.seg_blocks;
            const int nb = min(op.seg_blocks, nblocks - b0);
            const uint8_t* stage = stages + s * kStageBytes;
            // block groups of this segment (Q8_0: 8 blocks per group)
            const int gpb = op.type == kTypeQ8_0 ? 8 : 1;
            const int g0 = b0 / gpb;
            const int ngroups = (nb + gpb - 1) / gpb;
            for (int gi = cw; gi < ngroups; gi += kCW) {
                const int g = g0 + gi;
                float4 xr[NT][8];
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int f = 0; f < 8; ++f) xr[n][f] = xs4[(n * groups_per_tok + g) * 64 + f * 8 + c];
                if (op.type == kTypeQ8_0) {
                    const int blk = g * 8 + c;  // this lane's Q8_0 block
                    if (blk < b0 + nb) {
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int r = 4 * q + j;
                            const uintptr_t gaddr = reinterpret_cast<uintptr_t>(op.w + (r0 + r) * op.w_nb1 + b0 * bb);
                            const uint8_t* base = stage + r * kPieceStride + (gaddr & 15);
                            item_q8_0<NT>(base + (blk - b0) * 34, xr, acc[q]);
                        }
                    }
                } else if (op.type == kTypeQ4_K) {
                    float xs[NT][2];
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        float a = 0.f, b = 0.f;
#pragma unroll
                        for (int f = 0; f < 4; ++f) {
                            a += (xr[n][f].x + xr[n][f].y) + (xr[n][f].z + xr[n][f].w);
                            b += (xr[n][4 + f].x + xr[n][4 + f].y) + (xr[n][4 + f].z + xr[n][4 + f].w);
                        }
                        xs[n][0] = a;
                        xs[n][1] = b;
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int r = 4 * q + j;
                        const uintptr_t gaddr = reinterpret_cast<uintptr_t>(op.w + (r0 + r) * op.w_nb1 + b0 * bb);
                        const uint8_t* base = stage + r * kPieceStride + (gaddr & 15);
                        item_q4_k<NT>(base + (g - b0) * 144, c, xr, xs, acc[q]);
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
                    for (int q = 0; q < 2; ++q) {
                        const int r = 4 * q + j;
                        const uintptr_t gaddr = reinterpret_cast<uintptr_t>(op.w + (r0 + r) * op.w_nb1 + b0 * bb);
                        const uint8_t* base = stage + r * kPieceStride + (gaddr & 15);
                        item_q6_k<NT>(base + (g - b0) * 210, c, xr, xq, acc[q]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // ---- reduce: 8 lanes of a row, then the 8 consumer warps ----
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                float v = acc[q][n];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                if (c == 0) red[((rb * kCW + cw) * kRows + 4 * q + j) * NT + n] = v;
            }
        consumers_sync();
        if (ct < kRows * op.N && ct < kRows * NT) {
            const int r = ct / op.N, n = ct % op.N;
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

template <int NT>
size_t smem_bytes(int stages, int x_floats) {
    return static_cast<size_t>(stages) * kStageBytes + 4ull * x_floats + 4ull * 2 * kCW * kRows * NT +
           16ull * kMaxStages + 16;
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
            return false;  // 16-byte header/quant loads from shared memory
        if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;
    }
    return true;
}

int launch_stream(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms) {
    SList L{};
    L.n_ops = n_ops;
    int units = 0, max_n = 1, x_floats = 0;
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
        const int bb = block_bytes(o.type), be = block_elems(o.type);
        const int nblocks = o.K / be;
        int max_blocks = kPieceCap / bb;
        if (o.type == kTypeQ8_0) max_blocks = max_blocks / 8 * 8;  // whole 8-block groups per segment
        const int nseg = (nblocks + max_blocks - 1) / max_blocks;
        int seg = (nblocks + nseg - 1) / nseg;
        if (o.type == kTypeQ8_0) seg = (seg + 7) / 8 * 8;
        s.seg_blocks = seg;
        s.nseg = (nblocks + seg - 1) / seg;
        units += (o.M + kRows - 1) / kRows;
        max_n = o.N > max_n ? o.N : max_n;
        x_floats = (o.K * o.N > x_floats) ? o.K * o.N : x_floats;
    }
    L.total_units = units;
    L.x_floats = x_floats;
    const int NT = max_n <= 1 ? 1 : 2;
    const size_t fixed = (NT == 1 ? smem_bytes<1>(0, x_floats) : smem_bytes<2>(0, x_floats));
    int stages = static_cast<int>((static_cast<size_t>(kSmemBudget) - fixed) / kStageBytes);
    if (fixed > static_cast<size_t>(kSmemBudget)) stages = 0;
    stages = stages > kMaxStages ? kMaxStages : stages;
    if (stages < 2) stages = 2;
    L.stages = stages;
    const size_t smem = NT == 1 ? smem_bytes<1>(stages, x_floats) : smem_bytes<2>(stages, x_floats);
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
    if (NT == 1) {
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
