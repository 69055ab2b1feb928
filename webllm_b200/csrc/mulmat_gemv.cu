// Quantized MUL_MAT for the decode regime (N = 1..8 activation vectors):
// fused dequant + GEMV over raw GGUF blocks, one warp per output row.
//
// Each launch takes a list of independent ops (a whole q/k/v group, say);
// CTAs are handed out op by op, 8 rows per CTA. A warp streams its row's
// blocks with coalesced loads (a Q4_K block's 128 quant bytes are one
// 128-byte warp load), unpacks 4/6/8-bit values in registers, multiplies by
// the f32 activations and reduces with warp shuffles. Per-lane sums are
// formed per sub-block so the 6-bit scale/min products are applied once per
// 4-8 weights; the Q4_K min term uses sum(x) over the same elements.
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_blocks.cuh"
#include "wllm_internal.h"

namespace wllm {

namespace {

constexpr int kWarps = 8;
constexpr int kTokensPerPass = 8;

struct OpList {
    MulMatOp op[kMaxOpsPerLaunch];
    int32_t cta_begin[kMaxOpsPerLaunch + 1];
    int32_t n_ops;
};

__device__ __forceinline__ float4 ldx4(const float* p, bool vec) {
    if (vec) return __ldg(reinterpret_cast<const float4*>(p));
    return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q4_K row: lane handles qs bytes 4*lane..4*lane+3 of every block, i.e.
// 4 elements of sub-block 2p (low nibbles) and 4 of sub-block 2p+1 (high).
template <int NT>
__device__ __forceinline__ void row_q4_k(const uint8_t* wrow, const float* const* xs, int nt,
                                         int nblocks, bool vec, int lane, float (&acc)[NT]) {
    const int p = lane >> 3;
    const int l0 = (lane & 7) << 2;
    for (int b = 0; b < nblocks; ++b) {
        const uint8_t* blk = wrow + static_cast<size_t>(b) * 144;
        const uint32_t dm = ldg_u32(blk);
        uint32_t s[3];
        s[0] = ldg_u32(blk + 4);
        s[1] = ldg_u32(blk + 8);
        s[2] = ldg_u32(blk + 12);
        const uint32_t q = ldg_u32(blk + 16 + 4 * lane);
        const float d = f16_bits_to_f32(dm), dmin = f16_bits_to_f32(dm >> 16);
        int sc0, m0, sc1, m1;
        q4k_scale_min(s, 2 * p, sc0, m0);
        q4k_scale_min(s, 2 * p + 1, sc1, m1);
        const float ds0 = d * static_cast<float>(sc0), dm0 = dmin * static_cast<float>(m0);
        const float ds1 = d * static_cast<float>(sc1), dm1 = dmin * static_cast<float>(m1);
        float ql[4], qh[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ql[i] = static_cast<float>((q >> (8 * i)) & 0xFu);
            qh[i] = static_cast<float>((q >> (8 * i + 4)) & 0xFu);
        }
        const int k0 = b * 256 + 64 * p + l0;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            if (n < nt) {
                const float4 xl = ldx4(xs[n] + k0, vec);
                const float4 xh = ldx4(xs[n] + k0 + 32, vec);
                const float sl = ql[0] * xl.x + ql[1] * xl.y + ql[2] * xl.z + ql[3] * xl.w;
                const float sh = qh[0] * xh.x + qh[1] * xh.y + qh[2] * xh.z + qh[3] * xh.w;
                const float xsl = (xl.x + xl.y) + (xl.z + xl.w);
                const float xsh = (xh.x + xh.y) + (xh.z + xh.w);
                acc[n] += ds0 * sl - dm0 * xsl + ds1 * sh - dm1 * xsh;
            }
        }
    }
}

// IQ4_XS row: lane handles qs bytes 4*lane..4*lane+3 of every block, i.e.
// elements l0..l0+3 (low nibbles) and 16+l0..16+l0+3 (high nibbles) of
// sub-block j = lane/4, l0 = 4*(lane%4); the levels come from the table.
template <int NT>
__device__ __forceinline__ void row_iq4_xs(const uint8_t* wrow, const float* const* xs, int nt,
                                           int nblocks, bool vec, int lane, float (&acc)[NT]) {
    const int j = lane >> 2;
    const int l0 = (lane & 3) << 2;
    for (int b = 0; b < nblocks; ++b) {
        const uint8_t* blk = wrow + static_cast<size_t>(b) * 136;
        const float d = f16_bits_to_f32(ldg_u16(blk));
        const uint32_t sh = ldg_u16(blk + 2), sl = ldg_u16(blk + 4) | (ldg_u16(blk + 6) << 16);
        const uint32_t q = ldg_u32(blk + 8 + 4 * lane);
        const float dl = d * static_cast<float>(iq4xs_scale(sh, sl, j));
        float ql[4], qh[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ql[i] = static_cast<float>(iq4_level((q >> (8 * i)) & 0xFu));
            qh[i] = static_cast<float>(iq4_level((q >> (8 * i + 4)) & 0xFu));
        }
        const int k0 = b * 256 + 32 * j + l0;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            if (n < nt) {
                const float4 xl = ldx4(xs[n] + k0, vec);
                const float4 xh = ldx4(xs[n] + k0 + 16, vec);
                const float s = ql[0] * xl.x + ql[1] * xl.y + ql[2] * xl.z + ql[3] * xl.w + qh[0] * xh.x +
                                qh[1] * xh.y + qh[2] * xh.z + qh[3] * xh.w;
                acc[n] += dl * s;
            }
        }
    }
}

// Q5_K row: as Q4_K (qs at +48), with bit j of qh[l] as the fifth bit of
// sub-block j's element l.
template <int NT>
__device__ __forceinline__ void row_q5_k(const uint8_t* wrow, const float* const* xs, int nt,
                                         int nblocks, bool vec, int lane, float (&acc)[NT]) {
    const int p = lane >> 3;
    const int l0 = (lane & 7) << 2;
    for (int b = 0; b < nblocks; ++b) {
        const uint8_t* blk = wrow + static_cast<size_t>(b) * 176;
        const uint32_t dm = ldg_u32(blk);
        uint32_t s[3];
        s[0] = ldg_u32(blk + 4);
        s[1] = ldg_u32(blk + 8);
        s[2] = ldg_u32(blk + 12);
        const uint32_t q = ldg_u32(blk + 48 + 4 * lane);
        const uint32_t hb = ldg_u32(blk + 16 + l0);  // qh[l0 .. l0+3]
        const float d = f16_bits_to_f32(dm), dmin = f16_bits_to_f32(dm >> 16);
        int sc0, m0, sc1, m1;
        q4k_scale_min(s, 2 * p, sc0, m0);
        q4k_scale_min(s, 2 * p + 1, sc1, m1);
        const float ds0 = d * static_cast<float>(sc0), dm0 = dmin * static_cast<float>(m0);
        const float ds1 = d * static_cast<float>(sc1), dm1 = dmin * static_cast<float>(m1);
        float ql[4], qh[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ql[i] = static_cast<float>(((q >> (8 * i)) & 0xFu) | (((hb >> (8 * i + 2 * p)) & 1u) << 4));
            qh[i] = static_cast<float>(((q >> (8 * i + 4)) & 0xFu) | (((hb >> (8 * i + 2 * p + 1)) & 1u) << 4));
        }
        const int k0 = b * 256 + 64 * p + l0;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            if (n < nt) {
                const float4 xl = ldx4(xs[n] + k0, vec);
                const float4 xh = ldx4(xs[n] + k0 + 32, vec);
                const float sl = ql[0] * xl.x + ql[1] * xl.y + ql[2] * xl.z + ql[3] * xl.w;
                const float sh = qh[0] * xh.x + qh[1] * xh.y + qh[2] * xh.z + qh[3] * xh.w;
                const float xsl = (xl.x + xl.y) + (xl.z + xl.w);
                const float xsh = (xh.x + xh.y) + (xh.z + xh.w);
                acc[n] += ds0 * sl - dm0 * xsl + ds1 * sh - dm1 * xsh;
            }
        }
    }
}

// Q6_K row: lane handles l = 2*(lane%16), l+1 of half h = lane/16, i.e. the
// two elements at each of the four quarter offsets 0/32/64/96 of the half.
template <int NT>
__device__ __forceinline__ void row_q6_k(const uint8_t* wrow, const float* const* xs, int nt,
                                         int nblocks, int lane, float (&acc)[NT]) {
    const int h = lane >> 4;
    const int l = (lane & 15) << 1;
    const int is = l >> 4;
    for (int b = 0; b < nblocks; ++b) {
        const uint8_t* blk = wrow + static_cast<size_t>(b) * 210;
        const uint32_t qa = ldg_u16(blk + 64 * h + l);
        const uint32_t qb = ldg_u16(blk + 64 * h + 32 + l);
        const uint32_t qh = ldg_u16(blk + 128 + 32 * h + l);
        const float d = f16_bits_to_f32(ldg_u16(blk + 208));
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * h + is);
        const float s0 = d * static_cast<float>(sc[0]);
        const float s1 = d * static_cast<float>(sc[2]);
        const float s2 = d * static_cast<float>(sc[4]);
        const float s3 = d * static_cast<float>(sc[6]);
        float q[4][2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t a = (qa >> (8 * e)) & 0xffu, bb = (qb >> (8 * e)) & 0xffu;
            const uint32_t hh = (qh >> (8 * e)) & 0xffu;
            q[0][e] = static_cast<float>(static_cast<int>((a & 0xFu) | ((hh & 3u) << 4)) - 32);
            q[1][e] = static_cast<float>(static_cast<int>((bb & 0xFu) | (((hh >> 2) & 3u) << 4)) - 32);
            q[2][e] = static_cast<float>(static_cast<int>((a >> 4) | (((hh >> 4) & 3u) << 4)) - 32);
            q[3][e] = static_cast<float>(static_cast<int>((bb >> 4) | (((hh >> 6) & 3u) << 4)) - 32);
        }
        const int k0 = b * 256 + 128 * h + l;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            if (n < nt) {
                const float* x = xs[n] + k0;
                const float2 x0 = make_float2(__ldg(x), __ldg(x + 1));
                const float2 x1 = make_float2(__ldg(x + 32), __ldg(x + 33));
                const float2 x2 = make_float2(__ldg(x + 64), __ldg(x + 65));
                const float2 x3 = make_float2(__ldg(x + 96), __ldg(x + 97));
                acc[n] += s0 * (q[0][0] * x0.x + q[0][1] * x0.y) + s1 * (q[1][0] * x1.x + q[1][1] * x1.y) +
                          s2 * (q[2][0] * x2.x + q[2][1] * x2.y) + s3 * (q[3][0] * x3.x + q[3][1] * x3.y);
            }
        }
    }
}

// Q8_0 row: 8 blocks (256 elements) per warp step; lane handles 8 elements
// (4*2-byte loads, the blocks are only 2-byte aligned).
template <int NT>
__device__ __forceinline__ void row_q8_0(const uint8_t* wrow, const float* const* xs, int nt,
                                         int nblocks, bool vec, int lane, float (&acc)[NT]) {
    const int j = lane >> 2;
    const int part = lane & 3;
    for (int b0 = 0; b0 < nblocks; b0 += 8) {
        const int bi = b0 + j;
        if (bi < nblocks) {
            const uint8_t* blk = wrow + static_cast<size_t>(bi) * 34;
            const float d = f16_bits_to_f32(ldg_u16(blk));
            float q[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t v = ldg_u16(blk + 2 + 8 * part + 2 * i);
                q[2 * i] = static_cast<float>(static_cast<int8_t>(v & 0xffu));
                q[2 * i + 1] = static_cast<float>(static_cast<int8_t>(v >> 8));
            }
            const int k0 = bi * 32 + 8 * part;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                if (n < nt) {
                    const float4 xa = ldx4(xs[n] + k0, vec);
                    const float4 xb = ldx4(xs[n] + k0 + 4, vec);
                    const float s = q[0] * xa.x + q[1] * xa.y + q[2] * xa.z + q[3] * xa.w + q[4] * xb.x +
                                    q[5] * xb.y + q[6] * xb.z + q[7] * xb.w;
                    acc[n] += d * s;
                }
            }
        }
    }
}

// Q4_0 row: 8 blocks (256 elements) per warp step; lane handles 8 elements
// of block lane/4: part 0/1 the low nibbles of qs[0..7] / qs[8..15]
// (elements 0..15), part 2/3 their high nibbles (16..31).
template <int NT>
__device__ __forceinline__ void row_q4_0(const uint8_t* wrow, const float* const* xs, int nt,
                                         int nblocks, bool vec, int lane, float (&acc)[NT]) {
    const int j = lane >> 2;
    const int part = lane & 3;
    for (int b0 = 0; b0 < nblocks; b0 += 8) {
        const int bi = b0 + j;
        if (bi < nblocks) {
            const uint8_t* blk = wrow + static_cast<size_t>(bi) * 18;
            const float d = f16_bits_to_f32(ldg_u16(blk));
            const int sh = part >= 2 ? 4 : 0;
            float q[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t v = ldg_u16(blk + 2 + 8 * (part & 1) + 2 * i);
                q[2 * i] = static_cast<float>(static_cast<int>((v >> sh) & 0xFu) - 8);
                q[2 * i + 1] = static_cast<float>(static_cast<int>((v >> (8 + sh)) & 0xFu) - 8);
            }
            const int k0 = bi * 32 + 8 * part;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                if (n < nt) {
                    const float4 xa = ldx4(xs[n] + k0, vec);
                    const float4 xb = ldx4(xs[n] + k0 + 4, vec);
                    const float s = q[0] * xa.x + q[1] * xa.y + q[2] * xa.z + q[3] * xa.w + q[4] * xb.x +
                                    q[5] * xb.y + q[6] * xb.z + q[7] * xb.w;
                    acc[n] += d * s;
                }
            }
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const __grid_constant__ OpList L) {
    int oi = 0;
    while (oi + 1 < L.n_ops && static_cast<int>(blockIdx.x) >= L.cta_begin[oi + 1]) ++oi;
    const MulMatOp& op = L.op[oi];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t grow = static_cast<int64_t>(blockIdx.x - L.cta_begin[oi]) * kWarps + warp;
    const int64_t rows_total = static_cast<int64_t>(op.M) * op.ne2 * op.ne3;
    if (grow >= rows_total) return;
    const int m = static_cast<int>(grow % op.M);
    const int64_t bidx = grow / op.M;
    const int b2 = static_cast<int>(bidx % op.ne2), b3 = static_cast<int>(bidx / op.ne2);
    const uint8_t* wrow = op.w + static_cast<int64_t>(b2 / op.r2) * op.w_nb2 +
                          static_cast<int64_t>(b3 / op.r3) * op.w_nb3 + static_cast<int64_t>(m) * op.w_nb1;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(op.x) + b2 * op.x_nb2 + b3 * op.x_nb3;
    uint8_t* yb = reinterpret_cast<uint8_t*>(op.y) + b2 * op.y_nb2 + b3 * op.y_nb3;
    const bool vec = ((reinterpret_cast<uintptr_t>(xb) | static_cast<uintptr_t>(op.x_nb1)) & 15u) == 0;
    const int nblocks = op.K / ((op.type == kTypeQ8_0 || op.type == kTypeQ4_0) ? 32 : 256);

    for (int n0 = 0; n0 < op.N; n0 += NT) {
        const int nt = min(NT, op.N - n0);
        const float* xs[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n)
            xs[n] = reinterpret_cast<const float*>(xb + static_cast<int64_t>(n0 + (n < nt ? n : 0)) * op.x_nb1);
        float acc[NT];
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[n] = 0.f;
        if (op.type == kTypeQ4_K) {
            row_q4_k<NT>(wrow, xs, nt, nblocks, vec, lane, acc);
        } else if (op.type == kTypeQ5_K) {
            row_q5_k<NT>(wrow, xs, nt, nblocks, vec, lane, acc);
        } else if (op.type == kTypeQ6_K) {
            row_q6_k<NT>(wrow, xs, nt, nblocks, lane, acc);
        } else if (op.type == kTypeQ4_0) {
            row_q4_0<NT>(wrow, xs, nt, nblocks, vec, lane, acc);
        } else if (op.type == kTypeIQ4_XS) {
            row_iq4_xs<NT>(wrow, xs, nt, nblocks, vec, lane, acc);
        } else {
            row_q8_0<NT>(wrow, xs, nt, nblocks, vec, lane, acc);
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const float v = warp_sum(acc[n]);
            if (lane == 0 && n < nt)
                *reinterpret_cast<float*>(yb + static_cast<int64_t>(n0 + n) * op.y_nb1 + 4 * static_cast<int64_t>(m)) = v;
        }
    }
}

__global__ void dequant_kernel(int type, const uint8_t* __restrict__ src, float* __restrict__ dst, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (type == kTypeQ4_K) {
        dst[i] = q4k_dequant_elem(src + (i >> 8) * 144, static_cast<int>(i & 255));
    } else if (type == kTypeQ5_K) {
        dst[i] = q5k_dequant_elem(src + (i >> 8) * 176, static_cast<int>(i & 255));
    } else if (type == kTypeQ4_0) {
        dst[i] = q4_0_dequant_elem(src + (i >> 5) * 18, static_cast<int>(i & 31));
    } else if (type == kTypeQ6_K) {
        dst[i] = q6k_dequant_elem(src + (i >> 8) * 210, static_cast<int>(i & 255));
    } else if (type == kTypeIQ4_XS) {
        dst[i] = iq4xs_dequant_elem(src + (i >> 8) * 136, static_cast<int>(i & 255));
    } else {
        dst[i] = q8_0_dequant_elem(src + (i >> 5) * 34, static_cast<int>(i & 31));
    }
}

}  // namespace

const char* check_mulmat_op(const MulMatOp& op) {
    if (op.type != kTypeQ4_K && op.type != kTypeQ5_K && op.type != kTypeQ6_K && op.type != kTypeQ4_0 &&
        op.type != kTypeQ8_0 && op.type != kTypeIQ4_XS)
        return "unsupported src0 type";
    if (op.M <= 0 || op.K <= 0 || op.N <= 0 || op.ne2 <= 0 || op.ne3 <= 0) return "empty or negative shape";
    if (op.r2 <= 0 || op.r3 <= 0) return "bad broadcast factor";
    if (op.K % block_elems(op.type) != 0) return "K is not a multiple of the block size";
    const uintptr_t wa = reinterpret_cast<uintptr_t>(op.w);
    const int need = (op.type == kTypeQ4_K || op.type == kTypeQ5_K || op.type == kTypeIQ4_XS) ? 4 : 2;
    if ((wa | static_cast<uintptr_t>(op.w_nb1) | static_cast<uintptr_t>(op.w_nb2) |
         static_cast<uintptr_t>(op.w_nb3)) % need)
        return need == 4 ? "src0 data/strides must be 4-byte aligned for Q4_K/Q5_K/IQ4_XS"
                         : "src0 data/strides must be 2-byte aligned";
    if (op.w_nb1 < static_cast<int64_t>(op.K / block_elems(op.type)) * block_bytes(op.type)) return "src0 nb1 too small";
    if ((reinterpret_cast<uintptr_t>(op.x) | static_cast<uintptr_t>(op.x_nb1) | static_cast<uintptr_t>(op.x_nb2) |
         static_cast<uintptr_t>(op.x_nb3)) % 4)
        return "src1 must be 4-byte aligned";
    if ((reinterpret_cast<uintptr_t>(op.y) | static_cast<uintptr_t>(op.y_nb1) | static_cast<uintptr_t>(op.y_nb2) |
         static_cast<uintptr_t>(op.y_nb3)) % 4)
        return "dst must be 4-byte aligned";
    if (op.x_nb1 < 4LL * op.K) return "src1 nb1 too small";
    if (op.y_nb1 < 4LL * op.M) return "dst nb1 too small";
    return nullptr;
}

// Q4_K / Q5_K / Q6_K with 5 to 64 vectors (and 3 or 4 where the streaming
// kernel cannot take them), Q8_0 and IQ4_XS above 16 vectors run on the tcgen05
// small-batch GEMM, except small weights (at most 4096 x 4096) below 16
// vectors, where the mma.sync GEMM's shorter fixed costs win (13.5 against
// 15.1 us for Q4_K 4096 x 4096 at N = 8).
bool use_batched_tc(const MulMatOp& o) {
    if (!batched_tc_supported(o) || o.N < 3) return false;
    // Q8_0's and IQ4_XS's two weight planes (and IQ4_XS's level table) cost the
    // tcgen05 GEMM two to three times a Q4_K dequantization: the integer mma.sync
    // GEMM, which needs none, is faster up to 16 vectors (IQ4_XS 14336 x 4096 at
    // N = 8: 32.9 against 43.6 us; at N = 32: 54.6 against 47.2)
    if (o.type == kTypeQ8_0 || o.type == kTypeIQ4_XS)
        return o.N > 16 || (!batched_supported(o) && (o.N >= 5 || !stream_supported(&o, 1)));
    // Q6_K (also two planes) below 4096 x 4096 keeps the mma.sync GEMM through 16
    // vectors (1024 x 4096 at N = 16: 12.9 against 16.3 us)
    if (o.type == kTypeQ6_K && o.N <= 16 && static_cast<int64_t>(o.M) * o.K < 4096LL * 4096 && batched_supported(o))
        return false;
    if (o.N < 16 && static_cast<int64_t>(o.M) * o.K <= 4096LL * 4096 && batched_supported(o)) return false;
    return o.N >= 5 || !stream_supported(&o, 1);
}

size_t mulmat_workspace_bytes(const MulMatOp* ops, int n_ops) {
    size_t need = 0;
    for (int i = 0; i < n_ops; ++i) {
        size_t b = 0;
        if (prefill_supported(ops[i])) b = prefill_workspace_bytes(ops[i]);
        else if (use_batched_tc(ops[i])) b = batched_tc_workspace_bytes(ops[i]);
        else if (batched_supported(ops[i])) b = batched_workspace_bytes(ops[i]);
        need = b > need ? b : need;
    }
    return need;
}

int launch_mulmat(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms, void* workspace,
                  size_t workspace_bytes) {
    if (n_ops < 1 || n_ops > kMaxOpsPerLaunch) return -static_cast<int>(cudaErrorInvalidValue);
    // prefill-sized ops (Q4_K, Q5_K, Q8_0, Q4_0, IQ4_XS, or Q6_K rows the TMA can copy; N >= 65) and small batches (N >= 5, or 3-4 where
    // the streaming kernel cannot take them) run as tensor-core GEMMs, one
    // launch each; the rest together
    int launched = 0;
    MulMatOp rest[kMaxOpsPerLaunch];
    int n_rest = 0;
    for (int i = 0; i < n_ops; ++i) {
        if (prefill_supported(ops[i]) && workspace && workspace_bytes >= prefill_workspace_bytes(ops[i])) {
            const int rc = launch_prefill(ops[i], workspace, workspace_bytes, stream);
            if (rc < 0) return rc;
            launched += rc;
        } else if (use_batched_tc(ops[i]) && workspace && workspace_bytes >= batched_tc_workspace_bytes(ops[i])) {
            const int rc = launch_batched_tc(ops[i], workspace, workspace_bytes, stream, num_sms);
            if (rc < 0) return rc;
            launched += rc;
        } else if (batched_supported(ops[i]) && !(ops[i].N <= 4 && stream_supported(&ops[i], 1)) && workspace &&
                   workspace_bytes >= batched_workspace_bytes(ops[i])) {
            const int rc = launch_batched(ops[i], workspace, workspace_bytes, stream);
            if (rc < 0) return rc;
            launched += rc;
        } else {
            rest[n_rest++] = ops[i];
        }
    }
    if (n_rest == 0) return launched;
    const int rc = stream_supported(rest, n_rest) ? launch_stream(rest, n_rest, stream, num_sms)
                                                  : launch_mulmat_general(rest, n_rest, stream);
    return rc < 0 ? rc : launched + rc;
}

int launch_mulmat_general(const MulMatOp* ops, int n_ops, cudaStream_t stream) {
    if (n_ops < 1 || n_ops > kMaxOpsPerLaunch) return -static_cast<int>(cudaErrorInvalidValue);
    OpList L;
    L.n_ops = n_ops;
    int64_t ctas = 0;
    int max_n = 1;
    for (int i = 0; i < n_ops; ++i) {
        L.op[i] = ops[i];
        L.cta_begin[i] = static_cast<int32_t>(ctas);
        const int64_t rows = static_cast<int64_t>(ops[i].M) * ops[i].ne2 * ops[i].ne3;
        ctas += (rows + kWarps - 1) / kWarps;
        max_n = ops[i].N > max_n ? ops[i].N : max_n;
    }
    L.cta_begin[n_ops] = static_cast<int32_t>(ctas);
    if (ctas <= 0 || ctas > 0x7fffffffLL) return -static_cast<int>(cudaErrorInvalidValue);
    const dim3 grid(static_cast<unsigned>(ctas)), block(kWarps * 32);
    if (max_n <= 1) gemv_kernel<1><<<grid, block, 0, stream>>>(L);
    else if (max_n <= 2) gemv_kernel<2><<<grid, block, 0, stream>>>(L);
    else if (max_n <= 4) gemv_kernel<4><<<grid, block, 0, stream>>>(L);
    else gemv_kernel<kTokensPerPass><<<grid, block, 0, stream>>>(L);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -static_cast<int>(e);
}

int launch_dequantize(int type, const void* src, float* dst, int64_t n, cudaStream_t stream) {
    if (n <= 0) return 0;
    const int64_t blocks = (n + 255) / 256;
    dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(type, static_cast<const uint8_t*>(src), dst, n);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -static_cast<int>(e);
}

}  // namespace wllm
