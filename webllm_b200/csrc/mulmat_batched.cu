// Small-batch quantized MUL_MAT for Q8_0 weights (N >= 3 activation vectors:
// several sequences decoding together, the GEMV-to-GEMM crossover) on integer
// tensor cores (mma.sync m16n8k32, s8 x s8 -> s32).
//
//   y[m + M n] = sum_k W[m, k] x[k + K n]   (ggml MUL_MAT, matmul.ts:10-17)
//
// A Q8_0 block is 32 int8 quants q and an f16 scale d: W = d q. One MMA's
// k = 32 is exactly one block, so every MMA result is scaled by its rows' d
// in f32 and the quants enter the MMA as they are.
//
// Activations: a pre-pass turns x into two int8 limbs per element,
// x = (l0 + l1 / 128) / s with s = 127 / max|x| per 256 elements and vector
// (|error| <= max|x| / 32512), stored as [N][2][K] with the factors 1 / s as
// [K / 256][N rounded up to 4]. The eight B columns of an MMA are four vectors
// x two limbs.
//
// Tiling: a CTA (4 warps) computes 64 rows x NV vectors (NV = 8 .. 64); warp w
// rows 16 w .. 16 w + 15. K is walked in chunks of 256 (8 blocks): the chunk's
// raw rows (64 x 272 B) and limbs (NV x 2 x 256 B) go to shared memory with
// cp.async, 2 to 4 chunks in flight. Q8_0 blocks are 34 bytes, so a block sits at any
// even offset: A fragments come from aligned 32-bit loads and a funnel shift;
// B fragments from ldmatrix.
//
// Split K: grids below one wave of two CTAs per SM split the chunks S ways (grid z); each
// split stores its tile in workspace and the tile's last split sums the S
// tiles in split order (deterministic).
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
constexpr int kWRow = 272;                  // bytes of a row's chunk (8 blocks x 34)
constexpr int kXRow = kChunk + 16;          // bytes of a limb row in shared memory (ldmatrix bank spread)
constexpr int kMaxVec = 64;
constexpr int kSlotsB = 2 * 148;            // CTAs resident at once
constexpr int kMaxSplitsB = 16;

struct BatchedArgs {
    const uint8_t* w;
    int64_t w_nb1;
    const int8_t* xl;      // limbs [N][2][K]
    const float* inv_s;    // [K / 256][n_pad]
    float* y;
    int64_t y_nb1;         // bytes between output vectors
    int32_t M, K, N, n_pad;
    int32_t splits, chunks_per_split;
    float* partial;        // [tile][split][kMaxVec][kRowsB]
    unsigned* counters;    // [tile]
};

template <int NV>
__host__ __device__ constexpr int stage_bytes() {
    return kRowsB * kWRow + NV * 2 * kXRow + NV * 4;
}
// Pipeline depth: enough bytes in flight per SM (two CTAs) to cover the HBM
// latency, within the shared memory of two CTAs.
template <int NV>
__host__ __device__ constexpr int stages_of() {
    return NV <= 16 ? 4 : (NV == 32 ? 3 : 2);
}

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

// D = A (16x32 s8, row) * B (32x8 s8, col), s32.
__device__ __forceinline__ void imma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// 4 bytes at a 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* p) {
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);
    return __funnelshift_r(q[0], q[1], mis * 8);
}

// Pre-pass: one warp per (vector, 256-element block).
__global__ void x_limbs_kernel(const float* __restrict__ x, int64_t x_nb1, int8_t* __restrict__ xl,
                               float* __restrict__ inv_s, int K, int N, int n_pad) {
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
    uint32_t l0[2], l1[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int q0[4], q1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float e = v[4 * h + i];
            q0[i] = __float2int_rn(e * sc);                                     // |l0| <= 127
            q1[i] = __float2int_rn(fmaf(e, sc, -static_cast<float>(q0[i])) * 128.f);  // |l1| <= 64
        }
        l0[h] = __byte_perm(__byte_perm(q0[0], q0[1], 0x0040u), __byte_perm(q0[2], q0[3], 0x0040u), 0x5410u);
        l1[h] = __byte_perm(__byte_perm(q1[0], q1[1], 0x0040u), __byte_perm(q1[2], q1[3], 0x0040u), 0x5410u);
    }
    if (n < N) {
        int8_t* base = xl + (static_cast<int64_t>(n) * 2) * K + b * 256 + 8 * lane;
        *reinterpret_cast<uint2*>(base) = make_uint2(l0[0], l0[1]);
        *reinterpret_cast<uint2*>(base + K) = make_uint2(l1[0], l1[1]);
    }
    if (lane == 0) inv_s[static_cast<int64_t>(b) * n_pad + n] = mx * (1.f / 127.f);
}

template <int NV>
__global__ void __launch_bounds__(kThreadsB, 2) batched_q8_kernel(const __grid_constant__ BatchedArgs P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int SB = stage_bytes<NV>();
    constexpr int NT = NV / 4;  // MMA column tiles: 4 vectors x 2 limbs each
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int m0 = blockIdx.x * kRowsB, n0 = blockIdx.y * NV;
    const int nchunks = P.K / kChunk;
    const int ch0 = blockIdx.z * P.chunks_per_split;
    const int nch = min(nchunks - ch0, P.chunks_per_split);

    // one chunk's copies: 64 rows x 17 pieces of 16 B, NV x 2 limb rows x 16
    // pieces, NV factors (16 B pieces of 4)
    auto load = [&](int ch, int buf) {
        uint8_t* sw = smem + buf * SB;
        uint8_t* sx = sw + kRowsB * kWRow;
        uint8_t* ss = sx + NV * 2 * kXRow;
        const int k0 = (ch0 + ch) * kChunk;
        for (int i = threadIdx.x; i < kRowsB * 17; i += kThreadsB) {
            const int r = i / 17, pc = i - r * 17;
            const bool ok = m0 + r < P.M;
            const uint8_t* src = P.w + static_cast<int64_t>(ok ? m0 + r : 0) * P.w_nb1 + (k0 / 32) * 34 + 16 * pc;
            cp_async16(sw + r * kWRow + 16 * pc, src, ok);
        }
        for (int i = threadIdx.x; i < NV * 2 * 16; i += kThreadsB) {
            const int rowl = i >> 4, pc = i & 15;  // rowl = 2 v + limb
            const int v = rowl >> 1;
            const bool ok = n0 + v < P.N;
            const int8_t* src = P.xl + (static_cast<int64_t>(ok ? n0 + v : 0) * 2 + (rowl & 1)) * P.K + k0 + 16 * pc;
            cp_async16(sx + rowl * kXRow + 16 * pc, src, ok);
        }
        for (int i = threadIdx.x; i < NV / 4; i += kThreadsB) {
            const int v = 4 * i;
            const bool ok = n0 + v < P.n_pad;
            cp_async16(ss + 16 * i, P.inv_s + static_cast<int64_t>(ch0 + ch) * P.n_pad + (ok ? n0 + v : 0), ok);
        }
    };

    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = 0.f;

    constexpr int ST = stages_of<NV>();
#pragma unroll
    for (int sidx = 0; sidx < ST - 1; ++sidx) {
        if (sidx < nch) load(sidx, sidx);
        cp_async_commit();
    }
    for (int ch = 0; ch < nch; ++ch) {
        cp_async_wait<ST - 2>();  // chunk ch has landed
        __syncthreads();          // ... for every thread, and chunk ch - 1's buffer is free
        if (ch + ST - 1 < nch) load(ch + ST - 1, (ch + ST - 1) % ST);
        cp_async_commit();
        const uint8_t* sw = smem + (ch % ST) * SB;
        const uint8_t* sx = sw + kRowsB * kWRow;
        const float* ss = reinterpret_cast<const float*>(sx + NV * 2 * kXRow);
        float is[NT];  // 1 / s of this lane's vector in each column tile
#pragma unroll
        for (int t = 0; t < NT; ++t) is[t] = ss[4 * t + c];
        const uint8_t* rg = sw + (16 * warp + g) * kWRow;
        const uint8_t* rh = rg + 8 * kWRow;
        // ldmatrix row address: matrix mi = lane/8 (column tile 2 tp + mi/2, k half mi&1),
        // row rr = lane%8 = B column: vector rr/2, limb rr&1
        const int mi = lane >> 3, rr = lane & 7;
        const uint32_t xbase = smem_u32(sx) + static_cast<uint32_t>((2 * (4 * (mi >> 1) + (rr >> 1)) + (rr & 1)) * kXRow +
                                                                    16 * (mi & 1));
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint8_t* bg = rg + 34 * b;
            const uint8_t* bh = rh + 34 * b;
            const float dg = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bg));
            const float dh = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(bh));
            const uint32_t a0 = lds_u32_any(bg + 2 + 4 * c), a1 = lds_u32_any(bh + 2 + 4 * c);
            const uint32_t a2 = lds_u32_any(bg + 18 + 4 * c), a3 = lds_u32_any(bh + 18 + 4 * c);
#pragma unroll
            for (int tp = 0; tp < NT / 2; ++tp) {
                uint32_t xb[4];
                ldmatrix_x4(xb, xbase + static_cast<uint32_t>(tp * 8 * 2 * kXRow + 32 * b));
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int t = 2 * tp + h;
                    int D[4];
                    imma_s8(D, a0, a1, a2, a3, xb[2 * h], xb[2 * h + 1]);
                    const float vg = fmaf(static_cast<float>(D[1]), 0.0078125f, static_cast<float>(D[0]));
                    const float vh = fmaf(static_cast<float>(D[3]), 0.0078125f, static_cast<float>(D[2]));
                    acc[t][0] = fmaf(vg, dg * is[t], acc[t][0]);
                    acc[t][1] = fmaf(vh, dh * is[t], acc[t][1]);
                }
            }
        }
    }

    // ---- outputs: lane (g, c) holds rows 16 warp + g (+8) of vector 4 t + c ----
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (P.splits == 1) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int n = n0 + 4 * t + c;
            if (n >= P.N) continue;
            float* yn = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(P.y) + n * P.y_nb1);
            const int r = m0 + 16 * warp + g;
            if (r < P.M) yn[r] = acc[t][0];
            if (r + 8 < P.M) yn[r + 8] = acc[t][1];
        }
        return;
    }
    float* part = P.partial + (static_cast<int64_t>(tile) * P.splits + blockIdx.z) * (kMaxVec * kRowsB);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const int v = 4 * t + c;
        part[v * kRowsB + 16 * warp + g] = acc[t][0];
        part[v * kRowsB + 16 * warp + g + 8] = acc[t][1];
    }
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // this split's tile before the count
        last = atomicAdd(P.counters + tile, 1u) == static_cast<unsigned>(P.splits - 1);
        if (last) {
            P.counters[tile] = 0u;
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

int pick_nv(int N) { return N <= 8 ? 8 : (N <= 16 ? 16 : (N <= 32 ? 32 : 64)); }

void plan(const MulMatOp& o, int* nv, int* splits, int* cps) {
    *nv = pick_nv(o.N);
    const int tiles = ((o.M + kRowsB - 1) / kRowsB) * ((o.N + *nv - 1) / *nv);
    const int nchunks = o.K / kChunk;
    int s = kSlotsB / tiles;                         // at most one wave of two CTAs per SM
    s = s < kMaxSplitsB ? s : kMaxSplitsB;
    s = s < (nchunks + 1) / 2 ? s : (nchunks + 1) / 2;  // at least two chunks per split
    s = s > 1 ? s : 1;
    *cps = (nchunks + s - 1) / s;
    *splits = (nchunks + *cps - 1) / *cps;           // no empty split
}

size_t limbs_bytes(const MulMatOp& o) { return (static_cast<size_t>(o.N) * 2 * o.K + 255) & ~size_t(255); }
size_t factors_bytes(const MulMatOp& o) {
    const int n_pad = (o.N + 3) & ~3;
    return (static_cast<size_t>(o.K / 256) * n_pad * 4 + 255) & ~size_t(255);
}
size_t partial_bytes(const MulMatOp& o) {
    int nv, s, cps;
    plan(o, &nv, &s, &cps);
    if (s <= 1) return 0;
    const size_t tiles = static_cast<size_t>((o.M + kRowsB - 1) / kRowsB) * ((o.N + nv - 1) / nv);
    return tiles * s * kMaxVec * kRowsB * 4 + tiles * 4;
}

template <int NV>
cudaError_t launch_nv(const BatchedArgs& P, dim3 grid, cudaStream_t stream) {
    constexpr int smem = stages_of<NV>() * stage_bytes<NV>();
    static bool configured = false;
    if (!configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(batched_q8_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    batched_q8_kernel<NV><<<grid, kThreadsB, smem, stream>>>(P);
    return cudaGetLastError();
}

}  // namespace

bool batched_supported(const MulMatOp& o) {
    if (o.type != kTypeQ8_0 || o.N < 3 || o.ne2 != 1 || o.ne3 != 1) return false;
    if (o.K % 256 != 0 || o.M < 1) return false;
    if ((reinterpret_cast<uintptr_t>(o.w) | static_cast<uintptr_t>(o.w_nb1)) & 15) return false;  // 16-byte copies
    if ((reinterpret_cast<uintptr_t>(o.x) | static_cast<uintptr_t>(o.x_nb1)) & 15) return false;  // float4 reads
    return true;
}

size_t batched_workspace_bytes(const MulMatOp& o) { return limbs_bytes(o) + factors_bytes(o) + partial_bytes(o) + 256; }

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
    P.y = o.y;
    P.y_nb1 = o.y_nb1;
    P.M = o.M;
    P.K = o.K;
    P.N = o.N;
    P.n_pad = (o.N + 3) & ~3;
    P.splits = splits;
    P.chunks_per_split = cps;
    const int tiles_m = (o.M + kRowsB - 1) / kRowsB, tiles_n = (o.N + nv - 1) / nv;
    if (splits > 1) {
        P.partial = reinterpret_cast<float*>(ws + limbs_bytes(o) + factors_bytes(o));
        P.counters = reinterpret_cast<unsigned*>(P.partial + static_cast<size_t>(tiles_m) * tiles_n * splits * kMaxVec * kRowsB);
        const cudaError_t e = cudaMemsetAsync(P.counters, 0, static_cast<size_t>(tiles_m) * tiles_n * 4, stream);
        if (e != cudaSuccess) return -static_cast<int>(e);
    }
    {
        const int64_t items = static_cast<int64_t>(P.n_pad) * (o.K / 256);
        const int64_t blocks = (items * 32 + 255) / 256;
        x_limbs_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(o.x, o.x_nb1, const_cast<int8_t*>(P.xl),
                                                                          const_cast<float*>(P.inv_s), o.K, o.N,
                                                                          P.n_pad);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return -static_cast<int>(e);
    }
    const dim3 grid(tiles_m, tiles_n, splits);
    cudaError_t e;
    switch (nv) {
        case 8: e = launch_nv<8>(P, grid, stream); break;
        case 16: e = launch_nv<16>(P, grid, stream); break;
        case 32: e = launch_nv<32>(P, grid, stream); break;
        default: e = launch_nv<64>(P, grid, stream); break;
    }
    return e == cudaSuccess ? 2 : -static_cast<int>(e);
}

}  // namespace wllm
