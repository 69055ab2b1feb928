// Internal interface between the C-ABI runtime (runtime.cpp) and the CUDA
// kernels (*.cu). Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wllm {

// GGUF block geometry (src/models/gguf-parser.ts:273-294).
constexpr int kTypeF32 = 0;
constexpr int kTypeQ4_0 = 2;
constexpr int kTypeQ8_0 = 8;
constexpr int kTypeQ4_K = 12;
constexpr int kTypeQ5_K = 13;
constexpr int kTypeQ6_K = 14;
constexpr int kTypeIQ4_XS = 23;

inline int block_elems(int type) {
    switch (type) {
        case kTypeQ4_0: return 32;
        case kTypeQ8_0: return 32;
        case kTypeQ4_K: return 256;
        case kTypeQ5_K: return 256;
        case kTypeQ6_K: return 256;
        case kTypeIQ4_XS: return 256;
        case kTypeF32: return 1;
        default: return 0;
    }
}
inline int block_bytes(int type) {
    switch (type) {
        case kTypeQ4_0: return 18;
        case kTypeQ8_0: return 34;
        case kTypeQ4_K: return 144;
        case kTypeQ5_K: return 176;
        case kTypeQ6_K: return 210;
        case kTypeIQ4_XS: return 136;
        case kTypeF32: return 4;
        default: return 0;
    }
}

// One MUL_MAT node in device terms. Rows of W are raw GGUF blocks.
// y[m, n, b2, b3] = sum_k W[m, k, b2/r2, b3/r3] * x[k, n, b2, b3].
struct MulMatOp {
    const uint8_t* w;
    const float* x;
    float* y;
    int64_t w_nb1, w_nb2, w_nb3;  // bytes
    int64_t x_nb1, x_nb2, x_nb3;  // bytes
    int64_t y_nb1, y_nb2, y_nb3;  // bytes
    int32_t type, M, K, N;
    int32_t ne2, ne3;             // batch dims of x / y
    int32_t r2, r3;               // broadcast factors x.ne2/w.ne2, x.ne3/w.ne3
};

constexpr int kMaxOpsPerLaunch = 16;
// Device ordinals tracked by per-device caches (function attributes, symbol
// addresses): one process may drive several devices.
constexpr int kMaxDevices = 64;

// Checks alignment/shape preconditions the kernels rely on. Returns an
// empty string when the op can be launched, else the reason.
const char* check_mulmat_op(const MulMatOp& op);

// Enqueue n_ops independent MUL_MAT ops (1 <= n_ops <= kMaxOpsPerLaunch)
// on `stream`. Returns the number of kernels launched (>= 1) or a negative
// cudaError_t on launch failure.
int launch_mulmat(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms, void* workspace = nullptr,
                  size_t workspace_bytes = 0);
// The general kernel only (every shape; used by tests to compare paths).
int launch_mulmat_general(const MulMatOp* ops, int n_ops, cudaStream_t stream);

// Streaming decode kernel (mulmat_stream.cu): ne2 = ne3 = 1, N <= 2,
// K % 256 == 0, K <= 16384, 16-byte aligned activations (and Q4_K rows).
// Row-sharded launch: where the other ranks keep this rank's output rows and
// the signal arrays (see wllm_mul_mat_batch_tp in wllm_mulmat.h).
constexpr int kMaxRanks = 8;
struct TpLaunch {
    int32_t world, rank;
    uint32_t* sig[kMaxRanks];                     // rank r's signal array
    uint32_t* state;                              // this rank's counters: [0] CTAs done, [1] launches done
    float* y_peer[kMaxOpsPerLaunch][kMaxRanks];  // op i's rows on rank r (own rank unused)
};

// Fused prologue of every op's activations before the streaming GEMV.
enum ProKind : int32_t {
    kProNone = 0,
    kProNorm = 1,    // RMS_NORM (+ gain): x / sqrt(mean(x^2) + eps) * gain (gain null: none)
    kProSwiglu = 2,  // silu(x) * up
    kProGelu = 3,    // gelu(x) * up (tanh form, f16-rounded like ggml's CPU GELU)
};
struct ProLaunch {
    int32_t kind;
    const float* gain;  // kProNorm
    float eps;          // kProNorm
    const float* up;    // kProSwiglu / kProGelu: the up projection's output, laid out like x
    int64_t up_nb1;     // bytes between its vectors
};

bool stream_supported(const MulMatOp* ops, int n_ops);
int launch_stream(const MulMatOp* ops, int n_ops, cudaStream_t stream, int num_sms, const TpLaunch* tp = nullptr,
                  const ProLaunch* pro = nullptr);
// One-thread kernel that waits (bounded) for every peer's signal of the
// rank's last row-sharded launch.
int launch_tp_wait(const TpLaunch& tp, cudaStream_t stream);
// Error code recorded by a bounded wait that timed out (0 = none); clears it.
unsigned read_and_clear_stream_error();
// Polls a bounded wait of the streaming kernel (and the row-sharded peer
// wait) makes before it gives up; 0 restores the default (2^26, seconds).
void set_stream_wait_limit(uint32_t polls);

// Prefill GEMM (mulmat_prefill.cu): Q4_K, Q5_K, Q8_0 and Q4_0 weights, or Q6_K with
// rows of 16-byte multiples (or 8-byte, M even), with N >= kPrefillMinN vectors on tcgen05 tensor cores (f16 operands, f32 accumulation). The
// activations are first converted to f16 into caller-provided workspace of
// prefill_workspace_bytes(op) bytes (256-byte aligned). Returns the number of
// kernels launched (2) or a negative cudaError_t.
constexpr int kPrefillMinN = 65;
bool prefill_supported(const MulMatOp& op);
size_t prefill_workspace_bytes(const MulMatOp& op);
// The least workspace launch_prefill accepts (no K split).
size_t prefill_min_workspace_bytes(const MulMatOp& op);
int launch_prefill(const MulMatOp& op, void* workspace, size_t workspace_bytes, cudaStream_t stream);
unsigned read_and_clear_prefill_error();

// Small-batch GEMM (mulmat_batched.cu): Q8_0, Q4_K and Q6_K weights with
// N >= 3 vectors on integer tensor cores; workspace holds the activation limbs,
// factors and sub-block sums (and split-K partial tiles). Returns the number of kernels launched (2) or a negative
// cudaError_t.
bool batched_supported(const MulMatOp& op);
size_t batched_workspace_bytes(const MulMatOp& op);
int launch_batched(const MulMatOp& op, void* workspace, size_t workspace_bytes, cudaStream_t stream);

// Small-batch GEMM on tcgen05 (mulmat_batched_tc.cu): Q4_K and Q5_K weights,
// 1 <= N <= 64 vectors, exact to about 2^-22 of each activation (f16 hi/lo
// activations against the integer-scaled quants); workspace holds the
// activation and sums images and the split-K partial tiles. Returns the
// number of kernels launched (2) or a negative cudaError_t.
bool batched_tc_supported(const MulMatOp& op);
size_t batched_tc_workspace_bytes(const MulMatOp& op);
int launch_batched_tc(const MulMatOp& op, void* workspace, size_t workspace_bytes, cudaStream_t stream, int num_sms);
unsigned read_and_clear_btc_error();

// Size of the prefill path's fixed device workspace (wllm_mul_mat_prefill_static):
// ops with N * K * 2 + 256 bytes of f16 activations up to this size.
constexpr size_t kPrefillStaticWorkspaceBytes = 16u << 20;
// Its device address (looked up on first use on the current device); null and
// *err set on failure.
void* prefill_static_workspace(const char** err);

// Workspace the launch of `ops` needs (0 if none).
size_t mulmat_workspace_bytes(const MulMatOp* ops, int n_ops);

// Device dequantization of n elements to f32 (bit-exact with the oracle).
int launch_dequantize(int type, const void* src, float* dst, int64_t n, cudaStream_t stream);

}  // namespace wllm
