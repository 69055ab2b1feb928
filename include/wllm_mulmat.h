/*
 * wllm_mulmat — C ABI of the B200 quantized MUL_MAT library.
 *
 * Drop-in for one op of paulrobello/webllm: ggml MUL_MAT with a GGUF
 * quantized src0 (Q4_K, Q5_K, Q6_K, Q4_0, Q8_0, IQ4_XS) and f32 src1/dst. The ABI mirrors the
 * JSEP operator-plugin seam the ggml backend calls per graph node
 * (src/inference/jsep/index.ts:1-21,129-305): seven callbacks
 * alloc/free/write/read/clear/run_op/sync over integer buffer handles, and
 * the same per-op descriptor words (src/inference/jsep/ops/matmul.ts:22-41).
 *
 * Conventions
 *  - Status codes (src/inference/jsep/index.ts:31-33, jsep/README.md):
 *      WLLM_STATUS_OK (0), WLLM_STATUS_NOT_IMPLEMENTED (1: op or type not
 *      handled here, the caller falls back), WLLM_STATUS_FAILED (-1: bad
 *      arguments, validation failure or CUDA error; wllm_last_error() has
 *      the message). No C++ exception crosses this boundary.
 *  - Every call is ordered on the library's single CUDA stream for the
 *    bound device (one process or one host thread per GPU). The library
 *    guards its state with a mutex; calls from several host threads are
 *    serialised, not concurrent.
 *  - Buffers are owned by the library (handles >= 1, never 0). Host
 *    pointers passed in are owned by the caller and only used during the
 *    call.
 */
#ifndef WLLM_MULMAT_H
#define WLLM_MULMAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported with default visibility even when the library is built with
 * -fvisibility=hidden. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define WLLM_STATUS_OK 0
#define WLLM_STATUS_NOT_IMPLEMENTED 1
#define WLLM_STATUS_FAILED (-1)

/* ggml_op / ggml_type ids (jsep/index.ts:45, ggml-wasm.ts:8-25). */
#define WLLM_GGML_OP_MUL_MAT 29
#define WLLM_TYPE_F32 0
#define WLLM_TYPE_F16 1
#define WLLM_TYPE_Q4_0 2
#define WLLM_TYPE_Q8_0 8
#define WLLM_TYPE_Q4_K 12
#define WLLM_TYPE_Q5_K 13
#define WLLM_TYPE_Q6_K 14
#define WLLM_TYPE_IQ4_XS 23

/* Descriptor geometry (matmul.ts:22-41): [op, n_src, dst block, src blocks...],
 * each block = buf_handle, offset, type, ne[4] lo, ne[4] hi, nb[4] lo, nb[4] hi.
 * The hi halves carry the upper 32 bits of ne/nb (large vocab projections
 * exceed 2^31 bytes). `offset` is one unsigned 32-bit word. */
#define WLLM_TENSOR_BLOCK_I32 19
#define WLLM_DESC_HEADER_I32 2

/* Per-callback invocation counters (jsep/index.ts:92-105, JsepCounters)
 * plus the library's device-memory accounting. */
typedef struct wllm_counters {
    uint64_t alloc, free, write, read, clear, run_op, sync;
    uint64_t kernels_launched;   /* kernels this library launched */
    uint64_t bytes_live;         /* bytes held by live handles */
    uint64_t bytes_reserved;     /* bytes held from cudaMalloc incl. free lists */
} wllm_counters;

/* Bind the library to a CUDA device and create its stream. Replaces
 * installJsepCallbacks(module, device) (jsep/index.ts:129). Calling it again
 * for the same device is a no-op; for another device it fails. */
int32_t wllm_init(int32_t device);

/* Release every buffer, the stream and cached scratch. Replaces
 * destroyJsepCallbacks (jsep/index.ts:400-413). */
int32_t wllm_shutdown(void);

/* jsepAlloc(size) -> handle >= 1 (jsep/index.ts:163-166,
 * GpuDataManager.alloc gpu-data-manager.ts:65-103). Memory comes from
 * cudaMalloc through a size-class free list; size must be > 0. */
int32_t wllm_alloc(uint64_t size, int32_t* out_handle);

/* jsepFree(handle): idempotent, unknown handles are a no-op
 * (gpu-data-manager.ts:105-116). */
int32_t wllm_free(int32_t handle);

/* jsepWrite(h, off, ptr, size) (jsep/index.ts:173-228,
 * GpuDataManager.write gpu-data-manager.ts:128-142): stream-ordered after
 * every earlier call; the host buffer may be reused when the call returns. */
int32_t wllm_write(int32_t handle, uint64_t offset, const void* host_src, uint64_t size);

/* jsepRead(h, off, ptr, size) (jsep/index.ts:230-254, readAsync
 * gpu-data-manager.ts:144-170): waits for every earlier call, then copies. */
int32_t wllm_read(int32_t handle, uint64_t offset, void* host_dst, uint64_t size);

/* Non-blocking readback, begin/poll/finish/cancel
 * (webgpu-bridge.cpp:353-370, backend_tensor_get_async_*). poll returns
 * 1 when ready, 0 while pending, -1 on error. */
int32_t wllm_read_async_begin(int32_t handle, uint64_t offset, uint64_t size, int32_t* out_request);
int32_t wllm_read_async_poll(int32_t request);
int32_t wllm_read_async_finish(int32_t request, void* host_dst, uint64_t size);
int32_t wllm_read_async_cancel(int32_t request);

/* jsepClear(h, value, off, size) (jsep/index.ts:256-268): byte fill. */
int32_t wllm_clear(int32_t handle, int32_t value, uint64_t offset, uint64_t size);

/* jsepRunOp(descriptorPtr, descriptorWords, opParamsPtr, opParamsLen)
 * (jsep/index.ts:270-300) -> dispatchMatmul (matmul.ts:555-1000).
 * Enqueues the op and returns. op != MUL_MAT, or src0 of a type this
 * library does not compute, returns WLLM_STATUS_NOT_IMPLEMENTED; shape,
 * stride, range or handle violations return WLLM_STATUS_FAILED. dst may
 * share a buffer with a source; overlapping byte ranges are computed into
 * library scratch and copied back (matmul.ts:675-958 divert path). */
int32_t wllm_run_op(const int32_t* desc, int32_t desc_words,
                    const void* op_params, int32_t op_params_len);

/* Several independent MUL_MAT descriptors in one kernel launch (for example
 * the q/k/v projections of a layer, which read the same src1). No
 * descriptor's dst may overlap another's sources. Extension of the
 * jsepRunOp seam: ggml's graph_compute sees such sibling nodes together. */
int32_t wllm_run_ops(const int32_t* const* descs, const int32_t* desc_words, int32_t n_ops);

/* jsepSync() (jsep/index.ts:302-305): waits for all enqueued work and
 * reports any asynchronous CUDA error. */
int32_t wllm_sync(void);

/* Copy the last error message (NUL-terminated, truncated to len). Returns
 * the full message length. */
int32_t wllm_last_error(char* buf, int32_t len);

/* Counter snapshot (JsepCounters, jsep/index.ts:92-105). */
int32_t wllm_get_counters(wllm_counters* out);

/* Device address and capacity of a buffer handle, for hosts that drive the
 * device-pointer entry points below on library-owned memory. */
int32_t wllm_buffer_device_ptr(int32_t handle, void** out_ptr, uint64_t* out_size);

/* Device-pointer MUL_MAT on a caller-chosen stream (NULL = the library
 * stream): y[m + y_stride*n] = sum_k W[m,k] * x[k + x_stride*n] with W
 * given as M rows of w_row_bytes raw GGUF blocks. Same math as
 * wllm_run_op; used by the row-sharded multi-GPU path, where each rank
 * passes its own row slice. The pointers must be device memory of the
 * bound device; the library checks alignment, not extents. */
int32_t wllm_mul_mat(int32_t src0_type, const void* w, int64_t w_row_bytes,
                     const float* x, int64_t x_stride,
                     float* y, int64_t y_stride,
                     int32_t M, int32_t K, int32_t N, void* stream);

/* One device-pointer MUL_MAT for wllm_mul_mat_batch. */
typedef struct wllm_mulmat_args {
    int32_t src0_type;
    int32_t M, K, N;
    const void* w;
    int64_t w_row_bytes;
    const float* x;
    int64_t x_stride;  /* floats between activation vectors */
    float* y;
    int64_t y_stride;  /* floats between output vectors */
} wllm_mulmat_args;

/* Up to 16 independent device-pointer MUL_MATs in one kernel launch on
 * `stream` (NULL = the library stream). */
int32_t wllm_mul_mat_batch(const wllm_mulmat_args* ops, int32_t n_ops, void* stream);

/* wllm_mul_mat_batch with the RMS_NORM and gain MUL that feed the ops fused
 * into the kernel: each op reads x / sqrt(mean(x^2) + eps) * gain (per
 * vector, mean over K) instead of x. Replaces the graph's
 * MUL_MAT(W, MUL(RMS_NORM(x, eps), gain)) chain
 * (src/inference/model-inference.ts:2281 attn_norm -> q/k/v,
 * :2478-2481 ffn_norm -> gate/up; RMS_NORM per
 * src/inference/jsep/ops/rms-norm.ts:14-15,61-67). gain: K floats, 16-byte
 * aligned, or NULL for RMS_NORM alone; every op has the same K. Decode
 * shapes only (N <= 4, as the streaming kernel takes them): NOT_IMPLEMENTED
 * otherwise, and the caller runs the three ops unfused. x is not modified.
 * No op's y may overlap an op's x or the gain (WLLM_STATUS_FAILED). */
int32_t wllm_mul_mat_rms_norm_batch(const wllm_mulmat_args* ops, int32_t n_ops, const float* gain, float eps,
                                    void* stream);

/* GLU kinds for wllm_mul_mat_glu_batch. */
#define WLLM_GLU_SWIGLU 1 /* silu(gate) * up: gate / (1 + e^-gate), times up */
#define WLLM_GLU_GELU 2   /* gelu(gate) * up: tanh form, rounded to f16 like ggml's CPU GELU */

/* wllm_mul_mat_batch with the GLU between the FFN's gate/up projections and
 * its down projection fused into the kernel: the ops' x is the gate
 * projection's output, and each op reads act(x) * up instead of x. Replaces
 * MUL_MAT(W_down, SWIGLU_SPLIT(gate, up)) (src/inference/model-inference.ts:
 * 2484-2489; op_swiglu_split, src/wasm/webgpu-bridge.cpp:272-275) and, with
 * WLLM_GLU_GELU, the Gemma form MUL_MAT(W_down, MUL(GELU(gate), up))
 * (model-inference.ts:2486-2487). up: laid out like x, up_stride floats
 * between vectors (a multiple of 4), 16-byte aligned. Every op reads the
 * same x. Decode
 * shapes only (N <= 4, as the streaming kernel takes them): NOT_IMPLEMENTED
 * otherwise, and the caller runs the ops unfused. gate and up are not
 * modified; no op's y may overlap them (WLLM_STATUS_FAILED). */
int32_t wllm_mul_mat_glu_batch(const wllm_mulmat_args* ops, int32_t n_ops, const float* up, int64_t up_stride,
                               int32_t glu, void* stream);

/* ---- Row-sharded multi-GPU decode with the gather fused into the GEMV ----
 * No counterpart in the reference, which runs on one browser GPU. The
 * reference's op semantics (dst[m + M*n], matmul.ts:10-17) make output rows
 * independent, so rank r computes a contiguous row slice of every weight. The
 * GEMV's epilogue writes each finished row into every rank's gather buffer
 * over NVLink (peer memory opened with CUDA IPC, plain stores), and the last
 * CTA of the launch signals the peers. The next tensor-parallel launch on a
 * rank (or wllm_tp_wait) waits, bounded, until every peer has signalled the
 * previous one: no collective library call on the data path. */
#define WLLM_MAX_RANKS 8
#define WLLM_IPC_HANDLE_BYTES 64

/* Peer-mappable device memory: its own cudaMalloc, zero-filled, with the
 * 64-byte IPC handle another process on the node opens with wllm_ipc_open. */
int32_t wllm_ipc_alloc(uint64_t size, void** out_ptr, void* out_handle);
int32_t wllm_ipc_open(const void* handle, void** out_ptr);
int32_t wllm_ipc_close(void* ptr);  /* a pointer from wllm_ipc_open */
int32_t wllm_ipc_free(void* ptr);   /* a pointer from wllm_ipc_alloc */

/* The ranks of one node. sig[r] is rank r's signal array (WLLM_MAX_RANKS
 * uint32, wllm_ipc_alloc'd on rank r and opened on the others); state is this
 * rank's private counter block (4 uint32, zeroed). Every rank issues the same
 * sequence of tensor-parallel launches. */
typedef struct wllm_tp_group {
    int32_t world, rank;
    uint32_t* sig[WLLM_MAX_RANKS];
    uint32_t* state;
} wllm_tp_group;

/* Where every rank keeps this rank's rows of one op: y_rank[r] is rank r's
 * copy (y_rank[rank] is the op's own y). */
typedef struct wllm_tp_outputs {
    float* y_rank[WLLM_MAX_RANKS];
} wllm_tp_outputs;

/* wllm_mul_mat_batch for one rank's row slices, each output row also written
 * to y_rank[r] of every other rank r. Only the streaming decode shapes
 * (N <= 2, K % 256 == 0, 16-byte aligned activations) are accepted;
 * anything else returns WLLM_STATUS_FAILED. */
int32_t wllm_mul_mat_batch_tp(const wllm_mulmat_args* ops, const wllm_tp_outputs* outs, int32_t n_ops,
                              const wllm_tp_group* group, void* stream);

/* Enqueues a wait (bounded) until every peer has signalled the rank's last
 * tensor-parallel launch, so its gathered outputs are complete. A time-out
 * is reported by the next wllm_sync. */
int32_t wllm_tp_wait(const wllm_tp_group* group, void* stream);

/* How many polls a bounded device-side wait of the decode kernels (pipeline
 * barriers, a peer rank's signal) makes before it gives up, for launches
 * enqueued after this call; 0 restores the default of 2^26 polls (seconds).
 * A wait that gives up records an error code, the kernel still ends, and the
 * next wllm_sync returns WLLM_STATUS_FAILED with the code in its message: a
 * dead or stalled peer rank surfaces as an error rather than a hang. A small
 * limit can fail healthy but slow launches. No counterpart in the reference
 * (one browser GPU, no device-side waits). */
int32_t wllm_set_wait_limit(uint32_t polls);

/* The library's CUDA stream (a cudaStream_t), so a host can order its own
 * work (collectives, events) with the library's. */
int32_t wllm_get_stream(void** out_stream);

/* Record the run_op/run_ops calls made between begin and end into a CUDA
 * graph instead of executing them, then replay the whole sequence with one
 * launch per token (the graph_compute of a fixed decode graph,
 * webgpu-bridge.cpp:317-320). Buffer writes, reads, clears and syncs are
 * rejected while recording. Replays read the buffers' current contents. */
int32_t wllm_graph_begin(void);
int32_t wllm_graph_end(int32_t* out_graph);
int32_t wllm_graph_launch(int32_t graph);
int32_t wllm_graph_destroy(int32_t graph);

/* Prefill MUL_MAT that allocates nothing: the same arguments and result as
 * wllm_mul_mat for the prefill path (Q4_K, Q5_K, Q8_0 or Q4_0 weights; Q6_K or
 * IQ4_XS with rows of a multiple of 16 bytes, or of an even number of bytes with
 * M a multiple of the 2, 4 or 8 rows that make a multiple of 16 (IQ4_XS: pairs
 * only); N >= 65 vectors, 16-byte
 * aligned weights and activations), with the f16 activation workspace
 * in a fixed 16 MiB device array of the library instead of library-allocated
 * memory: N * K * 2 + 256 bytes must fit, otherwise WLLM_STATUS_FAILED with
 * the sizes in wllm_last_error(). No cudaMalloc or cudaFree happens. The
 * first call on a device looks up the array's address, so it must come
 * before any stream capture. Calls that overlap in time (other streams or
 * host threads) race on the one workspace. No counterpart in the reference
 * (its WGSL dispatch allocates its own buffers). */
int32_t wllm_mul_mat_prefill_static(int32_t src0_type, const void* w, int64_t w_row_bytes,
                                    const float* x, int64_t x_stride,
                                    float* y, int64_t y_stride,
                                    int32_t M, int32_t K, int32_t N, void* stream);

/* Device dequantization of n elements (n a multiple of the block size) of
 * raw GGUF blocks to f32. Replaces the libllama oracle shim
 * webllm_dequantize_q4_K (webgpu-bridge.cpp:692-708) on the device, for
 * Q4_K, Q5_K, Q6_K, Q4_0, Q8_0 and IQ4_XS. Returns -1 on bad arguments. */
int32_t wllm_dequantize(int32_t type, const void* src, float* dst, int64_t n, void* stream);

/* Library build/version string. */
const char* wllm_version(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif
