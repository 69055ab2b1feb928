// C-ABI runtime of libwllm_mulmat: buffer handles, descriptor decoding,
// validation and dispatch of quantized MUL_MAT onto the CUDA kernels.
//
// Mirrors the JSEP op-plugin runtime of paulrobello/webllm:
//   installJsepCallbacks / jsepAlloc..jsepSync   src/inference/jsep/index.ts:129-305
//   GpuDataManager (handles >= 1, idempotent free) src/inference/jsep/gpu-data-manager.ts:55-205
//   readDescriptor / dispatchMatmul validation    src/inference/jsep/ops/matmul.ts:150-181,555-1000
// Buffers live in HBM (cudaMalloc) behind a size-class free list; every call
// is ordered on one CUDA stream, which plays the role of the WebGPU queue.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/wllm_mulmat.h"
#include "wllm_internal.h"

namespace {

using wllm::MulMatOp;

struct Buffer {
    void* ptr = nullptr;
    uint64_t size = 0;  // requested bytes
    uint64_t cap = 0;   // bytes held (size class)
};

struct AsyncRead {
    void* pinned = nullptr;
    uint64_t size = 0;
    cudaEvent_t done = nullptr;
};

struct State {
    std::mutex mu;
    int device = -1;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    std::unordered_map<int32_t, Buffer> live;
    std::map<uint64_t, std::vector<void*>> free_lists;  // cap -> blocks
    int32_t next_handle = 1;
    wllm_counters counters{};
    std::string last_error;
    void* scratch = nullptr;  // divert target for aliased dst
    uint64_t scratch_cap = 0;
    void* workspace = nullptr;  // kernel workspace (f16 activations of the prefill GEMM)
    uint64_t workspace_cap = 0;
    std::unordered_map<int32_t, AsyncRead> reads;
    int32_t next_request = 1;
    bool capturing = false;
    uint64_t captured_kernels = 0;
    std::unordered_map<int32_t, cudaGraphExec_t> graphs;
    std::unordered_map<int32_t, uint64_t> graph_kernels;
    int32_t next_graph = 1;
    std::unordered_set<void*> ipc_owned;   // wllm_ipc_alloc
    std::unordered_set<void*> ipc_opened;  // wllm_ipc_open
};

State& S() {
    static State* s = new State();  // never destroyed: safe at process exit
    return *s;
}

int32_t fail(State& s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    s.last_error = buf;
    std::fprintf(stderr, "[wllm] %s\n", buf);
    return WLLM_STATUS_FAILED;
}

int32_t cuda_fail(State& s, cudaError_t e, const char* what) {
    return fail(s, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Size classes: < 1 MiB -> next power of two (>= 1 KiB); otherwise rounded
// up to 64 KiB, so large weight buffers waste at most 64 KiB. Every block
// carries 256 spare bytes so vector loads that round a tensor's end up to
// 16 bytes stay inside the allocation.
uint64_t size_class(uint64_t size) {
    const uint64_t need = size + 256;
    if (need < (1ull << 20)) {
        uint64_t c = 1024;
        while (c < need) c <<= 1;
        return c;
    }
    const uint64_t g = 64ull << 10;
    return (need + g - 1) / g * g;
}

// The src0 types this library runs (others: NOT_IMPLEMENTED, the caller falls back).
bool quant_type_supported(int32_t t) {
    return t == WLLM_TYPE_Q4_K || t == WLLM_TYPE_Q5_K || t == WLLM_TYPE_Q6_K || t == WLLM_TYPE_Q4_0 ||
           t == WLLM_TYPE_Q8_0 || t == WLLM_TYPE_IQ4_XS;
}

bool ensure_init(State& s) {
    if (s.device >= 0) return true;
    fail(s, "wllm_init has not been called");
    return false;
}

// Calls that copy to or from the host, or wait, cannot be recorded.
bool not_capturing(State& s, const char* what) {
    if (!s.capturing) return true;
    fail(s, "%s is not allowed while a graph is being recorded", what);
    return false;
}

Buffer* find(State& s, int32_t h) {
    auto it = s.live.find(h);
    return it == s.live.end() ? nullptr : &it->second;
}

int32_t release_all(State& s) {
    for (auto& kv : s.live) cudaFree(kv.second.ptr);
    s.live.clear();
    for (auto& kv : s.free_lists)
        for (void* p : kv.second) cudaFree(p);
    s.free_lists.clear();
    if (s.scratch) cudaFree(s.scratch);
    s.scratch = nullptr;
    s.scratch_cap = 0;
    if (s.workspace) cudaFree(s.workspace);
    s.workspace = nullptr;
    s.workspace_cap = 0;
    for (auto& kv : s.reads) {
        if (kv.second.done) cudaEventDestroy(kv.second.done);
        if (kv.second.pinned) cudaFreeHost(kv.second.pinned);
    }
    s.reads.clear();
    for (auto& kv : s.graphs) cudaGraphExecDestroy(kv.second);
    s.graphs.clear();
    s.graph_kernels.clear();
    for (void* p : s.ipc_opened) cudaIpcCloseMemHandle(p);
    s.ipc_opened.clear();
    for (void* p : s.ipc_owned) cudaFree(p);
    s.ipc_owned.clear();
    s.counters.bytes_live = 0;
    s.counters.bytes_reserved = 0;
    return WLLM_STATUS_OK;
}

// ---- descriptor decoding (matmul.ts:22-41,150-181) ----

struct TensorMeta {
    int32_t handle;
    uint32_t offset;
    int32_t type;
    int64_t ne[4];
    int64_t nb[4];
};

TensorMeta read_block(const int32_t* w) {
    TensorMeta t;
    t.handle = w[0];
    t.offset = static_cast<uint32_t>(w[1]);
    t.type = w[2];
    for (int i = 0; i < 4; ++i) {
        t.ne[i] = static_cast<int64_t>(static_cast<uint64_t>(static_cast<uint32_t>(w[3 + i])) |
                                       (static_cast<uint64_t>(static_cast<uint32_t>(w[7 + i])) << 32));
        t.nb[i] = static_cast<int64_t>(static_cast<uint64_t>(static_cast<uint32_t>(w[11 + i])) |
                                       (static_cast<uint64_t>(static_cast<uint32_t>(w[15 + i])) << 32));
    }
    return t;
}

// Byte span [first, last) the tensor touches inside its buffer.
bool tensor_span(const TensorMeta& t, int64_t inner_bytes, uint64_t* lo, uint64_t* hi) {
    uint64_t extent = static_cast<uint64_t>(inner_bytes);
    for (int i = 1; i < 4; ++i) {
        if (t.ne[i] <= 0 || t.nb[i] < 0) return false;
        extent += static_cast<uint64_t>(t.ne[i] - 1) * static_cast<uint64_t>(t.nb[i]);
    }
    *lo = t.offset;
    *hi = static_cast<uint64_t>(t.offset) + extent;
    return true;
}

struct Decoded {
    MulMatOp op;
    int32_t dst_handle;
    uint64_t dst_lo, dst_hi;
    int32_t src_handle[2];
    uint64_t src_lo[2], src_hi[2];
    TensorMeta dst;
};

// Returns OK, NOT_IMPLEMENTED or FAILED (with last_error set).
int32_t decode_mulmat(State& s, const int32_t* desc, int32_t desc_words, Decoded* out) {
    if (!desc || desc_words < WLLM_DESC_HEADER_I32) return fail(s, "run_op: null or short descriptor");
    const int32_t op = desc[0], n_src = desc[1];
    if (op != WLLM_GGML_OP_MUL_MAT) return WLLM_STATUS_NOT_IMPLEMENTED;
    if (n_src != 2) return fail(s, "dispatchMatmul: expected 2 srcs, got %d", n_src);
    if (desc_words < WLLM_DESC_HEADER_I32 + 3 * WLLM_TENSOR_BLOCK_I32)
        return fail(s, "run_op: descriptor has %d words, need %d", desc_words,
                    WLLM_DESC_HEADER_I32 + 3 * WLLM_TENSOR_BLOCK_I32);
    const TensorMeta dst = read_block(desc + 2);
    const TensorMeta src0 = read_block(desc + 2 + WLLM_TENSOR_BLOCK_I32);
    const TensorMeta src1 = read_block(desc + 2 + 2 * WLLM_TENSOR_BLOCK_I32);

    if (!quant_type_supported(src0.type))
        return WLLM_STATUS_NOT_IMPLEMENTED;  // F32/F16 and other quant types: caller falls back
    if (src1.type != WLLM_TYPE_F32 || dst.type != WLLM_TYPE_F32)
        return fail(s, "dispatchMatmul: only src1=F32, dst=F32 (got src1=%d, dst=%d)", src1.type, dst.type);

    const int64_t K = src0.ne[0], M = src0.ne[1], N = src1.ne[1];
    for (int i = 0; i < 4; ++i)
        if (src0.ne[i] <= 0 || src1.ne[i] <= 0 || dst.ne[i] <= 0)
            return fail(s, "dispatchMatmul: non-positive ne");
    if (src1.ne[0] != K || dst.ne[0] != M || dst.ne[1] != N)
        return fail(s, "dispatchMatmul: shape mismatch src0=[%lld,%lld] src1=[%lld,%lld] dst=[%lld,%lld]",
                    (long long)K, (long long)M, (long long)src1.ne[0], (long long)N, (long long)dst.ne[0],
                    (long long)dst.ne[1]);
    if (src1.ne[2] % src0.ne[2] != 0 || src1.ne[3] % src0.ne[3] != 0)
        return fail(s, "dispatchMatmul: GQA broadcast invariant violated (src1.ne2=%lld src0.ne2=%lld)",
                    (long long)src1.ne[2], (long long)src0.ne[2]);
    if (dst.ne[2] != src1.ne[2] || dst.ne[3] != src1.ne[3]) return fail(s, "dispatchMatmul: dst batch dims differ from src1");
    const int be = wllm::block_elems(src0.type), bb = wllm::block_bytes(src0.type);
    if (K % be != 0) return fail(s, "dispatchMatmul: K=%lld is not a multiple of %d", (long long)K, be);
    if (M > 0x7fffffffLL || K > 0x7fffffffLL || N > 0x7fffffffLL || src1.ne[2] > 0x7fffffffLL ||
        src1.ne[3] > 0x7fffffffLL)
        return fail(s, "dispatchMatmul: dimension exceeds 2^31");
    if (src0.nb[0] != bb) return fail(s, "dispatchMatmul: src0 nb0=%lld, expected block size %d", (long long)src0.nb[0], bb);
    if (src1.nb[0] != 4 || dst.nb[0] != 4) return fail(s, "dispatchMatmul: src1/dst must be contiguous f32 along ne0");

    Buffer* b0 = find(s, src0.handle);
    Buffer* b1 = find(s, src1.handle);
    Buffer* bd = find(s, dst.handle);
    if (!b0 || !b1 || !bd)
        return fail(s, "dispatchMatmul: invalid handle (src0=%d src1=%d dst=%d)", src0.handle, src1.handle, dst.handle);

    uint64_t lo0, hi0, lo1, hi1, lod, hid;
    const int64_t row_bytes = (K / be) * bb;
    if (!tensor_span(src0, row_bytes, &lo0, &hi0) || !tensor_span(src1, 4 * K, &lo1, &hi1) ||
        !tensor_span(dst, 4 * M, &lod, &hid))
        return fail(s, "dispatchMatmul: negative stride");
    if (hi0 > b0->size || hi1 > b1->size || hid > bd->size)
        return fail(s, "dispatchMatmul: tensor extends past its buffer (src0 %llu/%llu, src1 %llu/%llu, dst %llu/%llu)",
                    (unsigned long long)hi0, (unsigned long long)b0->size, (unsigned long long)hi1,
                    (unsigned long long)b1->size, (unsigned long long)hid, (unsigned long long)bd->size);

    MulMatOp& m = out->op;
    m.w = static_cast<const uint8_t*>(b0->ptr) + src0.offset;
    m.x = reinterpret_cast<const float*>(static_cast<const uint8_t*>(b1->ptr) + src1.offset);
    m.y = reinterpret_cast<float*>(static_cast<uint8_t*>(bd->ptr) + dst.offset);
    m.w_nb1 = src0.nb[1];
    m.w_nb2 = src0.nb[2];
    m.w_nb3 = src0.nb[3];
    m.x_nb1 = src1.nb[1];
    m.x_nb2 = src1.nb[2];
    m.x_nb3 = src1.nb[3];
    m.y_nb1 = dst.nb[1];
    m.y_nb2 = dst.nb[2];
    m.y_nb3 = dst.nb[3];
    m.type = src0.type;
    m.M = static_cast<int32_t>(M);
    m.K = static_cast<int32_t>(K);
    m.N = static_cast<int32_t>(N);
    m.ne2 = static_cast<int32_t>(src1.ne[2]);
    m.ne3 = static_cast<int32_t>(src1.ne[3]);
    m.r2 = static_cast<int32_t>(src1.ne[2] / src0.ne[2]);
    m.r3 = static_cast<int32_t>(src1.ne[3] / src0.ne[3]);
    if (const char* why = wllm::check_mulmat_op(m)) return fail(s, "dispatchMatmul: %s", why);

    out->dst = dst;
    out->dst_handle = dst.handle;
    out->dst_lo = lod;
    out->dst_hi = hid;
    out->src_handle[0] = src0.handle;
    out->src_lo[0] = lo0;
    out->src_hi[0] = hi0;
    out->src_handle[1] = src1.handle;
    out->src_lo[1] = lo1;
    out->src_hi[1] = hi1;
    return WLLM_STATUS_OK;
}

bool overlaps(int32_t ha, uint64_t la, uint64_t ua, int32_t hb, uint64_t lb, uint64_t ub) {
    return ha == hb && la < ub && lb < ua;
}

void* get_scratch(State& s, uint64_t bytes) {
    if (s.scratch_cap >= bytes) return s.scratch;
    if (s.capturing) return nullptr;  // cannot allocate or wait while recording
    if (s.scratch) {
        cudaStreamSynchronize(s.stream);
        cudaFree(s.scratch);
        s.counters.bytes_reserved -= s.scratch_cap;
    }
    s.scratch = nullptr;
    s.scratch_cap = 0;
    if (cudaMalloc(&s.scratch, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    s.scratch_cap = bytes;
    s.counters.bytes_reserved += bytes;
    return s.scratch;
}

// Grows the kernel workspace to `bytes` (kept across calls; not while a graph
// is being recorded, since that cannot allocate or wait).
void* get_workspace(State& s, uint64_t bytes) {
    if (s.workspace_cap >= bytes) return s.workspace;
    if (s.capturing) return nullptr;
    if (s.workspace) {
        cudaStreamSynchronize(s.stream);
        cudaFree(s.workspace);
        s.counters.bytes_reserved -= s.workspace_cap;
    }
    s.workspace = nullptr;
    s.workspace_cap = 0;
    if (cudaMalloc(&s.workspace, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    s.workspace_cap = bytes;
    s.counters.bytes_reserved += bytes;
    return s.workspace;
}

int32_t launch(State& s, const MulMatOp* ops, int n, cudaStream_t stream) {
    const size_t need = wllm::mulmat_workspace_bytes(ops, n);
    void* ws = need ? get_workspace(s, need) : nullptr;
    if (need && !ws)
        return fail(s, "MUL_MAT: cannot %s %llu bytes of kernel workspace",
                    s.capturing ? "grow (while recording a graph) to" : "allocate", (unsigned long long)need);
    const int rc = wllm::launch_mulmat(ops, n, stream, s.num_sms, ws, ws ? s.workspace_cap : 0);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "MUL_MAT launch");
    if (s.capturing) s.captured_kernels += static_cast<uint64_t>(rc);
    else s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

// Converts and checks device-pointer ops; nonzero status (already reported)
// on failure.
int32_t ops_from_args(State& s, const char* what, const wllm_mulmat_args* ops, int32_t n_ops, MulMatOp* m) {
    if (!ops || n_ops < 1 || n_ops > wllm::kMaxOpsPerLaunch)
        return fail(s, "%s: n_ops=%d outside 1..%d", what, n_ops, wllm::kMaxOpsPerLaunch);
    for (int i = 0; i < n_ops; ++i) {
        const wllm_mulmat_args& a = ops[i];
        if (!quant_type_supported(a.src0_type)) return WLLM_STATUS_NOT_IMPLEMENTED;
        if (!a.w || !a.x || !a.y) return fail(s, "%s: null pointer in op %d", what, i);
        MulMatOp& o = m[i];
        o = MulMatOp{};
        o.w = static_cast<const uint8_t*>(a.w);
        o.x = a.x;
        o.y = a.y;
        o.w_nb1 = a.w_row_bytes;
        o.w_nb2 = o.w_nb3 = a.w_row_bytes * a.M;
        o.x_nb1 = 4 * a.x_stride;
        o.x_nb2 = o.x_nb3 = 4 * a.x_stride * a.N;
        o.y_nb1 = 4 * a.y_stride;
        o.y_nb2 = o.y_nb3 = 4 * a.y_stride * a.N;
        o.type = a.src0_type;
        o.M = a.M;
        o.K = a.K;
        o.N = a.N;
        o.ne2 = o.ne3 = 1;
        o.r2 = o.r3 = 1;
        if (const char* why = wllm::check_mulmat_op(o)) return fail(s, "%s op %d: %s", what, i, why);
    }
    return WLLM_STATUS_OK;
}

// Checks a row-sharded group and copies it into the kernel's form.
int32_t tp_from_group(State& s, const char* what, const wllm_tp_group* g, wllm::TpLaunch* t) {
    if (!g) return fail(s, "%s: null group", what);
    if (g->world < 2 || g->world > WLLM_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
        return fail(s, "%s: world=%d rank=%d (world must be 2..%d)", what, g->world, g->rank, WLLM_MAX_RANKS);
    if (!g->state) return fail(s, "%s: null state", what);
    *t = wllm::TpLaunch{};
    t->world = g->world;
    t->rank = g->rank;
    t->state = g->state;
    for (int r = 0; r < g->world; ++r) {
        if (!g->sig[r]) return fail(s, "%s: null signal array of rank %d", what, r);
        t->sig[r] = g->sig[r];
    }
    return WLLM_STATUS_OK;
}

}  // namespace

extern "C" {

int32_t wllm_init(int32_t device) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (s.device >= 0) {
        if (s.device == device) return WLLM_STATUS_OK;
        return fail(s, "wllm_init: already bound to device %d", s.device);
    }
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(s, "wllm_init: device %d out of range (%d devices)", device, count);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaSetDevice");
    e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaStreamCreate");
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0) s.num_sms = sms;
    s.device = device;
    return WLLM_STATUS_OK;
}

int32_t wllm_shutdown(void) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (s.device < 0) return WLLM_STATUS_OK;
    cudaSetDevice(s.device);
    if (s.capturing) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(s.stream, &g);
        if (g) cudaGraphDestroy(g);
        s.capturing = false;
    }
    cudaStreamSynchronize(s.stream);
    release_all(s);
    cudaStreamDestroy(s.stream);
    s.stream = nullptr;
    s.device = -1;
    return WLLM_STATUS_OK;
}

int32_t wllm_alloc(uint64_t size, int32_t* out_handle) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!out_handle) return fail(s, "wllm_alloc: null out_handle");
    *out_handle = 0;
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (size == 0) return fail(s, "GpuDataManager.alloc: invalid size 0");
    s.counters.alloc++;
    const uint64_t cap = size_class(size);
    Buffer b;
    b.size = size;
    b.cap = cap;
    auto it = s.free_lists.find(cap);
    if (it != s.free_lists.end() && !it->second.empty()) {
        b.ptr = it->second.back();
        it->second.pop_back();
    } else {
        cudaError_t e = cudaMalloc(&b.ptr, cap);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return cuda_fail(s, e, "cudaMalloc");
        }
        s.counters.bytes_reserved += cap;
    }
    const int32_t h = s.next_handle++;
    s.live[h] = b;
    s.counters.bytes_live += size;
    *out_handle = h;
    return WLLM_STATUS_OK;
}

int32_t wllm_free(int32_t handle) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.live.find(handle);
    if (it == s.live.end()) return WLLM_STATUS_OK;  // idempotent
    s.counters.free++;
    // The block may still be read by enqueued kernels; it only returns to the
    // free list, and a later alloc reuses it in stream order.
    s.free_lists[it->second.cap].push_back(it->second.ptr);
    s.counters.bytes_live -= it->second.size;
    s.live.erase(it);
    return WLLM_STATUS_OK;
}

int32_t wllm_write(int32_t handle, uint64_t offset, const void* host_src, uint64_t size) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!not_capturing(s, "wllm_write")) return WLLM_STATUS_FAILED;
    s.counters.write++;
    Buffer* b = find(s, handle);
    if (!b) return fail(s, "GpuDataManager.write: invalid handle %d", handle);
    if (offset > b->size || size > b->size - offset) return fail(s, "wllm_write: range past end of buffer");
    if (size == 0) return WLLM_STATUS_OK;
    if (!host_src) return fail(s, "wllm_write: null host pointer");
    cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(b->ptr) + offset, host_src, size, cudaMemcpyHostToDevice,
                                    s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_write");
    // Pinned sources are read asynchronously by the DMA engine; wait so the
    // caller may reuse the buffer on return (pageable sources are staged
    // before cudaMemcpyAsync returns).
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, host_src) == cudaSuccess && attr.type == cudaMemoryTypeHost) {
        e = cudaStreamSynchronize(s.stream);
        if (e != cudaSuccess) return cuda_fail(s, e, "wllm_write sync");
    }
    cudaGetLastError();
    return WLLM_STATUS_OK;
}

int32_t wllm_read(int32_t handle, uint64_t offset, void* host_dst, uint64_t size) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!not_capturing(s, "wllm_read")) return WLLM_STATUS_FAILED;
    s.counters.read++;
    Buffer* b = find(s, handle);
    if (!b) return fail(s, "GpuDataManager.readAsync: invalid handle %d", handle);
    if (offset > b->size || size > b->size - offset) return fail(s, "wllm_read: range past end of buffer");
    if (size == 0) return WLLM_STATUS_OK;
    if (!host_dst) return fail(s, "wllm_read: null host pointer");
    cudaError_t e = cudaMemcpyAsync(host_dst, static_cast<uint8_t*>(b->ptr) + offset, size, cudaMemcpyDeviceToHost,
                                    s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_read");
    e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_read sync");
    return WLLM_STATUS_OK;
}

int32_t wllm_read_async_begin(int32_t handle, uint64_t offset, uint64_t size, int32_t* out_request) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!out_request) return fail(s, "wllm_read_async_begin: null out_request");
    *out_request = 0;
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!not_capturing(s, "wllm_read_async_begin")) return WLLM_STATUS_FAILED;
    s.counters.read++;
    Buffer* b = find(s, handle);
    if (!b) return fail(s, "wllm_read_async_begin: invalid handle %d", handle);
    if (offset > b->size || size > b->size - offset || size == 0)
        return fail(s, "wllm_read_async_begin: bad range");
    AsyncRead r;
    r.size = size;
    cudaError_t e = cudaMallocHost(&r.pinned, size);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaMallocHost");
    e = cudaEventCreateWithFlags(&r.done, cudaEventDisableTiming);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(r.pinned, static_cast<uint8_t*>(b->ptr) + offset, size, cudaMemcpyDeviceToHost, s.stream);
    if (e == cudaSuccess) e = cudaEventRecord(r.done, s.stream);
    if (e != cudaSuccess) {
        if (r.done) cudaEventDestroy(r.done);
        cudaFreeHost(r.pinned);
        return cuda_fail(s, e, "wllm_read_async_begin");
    }
    const int32_t id = s.next_request++;
    s.reads[id] = r;
    *out_request = id;
    return WLLM_STATUS_OK;
}

int32_t wllm_read_async_poll(int32_t request) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.reads.find(request);
    if (it == s.reads.end()) return fail(s, "wllm_read_async_poll: unknown request %d", request);
    const cudaError_t e = cudaEventQuery(it->second.done);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    return cuda_fail(s, e, "wllm_read_async_poll");
}

int32_t wllm_read_async_finish(int32_t request, void* host_dst, uint64_t size) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.reads.find(request);
    if (it == s.reads.end()) return fail(s, "wllm_read_async_finish: unknown request %d", request);
    AsyncRead r = it->second;
    s.reads.erase(it);
    cudaError_t e = cudaEventSynchronize(r.done);
    int32_t rc = WLLM_STATUS_OK;
    if (e != cudaSuccess) rc = cuda_fail(s, e, "wllm_read_async_finish");
    else if (!host_dst || size > r.size) rc = fail(s, "wllm_read_async_finish: bad destination or size");
    else std::memcpy(host_dst, r.pinned, size);
    cudaEventDestroy(r.done);
    cudaFreeHost(r.pinned);
    return rc;
}

int32_t wllm_read_async_cancel(int32_t request) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.reads.find(request);
    if (it == s.reads.end()) return WLLM_STATUS_OK;
    cudaEventSynchronize(it->second.done);
    cudaEventDestroy(it->second.done);
    cudaFreeHost(it->second.pinned);
    s.reads.erase(it);
    return WLLM_STATUS_OK;
}

int32_t wllm_clear(int32_t handle, int32_t value, uint64_t offset, uint64_t size) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!not_capturing(s, "wllm_clear")) return WLLM_STATUS_FAILED;
    s.counters.clear++;
    Buffer* b = find(s, handle);
    if (!b) return fail(s, "GpuDataManager.clear: invalid handle %d", handle);
    if (offset > b->size || size > b->size - offset) return fail(s, "wllm_clear: range past end of buffer");
    if (size == 0) return WLLM_STATUS_OK;
    const cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(b->ptr) + offset, value & 0xff, size, s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_clear");
    return WLLM_STATUS_OK;
}

static int32_t run_ops_locked(State& s, const int32_t* const* descs, const int32_t* words, int32_t n_ops) {
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (n_ops < 1 || n_ops > wllm::kMaxOpsPerLaunch)
        return fail(s, "wllm_run_ops: n_ops=%d outside 1..%d", n_ops, wllm::kMaxOpsPerLaunch);
    Decoded dec[wllm::kMaxOpsPerLaunch];
    for (int i = 0; i < n_ops; ++i) {
        const int32_t rc = decode_mulmat(s, descs[i], words[i], &dec[i]);
        if (rc != WLLM_STATUS_OK) return rc;
    }
    // A dst that overlaps a source of any op in the launch is computed into
    // scratch and copied back afterwards (the divert of matmul.ts:675-958).
    bool divert = false;
    for (int i = 0; i < n_ops && !divert; ++i)
        for (int j = 0; j < n_ops && !divert; ++j)
            for (int k = 0; k < 2; ++k)
                if (overlaps(dec[i].dst_handle, dec[i].dst_lo, dec[i].dst_hi, dec[j].src_handle[k], dec[j].src_lo[k],
                             dec[j].src_hi[k]))
                    divert = true;
    for (int i = 0; i < n_ops && !divert; ++i)
        for (int j = i + 1; j < n_ops; ++j)
            if (overlaps(dec[i].dst_handle, dec[i].dst_lo, dec[i].dst_hi, dec[j].dst_handle, dec[j].dst_lo, dec[j].dst_hi))
                return fail(s, "wllm_run_ops: two ops write overlapping dst ranges");
    if (!divert) {
        MulMatOp ops[wllm::kMaxOpsPerLaunch];
        for (int i = 0; i < n_ops; ++i) ops[i] = dec[i].op;
        return launch(s, ops, n_ops, s.stream);
    }
    // Divert: each op's dst goes to a contiguous [M, N, ne2, ne3] f32 region.
    uint64_t total = 0;
    std::vector<uint64_t> off(n_ops);
    for (int i = 0; i < n_ops; ++i) {
        const MulMatOp& m = dec[i].op;
        off[i] = total;
        total += 4ull * m.M * m.N * m.ne2 * m.ne3;
        total = (total + 255) / 256 * 256;
    }
    uint8_t* tmp = static_cast<uint8_t*>(get_scratch(s, total));
    if (!tmp) return fail(s, "dispatchMatmul: cannot allocate %llu bytes of divert scratch", (unsigned long long)total);
    MulMatOp ops[wllm::kMaxOpsPerLaunch];
    for (int i = 0; i < n_ops; ++i) {
        ops[i] = dec[i].op;
        ops[i].y = reinterpret_cast<float*>(tmp + off[i]);
        ops[i].y_nb1 = 4LL * ops[i].M;
        ops[i].y_nb2 = ops[i].y_nb1 * ops[i].N;
        ops[i].y_nb3 = ops[i].y_nb2 * ops[i].ne2;
    }
    int32_t rc = launch(s, ops, n_ops, s.stream);
    if (rc != WLLM_STATUS_OK) return rc;
    for (int i = 0; i < n_ops; ++i) {
        const MulMatOp& m = dec[i].op;
        for (int b3 = 0; b3 < m.ne3; ++b3)
            for (int b2 = 0; b2 < m.ne2; ++b2) {
                uint8_t* dst = reinterpret_cast<uint8_t*>(m.y) + b2 * m.y_nb2 + b3 * m.y_nb3;
                const uint8_t* src = tmp + off[i] + (static_cast<uint64_t>(b3) * m.ne2 + b2) * 4ull * m.M * m.N;
                const cudaError_t e = cudaMemcpy2DAsync(dst, m.y_nb1, src, 4ull * m.M, 4ull * m.M, m.N,
                                                        cudaMemcpyDeviceToDevice, s.stream);
                if (e != cudaSuccess) return cuda_fail(s, e, "divert copy-back");
            }
    }
    return WLLM_STATUS_OK;
}

int32_t wllm_run_op(const int32_t* desc, int32_t desc_words, const void* op_params, int32_t op_params_len) {
    (void)op_params;
    (void)op_params_len;  // MUL_MAT carries no op params
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    s.counters.run_op++;
    const int32_t* d[1] = {desc};
    return run_ops_locked(s, d, &desc_words, 1);
}

int32_t wllm_run_ops(const int32_t* const* descs, const int32_t* desc_words, int32_t n_ops) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    s.counters.run_op += n_ops > 0 ? static_cast<uint64_t>(n_ops) : 0;
    if (!descs || !desc_words) return fail(s, "wllm_run_ops: null arguments");
    for (int i = 0; i < n_ops; ++i) {
        if (!descs[i] || desc_words[i] < WLLM_DESC_HEADER_I32) return fail(s, "wllm_run_ops: bad descriptor %d", i);
        if (descs[i][0] != WLLM_GGML_OP_MUL_MAT) return WLLM_STATUS_NOT_IMPLEMENTED;
    }
    return run_ops_locked(s, descs, desc_words, n_ops);
}

int32_t wllm_sync(void) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!not_capturing(s, "wllm_sync")) return WLLM_STATUS_FAILED;
    s.counters.sync++;
    cudaError_t e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_sync");
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_sync (pending error)");
    const unsigned kerr = wllm::read_and_clear_stream_error() | (wllm::read_and_clear_prefill_error() << 8) |
                          (wllm::read_and_clear_btc_error() << 16);
    if (kerr)
        return fail(s,
                    "wllm_sync: a kernel gave up waiting (code 0x%x: bits 0-1 a pipeline barrier, 2 a row-sharded "
                    "peer's signal, 3 an in-flight copy; bits 8-15 the prefill GEMM, 16+ the small-batch tcgen05 GEMM)",
                    kerr);
    return WLLM_STATUS_OK;
}

int32_t wllm_set_wait_limit(uint32_t polls) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    wllm::set_stream_wait_limit(polls);
    return WLLM_STATUS_OK;
}

int32_t wllm_last_error(char* buf, int32_t len) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (buf && len > 0) {
        const size_t n = std::min<size_t>(static_cast<size_t>(len - 1), s.last_error.size());
        std::memcpy(buf, s.last_error.data(), n);
        buf[n] = '\0';
    }
    return static_cast<int32_t>(s.last_error.size());
}

int32_t wllm_get_counters(wllm_counters* out) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!out) return fail(s, "wllm_get_counters: null out");
    *out = s.counters;
    return WLLM_STATUS_OK;
}

int32_t wllm_buffer_device_ptr(int32_t handle, void** out_ptr, uint64_t* out_size) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    Buffer* b = find(s, handle);
    if (!b || !out_ptr) return fail(s, "wllm_buffer_device_ptr: invalid handle %d", handle);
    *out_ptr = b->ptr;
    if (out_size) *out_size = b->size;
    return WLLM_STATUS_OK;
}

int32_t wllm_mul_mat(int32_t src0_type, const void* w, int64_t w_row_bytes, const float* x, int64_t x_stride,
                     float* y, int64_t y_stride, int32_t M, int32_t K, int32_t N, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!quant_type_supported(src0_type)) return WLLM_STATUS_NOT_IMPLEMENTED;
    if (!w || !x || !y) return fail(s, "wllm_mul_mat: null pointer");
    MulMatOp m{};
    m.w = static_cast<const uint8_t*>(w);
    m.x = x;
    m.y = y;
    m.w_nb1 = w_row_bytes;
    m.w_nb2 = m.w_nb3 = w_row_bytes * M;
    m.x_nb1 = 4 * x_stride;
    m.x_nb2 = m.x_nb3 = 4 * x_stride * N;
    m.y_nb1 = 4 * y_stride;
    m.y_nb2 = m.y_nb3 = 4 * y_stride * N;
    m.type = src0_type;
    m.M = M;
    m.K = K;
    m.N = N;
    m.ne2 = m.ne3 = 1;
    m.r2 = m.r3 = 1;
    if (const char* why = wllm::check_mulmat_op(m)) return fail(s, "wllm_mul_mat: %s", why);
    return launch(s, &m, 1, stream ? static_cast<cudaStream_t>(stream) : s.stream);
}

int32_t wllm_mul_mat_prefill_static(int32_t src0_type, const void* w, int64_t w_row_bytes, const float* x,
                                    int64_t x_stride, float* y, int64_t y_stride, int32_t M, int32_t K, int32_t N,
                                    void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!w || !x || !y) return fail(s, "wllm_mul_mat_prefill_static: null pointer");
    MulMatOp m{};
    m.w = static_cast<const uint8_t*>(w);
    m.x = x;
    m.y = y;
    m.w_nb1 = w_row_bytes;
    m.w_nb2 = m.w_nb3 = w_row_bytes * M;
    m.x_nb1 = 4 * x_stride;
    m.x_nb2 = m.x_nb3 = 4 * x_stride * N;
    m.y_nb1 = 4 * y_stride;
    m.y_nb2 = m.y_nb3 = 4 * y_stride * N;
    m.type = src0_type;
    m.M = M;
    m.K = K;
    m.N = N;
    m.ne2 = m.ne3 = 1;
    m.r2 = m.r3 = 1;
    if (const char* why = wllm::check_mulmat_op(m)) return fail(s, "wllm_mul_mat_prefill_static: %s", why);
    if (!wllm::prefill_supported(m))
        return fail(s,
                    "wllm_mul_mat_prefill_static: only the prefill path (Q4_K, Q5_K, Q8_0, Q4_0; Q6_K / IQ4_XS rows of a 16-byte "
                    "multiple, or of an even number of bytes with M a multiple of the 2, 4 or 8 rows that make one; "
                    "N >= %d, 16-byte aligned rows and activations) is available here",
                    wllm::kPrefillMinN);
    const size_t need = wllm::prefill_min_workspace_bytes(m);
    if (need > wllm::kPrefillStaticWorkspaceBytes)
        return fail(s, "wllm_mul_mat_prefill_static: N*K = %lld needs %llu workspace bytes, above the fixed %llu",
                    static_cast<long long>(N) * K, static_cast<unsigned long long>(need),
                    static_cast<unsigned long long>(wllm::kPrefillStaticWorkspaceBytes));
    const char* err = nullptr;
    void* ws = wllm::prefill_static_workspace(&err);
    if (!ws) return fail(s, "wllm_mul_mat_prefill_static: %s", err ? err : "no workspace");
    const int rc = wllm::launch_prefill(m, ws, wllm::kPrefillStaticWorkspaceBytes,
                                        stream ? static_cast<cudaStream_t>(stream) : s.stream);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "wllm_mul_mat_prefill_static launch");
    s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_dequantize(int32_t type, const void* src, float* dst, int64_t n, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!quant_type_supported(type)) return fail(s, "wllm_dequantize: unsupported type %d", type);
    if (!src || !dst || n <= 0 || n % wllm::block_elems(type) != 0)
        return fail(s, "wllm_dequantize: bad arguments");
    if (reinterpret_cast<uintptr_t>(src) % 2) return fail(s, "wllm_dequantize: src must be 2-byte aligned");
    const int rc = wllm::launch_dequantize(type, src, dst, n, stream ? static_cast<cudaStream_t>(stream) : s.stream);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "dequantize launch");
    s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_mul_mat_batch(const wllm_mulmat_args* ops, int32_t n_ops, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    MulMatOp m[wllm::kMaxOpsPerLaunch];
    if (const int32_t rc = ops_from_args(s, "wllm_mul_mat_batch", ops, n_ops, m)) return rc;
    return launch(s, m, n_ops, stream ? static_cast<cudaStream_t>(stream) : s.stream);
}

namespace {

// Byte range [first, end) of n vectors of len floats, stride floats apart.
struct ByteRange {
    uintptr_t first, end;
};
ByteRange vec_range(const void* p, int64_t stride, int32_t n, int64_t len) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(p);
    return {b, b + 4 * static_cast<uintptr_t>(stride * (n - 1) + len)};
}
bool overlap(ByteRange a, ByteRange b) { return a.first < b.end && b.first < a.end; }

// The fused entry points read their inputs (x, gain, up) in every CTA while
// other CTAs store outputs: no op's y may overlap any of them.
const char* fused_output_overlap(const wllm_mulmat_args* ops, int32_t n_ops, ByteRange extra) {
    for (int i = 0; i < n_ops; ++i) {
        const ByteRange y = vec_range(ops[i].y, ops[i].y_stride, ops[i].N, ops[i].M);
        if (extra.end > extra.first && overlap(y, extra)) return "an op's y overlaps the gain / up input";
        for (int j = 0; j < n_ops; ++j)
            if (overlap(y, vec_range(ops[j].x, ops[j].x_stride, ops[j].N, ops[j].K)))
                return "an op's y overlaps an op's x";
    }
    return nullptr;
}

}  // namespace

int32_t wllm_mul_mat_rms_norm_batch(const wllm_mulmat_args* ops, int32_t n_ops, const float* gain, float eps,
                                    void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    const char* what = "wllm_mul_mat_rms_norm_batch";
    MulMatOp m[wllm::kMaxOpsPerLaunch];
    if (const int32_t rc = ops_from_args(s, what, ops, n_ops, m)) return rc;
    if (!(eps >= 0.f) || eps > 1.f) return fail(s, "%s: eps must be in [0, 1]", what);
    if (gain && (reinterpret_cast<uintptr_t>(gain) & 15)) return fail(s, "%s: gain must be 16-byte aligned", what);
    for (int i = 1; i < n_ops; ++i)
        if (m[i].K != m[0].K) return fail(s, "%s: every op must have the same K (one gain vector)", what);
    if (const char* why = fused_output_overlap(ops, n_ops, gain ? vec_range(gain, 0, 1, m[0].K) : ByteRange{0, 0}))
        return fail(s, "%s: %s", what, why);
    // the fused form exists for the decode regime only: the caller runs the
    // RMS_NORM, MUL and MUL_MAT ops unfused otherwise
    if (!wllm::stream_supported(m, n_ops)) return WLLM_STATUS_NOT_IMPLEMENTED;
    const wllm::ProLaunch pl{wllm::kProNorm, gain, eps, nullptr, 0};
    const int rc = wllm::launch_stream(m, n_ops, stream ? static_cast<cudaStream_t>(stream) : s.stream, s.num_sms,
                                       nullptr, &pl);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "wllm_mul_mat_rms_norm_batch launch");
    s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_mul_mat_glu_batch(const wllm_mulmat_args* ops, int32_t n_ops, const float* up, int64_t up_stride,
                               int32_t glu, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    const char* what = "wllm_mul_mat_glu_batch";
    MulMatOp m[wllm::kMaxOpsPerLaunch];
    if (const int32_t rc = ops_from_args(s, what, ops, n_ops, m)) return rc;
    if (glu != WLLM_GLU_SWIGLU && glu != WLLM_GLU_GELU) return fail(s, "%s: unknown glu kind %d", what, glu);
    if (!up) return fail(s, "%s: null up", what);
    if ((reinterpret_cast<uintptr_t>(up) & 15) || (up_stride & 3))
        return fail(s, "%s: up must be 16-byte aligned and up_stride a multiple of 4", what);
    if (m[0].N > 1 && up_stride < m[0].K) return fail(s, "%s: up_stride below one vector (K floats)", what);
    const int64_t up_nb1 = 4 * up_stride;
    for (int i = 1; i < n_ops; ++i)
        if (m[i].x != m[0].x || m[i].x_nb1 != m[0].x_nb1 || m[i].K != m[0].K || m[i].N != m[0].N)
            return fail(s, "%s: every op must read the same activations (one up tensor)", what);
    if (const char* why = fused_output_overlap(ops, n_ops, vec_range(up, up_stride, m[0].N, m[0].K)))
        return fail(s, "%s: %s", what, why);
    // the fused form exists for the decode regime only: the caller runs the
    // GLU and MUL_MAT ops unfused otherwise
    if (!wllm::stream_supported(m, n_ops)) return WLLM_STATUS_NOT_IMPLEMENTED;
    const wllm::ProLaunch pl{glu == WLLM_GLU_SWIGLU ? wllm::kProSwiglu : wllm::kProGelu, nullptr, 0.f, up, up_nb1};
    const int rc = wllm::launch_stream(m, n_ops, stream ? static_cast<cudaStream_t>(stream) : s.stream, s.num_sms,
                                       nullptr, &pl);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "wllm_mul_mat_glu_batch launch");
    s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_ipc_alloc(uint64_t size, void** out_ptr, void* out_handle) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!out_ptr || !out_handle || size == 0) return fail(s, "wllm_ipc_alloc: null out or zero size");
    if (s.capturing) return fail(s, "wllm_ipc_alloc: not while recording a graph");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, size);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_ipc_alloc cudaMalloc");
    e = cudaMemset(p, 0, size);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(s, e, "wllm_ipc_alloc");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == WLLM_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(out_handle, &h, sizeof(h));
    s.ipc_owned.insert(p);
    *out_ptr = p;
    return WLLM_STATUS_OK;
}

int32_t wllm_ipc_open(const void* handle, void** out_ptr) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!handle || !out_ptr) return fail(s, "wllm_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(s, e, "wllm_ipc_open");
    s.ipc_opened.insert(p);
    *out_ptr = p;
    return WLLM_STATUS_OK;
}

int32_t wllm_ipc_close(void* ptr) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!s.ipc_opened.erase(ptr)) return fail(s, "wllm_ipc_close: %p was not opened here", ptr);
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? WLLM_STATUS_OK : cuda_fail(s, e, "wllm_ipc_close");
}

int32_t wllm_ipc_free(void* ptr) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!s.ipc_owned.erase(ptr)) return fail(s, "wllm_ipc_free: %p was not allocated here", ptr);
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? WLLM_STATUS_OK : cuda_fail(s, e, "wllm_ipc_free");
}

int32_t wllm_mul_mat_batch_tp(const wllm_mulmat_args* ops, const wllm_tp_outputs* outs, int32_t n_ops,
                              const wllm_tp_group* group, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    const char* what = "wllm_mul_mat_batch_tp";
    MulMatOp m[wllm::kMaxOpsPerLaunch];
    if (const int32_t rc = ops_from_args(s, what, ops, n_ops, m)) return rc;
    wllm::TpLaunch t;
    if (const int32_t rc = tp_from_group(s, what, group, &t)) return rc;
    if (!outs) return fail(s, "%s: null outputs", what);
    for (int i = 0; i < n_ops; ++i)
        for (int r = 0; r < t.world; ++r) {
            if (r != t.rank && !outs[i].y_rank[r]) return fail(s, "%s: op %d has no output on rank %d", what, i, r);
            t.y_peer[i][r] = r == t.rank ? nullptr : outs[i].y_rank[r];
        }
    if (!wllm::stream_supported(m, n_ops))
        return fail(s, "%s: only decode shapes (N <= 2, K %% 256 == 0, 16-byte aligned x) are row-sharded", what);
    const int rc = wllm::launch_stream(m, n_ops, stream ? static_cast<cudaStream_t>(stream) : s.stream, s.num_sms, &t);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "wllm_mul_mat_batch_tp launch");
    if (s.capturing) s.captured_kernels += static_cast<uint64_t>(rc);
    else s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_tp_wait(const wllm_tp_group* group, void* stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    wllm::TpLaunch t;
    if (const int32_t rc = tp_from_group(s, "wllm_tp_wait", group, &t)) return rc;
    const int rc = wllm::launch_tp_wait(t, stream ? static_cast<cudaStream_t>(stream) : s.stream);
    if (rc < 0) return cuda_fail(s, static_cast<cudaError_t>(-rc), "wllm_tp_wait launch");
    if (s.capturing) s.captured_kernels += static_cast<uint64_t>(rc);
    else s.counters.kernels_launched += static_cast<uint64_t>(rc);
    return WLLM_STATUS_OK;
}

int32_t wllm_get_stream(void** out_stream) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (!out_stream) return fail(s, "wllm_get_stream: null out");
    *out_stream = s.stream;
    return WLLM_STATUS_OK;
}

int32_t wllm_graph_begin(void) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s)) return WLLM_STATUS_FAILED;
    if (s.capturing) return fail(s, "wllm_graph_begin: already recording");
    const cudaError_t e = cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaStreamBeginCapture");
    s.capturing = true;
    s.captured_kernels = 0;
    return WLLM_STATUS_OK;
}

int32_t wllm_graph_end(int32_t* out_graph) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!s.capturing) return fail(s, "wllm_graph_end: not recording");
    s.capturing = false;
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(s.stream, &graph);
    if (e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return cuda_fail(s, e, "cudaStreamEndCapture");
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaGraphInstantiate");
    const int32_t id = s.next_graph++;
    s.graphs[id] = exec;
    s.graph_kernels[id] = s.captured_kernels;
    if (out_graph) *out_graph = id;
    return WLLM_STATUS_OK;
}

int32_t wllm_graph_launch(int32_t graph) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    if (!ensure_init(s) || !not_capturing(s, "wllm_graph_launch")) return WLLM_STATUS_FAILED;
    auto it = s.graphs.find(graph);
    if (it == s.graphs.end()) return fail(s, "wllm_graph_launch: unknown graph %d", graph);
    const cudaError_t e = cudaGraphLaunch(it->second, s.stream);
    if (e != cudaSuccess) return cuda_fail(s, e, "cudaGraphLaunch");
    s.counters.kernels_launched += s.graph_kernels[graph];
    return WLLM_STATUS_OK;
}

int32_t wllm_graph_destroy(int32_t graph) {
    State& s = S();
    std::lock_guard<std::mutex> g(s.mu);
    auto it = s.graphs.find(graph);
    if (it == s.graphs.end()) return WLLM_STATUS_OK;
    cudaGraphExecDestroy(it->second);
    s.graphs.erase(it);
    s.graph_kernels.erase(graph);
    return WLLM_STATUS_OK;
}

const char* wllm_version(void) { return "wllm_mulmat 0.1 (sm_100a)"; }

}  // extern "C"
