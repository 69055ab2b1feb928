/*
 * CPU oracle for the quantized MUL_MAT path (TEST INFRASTRUCTURE ONLY).
 *
 * This is a plain-C restatement of the reference's algorithm for
 * ggml MUL_MAT with a quantized src0 (Q4_K, Q5_K, Q6_K, Q4_0, Q8_0) and f32
 * src1/dst.
 * It is the checker for the CUDA path and the timed CPU baseline; it is
 * never linked into, loaded by or called from the product library.
 *
 * Sources restated (paths inside paulrobello/webllm):
 *   Q4_K block layout + dequant: src/inference/jsep/ops/matmul.ts:387-460
 *     (WGSL load_q4_K / q4k_unpack_scale_min), smoke-test/p2-v2-spike.src.ts:1037-1096
 *     (JS dequantQ4_KTile), tests/jsep-matmul-golden.test.ts:200-254 (packQ4_K);
 *     libllama's dequantize_row_q4_K reached via src/wasm/webgpu-bridge.cpp:702-708.
 *   Q6_K / Q8_0: no code in the reference repo; block sizes from
 *     src/models/gguf-parser.ts:282,288. The bit layout is ggml's published
 *     block_q6_K / block_q8_0 format (llama.cpp ggml-quants.c
 *     dequantize_row_q6_K / dequantize_row_q8_0, also restated by the gguf
 *     python package 0.19.0, gguf/quants.py:396-402,554-575).
 *   Q5_K / Q4_0 (fleet formats listed in docs/MODEL_SUPPORT.md:133-138): no
 *     code in the reference repo either; ggml's block_q5_K / block_q4_0
 *     (dequantize_row_q5_K / dequantize_row_q4_0), restated by gguf 0.19.0
 *     gguf/quants.py:241-251 (Q4_0) and :525-549 (Q5_K).
 *   MUL_MAT semantics dst[m + M*n] = sum_k W[m,k] * x[k + K*n]:
 *     tests/jsep-matmul-golden.test.ts:67-90 (cpuMatmul),
 *     smoke-test/p2-v2-spike.src.ts:1197-1214 (k-major f32 loop + f64 reference).
 */
#ifndef WLLM_ORACLE_QUANT_REF_H
#define WLLM_ORACLE_QUANT_REF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids (src/inference/ggml-wasm.ts:8-25). */
enum {
    ORACLE_TYPE_F32 = 0,
    ORACLE_TYPE_Q4_0 = 2,
    ORACLE_TYPE_Q8_0 = 8,
    ORACLE_TYPE_Q4_K = 12,
    ORACLE_TYPE_Q5_K = 13,
    ORACLE_TYPE_Q6_K = 14,
    ORACLE_TYPE_IQ4_XS = 23
};

/* Exact IEEE binary16 -> binary32 (normals, subnormals, inf, nan). */
float oracle_f16_to_f32(uint16_t h);

/* Elements per block and bytes per block; 0 for unknown types. */
int32_t oracle_block_elems(int32_t type);
int32_t oracle_block_bytes(int32_t type);

/* Dequantize k elements (k a multiple of the block size) of one row.
 * Return 0 on success, -1 on bad arguments (mirrors webgpu-bridge.cpp:702-708). */
int32_t oracle_dequantize_row(int32_t type, const void* src, float* dst, int64_t k);

/* MUL_MAT, f64 accumulation of exact f32 dequantized weights times f32 x.
 * w: M rows of row_bytes each; x: N vectors with stride x_stride floats;
 * out: out[m + M*n] (double). This is the parity reference r. */
int32_t oracle_mul_mat_f64(int32_t type, const void* w, int64_t row_bytes,
                           const float* x, int64_t x_stride,
                           double* out, int32_t M, int32_t K, int32_t N);

/* MUL_MAT, f32 dequant-then-dot with f32 accumulation (the reference's
 * refF32Loop, p2-v2-spike.src.ts:1197-1210, accumulates k-major in one f32
 * sum; here element k goes to partial sum k%16 so the loop vectorises).
 * out[m + out_stride*n]. Parallel over rows with OpenMP (threads);
 * this is the timed CPU baseline. */
int32_t oracle_mul_mat_f32(int32_t type, const void* w, int64_t row_bytes,
                           const float* x, int64_t x_stride,
                           float* out, int64_t out_stride,
                           int32_t M, int32_t K, int32_t N, int32_t threads);

/* Number of OpenMP threads the baseline would use by default. */
int32_t oracle_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
