/*
 * nemo_ops.h -- kernel-level C ABI of libnemo_b200.so.
 *
 * One entry point per device kernel of the forward pass, on caller-owned
 * device memory (plain device pointers as void*), so each kernel can be
 * checked on its own against the CPU oracle. These stand where the
 * reference's per-kernel `createRun` / `encode` pairs stand
 * (src/webgpu/ops.ts, src/webgpu/quant-matmul.ts): same inputs, same
 * outputs, packed valid-token rows instead of padded [batch x sequence] rows.
 * Every call launches on the legacy default stream and synchronises before it
 * returns; errors follow nemo.h.
 */
#ifndef NEMO_OPS_H
#define NEMO_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight block formats for nemo_op_decode. */
#define NEMO_FMT_Q4_K 0         /* GGUF row-major 144-byte blocks, quantization.ts:19-38 */
#define NEMO_FMT_Q6_K 1         /* GGUF row-major 210-byte blocks, quantization.ts:46-74 */
#define NEMO_FMT_Q4_0 2         /* GGUF row-major 18-byte blocks, quantization.ts:40-44 */
#define NEMO_FMT_Q4_0_TILE32 3  /* q4_0-tile32-compact, format.ts:65-99 / quant-matmul.ts:99-108 */

/* Decodes a [rows x k] quantised matrix: out16 receives f16(value) (the
 * effective weights of every reference matmul pipeline), out32 (optional)
 * the exact f32 value of the CPU decoders. */
int nemo_op_decode(int fmt, const void* d_src, int rows, int k, void* d_out16, void* d_out32);

/* Size in bytes of the per-run metadata block the ops below take. */
size_t nemo_op_meta_bytes(void);
/* Builds the metadata of a run from d_lengths [batch] (model.ts:226-233). */
int nemo_op_meta(const void* d_lengths, int batch, int sequence, void* d_meta);
/* Device ints inside the metadata block: valid tokens before / after the merge. */
void* nemo_op_meta_tokens(void* d_meta, int merged);

/* ops.ts:680-725: d_ids [batch*sequence] u32 padded rows, Q6_K table ->
 * d_x [tokens x 2048] f16 (packed valid tokens). */
int nemo_op_embedding(const void* d_ids, const void* d_table, int vocab, const void* d_meta,
                      int max_tokens, void* d_x);

/* ops.ts:21-72: x (+)= residual (stored f16), norm = f16(x*rsqrt(mean x^2+1e-5)*w).
 * d_residual may be NULL; *d_rows (device int) rows of width 2048. */
int nemo_op_rmsnorm(void* d_x, const void* d_residual, const void* d_w, void* d_norm,
                    const void* d_rows, int max_rows);

/* model.ts:95-107 on the host: the YaRN RoPE table [sequence x 64 x (cos,sin)] f32. */
int nemo_rope_table(int sequence, float* out);

/* ops.ts:168-194: d_qkv [tokens x 5120] -> d_q [tokens x 3072], d_k [tokens x 1024]. */
int nemo_op_rope(const void* d_qkv, const void* d_table, const void* d_meta, int merged,
                 int max_tokens, void* d_q, void* d_k);

/* ops.ts:213-362: bidirectional GQA attention with the >2048 stride-3 key
 * sampling; V read from d_qkv columns 4096..5119. d_out [tokens x 3072]. */
int nemo_op_attention(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta,
                      int merged, int batch, int max_len, void* d_out);

/* Same attention on the tcgen05 tensor cores (the kernel the plans run).
 * d_q, d_k, d_qkv hold `rows` token rows (rows >= the metadata's token count);
 * sampled layers (> 2048 valid keys) gather their keys into scratch buffers
 * this call allocates. */
int nemo_op_attention_tc(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta, int merged,
                         int batch, int max_len, int rows, void* d_out);

/* nemo_op_attention_tc without any device allocation. No counterpart in the
 * reference: it is for hosts that cannot call cudaMalloc/cudaFree where
 * attention runs (device memory owned by another allocator or reserved up
 * front; cudaFree would synchronise the whole device under a latency-bound
 * server). Its scratch is one fixed device array of 8 MiB + 256 B per GPU,
 * held until exit. The call reads d_meta back to learn how many sampled key
 * rows the run needs (requests longer than 2048 keep every third key; none in
 * exact-attention metadata) and fails with NEMO_ERR_ARGS when that exceeds
 * 2048. All calls share the array: calls that overlap on the GPU race. The
 * first call on a device looks up the array's address; make it before any
 * stream capture. Same arguments and results as nemo_op_attention_tc. */
int nemo_op_attention_tc_noalloc(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta, int merged,
                                 int batch, int max_len, int rows, void* d_out);

/* ops.ts:74-89: [rows x 12288] (gate | up) -> [rows x 6144]. */
int nemo_op_swiglu(const void* d_gate_up, const void* d_rows, int max_rows, void* d_out);

/* ops.ts:629-661 applied to x and normalized: -> d_xm, d_nm [merged tokens x 2048]. */
int nemo_op_merge(const void* d_x, const void* d_norm, const void* d_meta, int max_out, void* d_xm,
                  void* d_nm);

/* ops.ts:596-616: d_norm merged rows -> d_out [batch x 2048] f32, L2-normalised. */
int nemo_op_pool(const void* d_norm, const void* d_meta, int batch, void* d_out);

/* Projection GEMM Y[M x N] = X[M x K] . W[N x K]^T (f16 in, f32 accumulate,
 * f16 out; quant-matmul.ts:438-563 with f32 accumulation). impl 0 = CUDA-core
 * validation kernel, impl 1 = tcgen05 tensor-core kernel (bn = 64/128/256).
 * M = *d_rows <= max_rows; d_x has max_rows rounded up to 128 rows. */
int nemo_op_gemm(int impl, const void* d_x, const void* d_w, void* d_y, const void* d_rows,
                 int max_rows, int n, int k, int bn);

/* Standalone quantised matmul, the operation of the reference's
 * QuantMatmulKernel (src/webgpu/quant-matmul.ts:438-563: a GGUF Q4_K / Q6_K /
 * Q4_0 or q4_0-tile32-compact weight buffer, an [m x k] f16 activation buffer,
 * K divisible by 256, quant-matmul.ts:513), with f32 output:
 *   Y[m x n] = X[m x k] . W[n x k]^T, W = f16(decode(blocks)).
 * fmt is a NEMO_FMT_* value; n must be a multiple of 128.
 *
 * nemo_op_qmatmul_image_bytes / nemo_op_qmatmul_image re-tile the blocks on
 * the device into the tile-slab image the projection kernels stream (what
 * model load does for every projection); d_image is 256-byte aligned device
 * memory of that size. nemo_op_qmatmul_enqueue runs the matmul on an image
 * asynchronously on `stream` (a cudaStream_t, NULL = legacy default stream):
 * the fused-dequant split-K kernel for m <= 64, the dequant-fused batched GEMM
 * above. d_err is a zeroed 4-byte device word that becomes nonzero if a
 * bounded wait gave up. nemo_op_qmatmul does all of it on packed blocks and
 * synchronises (it allocates the image and error word and frees them). */
size_t nemo_op_qmatmul_image_bytes(int fmt, int n, int k);
int nemo_op_qmatmul_image(int fmt, const void* d_packed, int n, int k, void* d_image);
int nemo_op_qmatmul_enqueue(int fmt, const void* d_image, const void* d_x, int m, int n, int k, void* d_y,
                            void* d_err, void* stream);
int nemo_op_qmatmul(int fmt, const void* d_packed, const void* d_x, int m, int n, int k, void* d_y);

/* Decode of a tile-slab image by the per-row decoders every projection kernel
 * runs (the same launch model load uses to build the batched path's f16
 * weights): d_w16 = f16(decode(blocks)) as a row-major [n x k] f16 matrix,
 * 16-byte aligned. Replaces the reference's dequantisation for parity checks:
 * src/gguf/quantization.ts:19-74 rounded to f16 as quant-matmul.ts:106 does.
 * Synchronises. */
int nemo_op_qmatmul_image_decode(int fmt, const void* d_image, int n, int k, void* d_w16);

/* Routing of the head-parallel path (no reference counterpart; the index
 * functions its QKV GEMM and attention epilogues use, exported for layout
 * tests without a GPU), n_devices in {2, 4, 8}:
 * nemo_hp_qkv_route: for each QKV column c < 5120, the device that owns its
 *   head group, the buffer there (0 Q, 1 K, 2 V) and the column in it;
 * nemo_hp_row_owner: for positions 0..n_positions-1 of a request sharded in
 *   rows_per_device-row shards (the last one shorter), the owning device. */
int nemo_hp_qkv_route(int n_devices, int* device, int* buffer, int* column);
int nemo_hp_row_owner(int n_devices, int rows_per_device, int n_positions, int* device);

#ifdef __cplusplus
}
#endif
#endif /* NEMO_OPS_H */
