/*
 * CPU oracle for the Nemotron-3-Embed-1B encoder forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may use it.
 *
 * It restates, in plain C++:
 *   - the reference's CPU decode/encode code (src/gguf/quantization.ts,
 *     src/math/f16.ts) bit-exactly, with f64 arithmetic where the JS code uses
 *     JS numbers and f32 where it stores into a Float32Array;
 *   - the reference's tile32 packing (src/prepacked/format.ts:65-99);
 *   - the WGSL shader math of the forward pass (src/webgpu/ops.ts and
 *     src/webgpu/quant-matmul.ts, wired by src/webgpu/model.ts:73-176) in f32
 *     with f16 rounding (round-to-nearest-even, the shader's f16() cast) at the
 *     reference's storage points. Dot products accumulate in f32/f64 instead of
 *     the f16 accumulators of some reference pipelines.
 *
 * Parity of the quantisation and format code is pinned by the reference's own
 * known-answer tests (tests/quantization.test.ts, tests/prepacked-format.test.ts,
 * tests/model-config.test.ts). The forward pass has no golden vectors in the
 * reference; this restatement is its only pin.
 */
#ifndef NEMO_ORACLE_H
#define NEMO_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor types used by the path (src/gguf/types.ts:17-23). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_K = 12, ORC_Q6_K = 14 };

/* f16 helpers. */
double orc_half_to_float(uint16_t bits);   /* quantization.ts:2-9 */
uint16_t orc_float_to_half(double value);  /* f16.ts:4-25, half-up rounding */
uint16_t orc_f16_rne(float value);         /* WGSL f16() cast: round to nearest even */
float orc_f16_to_f32(uint16_t bits);

/* Block decoders: exact values stored as f32 (the JS Float32Array). */
void orc_dequant_q4k_block(const uint8_t* block, float* out256);  /* quantization.ts:19-38 */
void orc_dequant_q40_block(const uint8_t* block, float* out32);   /* quantization.ts:40-44 */
void orc_dequant_q6k_block(const uint8_t* block, float* out256);  /* quantization.ts:46-74 */

/* Offline encoders. */
void orc_quantize_q40_block(const float* values32, uint8_t* out18);  /* quantization.ts:77-98 */
int orc_requantize_to_q40(const uint8_t* src, size_t src_bytes, int type, int k, int n,
                          uint8_t* out);                              /* quantization.ts:101-131 */
/* packQ40Tile32: parts are row-major Q4_0 (18-byte blocks); out has
 * ceil(n/32) * (k/32) * 32 * 20 bytes, n = sum of part_rows. */
int orc_pack_q40_tile32(const uint8_t* const* parts, const int* part_rows, int nparts, int k,
                        uint8_t* out);                                /* format.ts:65-99 */

/* Exact f32 decode of a whole [n x k] matrix held in one storage format.
 * compact != 0 selects the q4_0-tile32-compact layout (format.ts:84-97, decoded
 * like quant-matmul.ts:99-108); otherwise GGUF row-major blocks. */
int orc_decode_matrix(const uint8_t* bytes, size_t nbytes, int type, int compact, int k, int n,
                      float* out);

/* contextualMergedLength, model.ts:30-32. */
uint32_t orc_merged_length(uint32_t sequence);

/* One row segment of a projection matrix. */
typedef struct {
  const uint8_t* data;
  size_t nbytes;
  int type;    /* ORC_Q4_0 / ORC_Q4_K / ORC_Q6_K */
  int compact; /* 1 = q4_0-tile32-compact */
  int k;
  int n;
} orc_part;

typedef struct {
  orc_part parts[3];
  int nparts;
} orc_proj;

typedef struct {
  int n_layers;                 /* 16 for the real model; >= 5 accepted */
  int vocab;
  const uint8_t* token_embd;    /* Q6_K, vocab rows x 8 blocks x 210 B */
  size_t token_embd_bytes;
  const float* attn_norm[16];
  const float* ffn_norm[16];
  const float* output_norm;
  orc_proj qkv[16];     /* n = 5120 (q 3072 | k 1024 | v 1024), k = 2048 */
  orc_proj o[16];       /* n = 2048, k = 3072 */
  orc_proj gate_up[16]; /* n = 12288 (gate 6144 | up 6144), k = 2048 */
  orc_proj down[16];    /* n = 2048, k = 6144 */
} orc_model_desc;

typedef struct orc_model orc_model;

/* Decodes every projection to its effective f16 values once (f16(decode)). */
orc_model* orc_model_create(const orc_model_desc* desc, char* err, size_t errlen);
void orc_model_destroy(orc_model* model);
/* Copies the effective f16 weights of one projection (n x k row-major). which:
 * 0 qkv, 1 o, 2 gate_up, 3 down. */
int orc_model_weights_f16(const orc_model* model, int layer, int which, uint16_t* out);

/*
 * Forward pass of NemotronExecutionPlan.run (model.ts:146-176) for one plan
 * (batch, sequence). ids: batch*sequence u32 (rows padded), lengths: batch.
 * out: batch*2048 f32 L2-normalised embeddings.
 *
 * Optional dumps (may be NULL): for each layer l, x_dump + l*stride and
 * norm_dump + l*stride receive the residual stream and the normalised state
 * (f16 bits) of the valid tokens after layer l, packed request-major; stride =
 * batch*sequence*2048 elements. tokens_per_layer[l] receives how many tokens
 * were written. Returns 0 on success, < 0 on bad arguments (err filled).
 */
int orc_forward(const orc_model* model, int batch, int sequence, const uint32_t* ids,
                const uint32_t* lengths, float* out, uint16_t* x_dump, uint16_t* norm_dump,
                int* tokens_per_layer, char* err, size_t errlen);
/* Same with exact != 0: no layer-4 token merge and no stride-3 key sampling
 * (every layer attends over every valid key of the request). Not a reference
 * mode: the oracle of the build's exact-attention plans. */
int orc_forward_ex(const orc_model* model, int batch, int sequence, const uint32_t* ids,
                   const uint32_t* lengths, int exact, float* out, uint16_t* x_dump, uint16_t* norm_dump,
                   int* tokens_per_layer, char* err, size_t errlen);

/* Individual stages on packed valid tokens, for kernel-level parity tests.
 * All f16 buffers hold bit patterns. */
void orc_embedding(const uint8_t* token_embd, int vocab, const uint32_t* ids, int tokens,
                   uint16_t* out);                                          /* ops.ts:680-725 */
void orc_residual_rmsnorm(uint16_t* x, const uint16_t* residual, const float* weight,
                          uint16_t* normalized, int rows, int width, float eps); /* ops.ts:21-72 */
void orc_matmul_f16(const uint16_t* x, const uint16_t* w, int m, int n, int k, float* out_f32,
                    uint16_t* out_f16);                                     /* quant-matmul.ts */
void orc_rope_table(int sequence, float* table);                             /* model.ts:95-107 */
void orc_rope(const uint16_t* qkv, const int* positions, int tokens, const float* table,
              uint16_t* q, uint16_t* k);                                     /* ops.ts:168-194 */
void orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, const int* offsets,
                   const uint32_t* lengths, int batch, uint16_t* out);
/* sample = 0: every key, whatever the length. */
void orc_attention_ex(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, const int* offsets,
                      const uint32_t* lengths, int batch, int sample, uint16_t* out);       /* ops.ts:213-362 */
void orc_swiglu(const uint16_t* gate_up, int rows, uint16_t* out);           /* ops.ts:74-89 */
void orc_token_merge(const uint16_t* in, const int* src_offsets, const uint32_t* src_lengths,
                     const int* dst_offsets, const uint32_t* dst_lengths, int batch,
                     uint16_t* out);                                         /* ops.ts:629-661 */
void orc_mean_pool(const uint16_t* in, const int* offsets, const uint32_t* lengths, int batch,
                   float* out);                                              /* ops.ts:596-616 */

/* Number of OpenMP threads the oracle uses (for reporting). */
int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
