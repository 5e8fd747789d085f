/*
 * nemo.h -- C ABI of the B200 Nemotron-3-Embed-1B encoder library
 * (libnemo_b200.so). This is the boundary a host binding (the N-API addon for
 * the reference's TypeScript engine, or ctypes) calls; no CUDA or torch types
 * appear in the signatures.
 *
 * Threading: a model is immutable after load and may be shared by many plans;
 * distinct plans may run concurrently from different threads; one plan must
 * not be run from two threads at once (the reference's engine never does).
 * Errors: every int-returning call returns NEMO_OK (0) or a negative
 * nemo_status; nemo_last_error() then describes the failure (thread-local).
 */
#ifndef NEMO_H
#define NEMO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEMO_HIDDEN 2048       /* embedding width, src/webgpu/model.ts:19 */
#define NEMO_MAX_BATCH 16      /* src/webgpu/embedding-engine.ts:37 */
#define NEMO_MAX_SEQUENCE 32768
#define NEMO_NUM_STAGES 12

typedef enum {
  NEMO_OK = 0,
  NEMO_ERR_ARGS = -1,    /* bad argument (shape, length, id range, null pointer) */
  NEMO_ERR_FORMAT = -2,  /* malformed or unsupported .wgpack */
  NEMO_ERR_CUDA = -3,    /* CUDA runtime / driver failure */
  NEMO_ERR_NCCL = -4,    /* collective failure */
  NEMO_ERR_TIMEOUT = -5, /* a bounded device-side wait gave up */
  NEMO_ERR_STATE = -6    /* object used in a state that does not allow the call */
} nemo_status;

typedef struct nemo_model nemo_model;
typedef struct nemo_plan nemo_plan;

typedef struct {
  int n_layers;           /* 16 for Nemotron-3-Embed-1B */
  int vocab;              /* token_embd rows */
  int n_devices;          /* devices holding a replica */
  int compact_matrices;   /* projections stored q4_0-tile32-compact */
  int kquant_matrices;    /* projection parts stored as raw Q4_K / Q6_K / Q4_0 */
  uint64_t packed_weight_bytes;  /* quantised projection bytes (one replica) */
  uint64_t device_bytes;         /* device memory held per replica */
} nemo_model_info;

/* Loads a .wgpack image and uploads one replica per listed CUDA device.
 * Replaces `new NemotronWebGPUModel(device, parsePrepackedModel(buffer))`
 * (src/webgpu/model.ts:253-305; src/prepacked/format.ts:146-169). Projections
 * may be q4_0-tile32-compact fused tensors (attn_qkv, attn_output,
 * ffn_gate_up, ffn_down) or raw GGML Q4_K / Q6_K / Q4_0 parts (attn_q/k/v,
 * attn_output, ffn_gate/up/down); they are decoded once to their effective
 * f16 values on each device. devices == NULL or ndev == 0 selects device 0. */
int nemo_model_load(const void* wgpack, size_t bytes, const int* devices, int ndev, nemo_model** out);

/* Rewrites a .wgpack as a B200-tiled pack: token table and norms unchanged,
 * every projection stored as the tile-slab image the device kernels stream,
 * in one raw tensor blk.<l>.<fused name>.b200_tiles ([tile table][128-row x
 * 256-column chunks]). nemo_model_load then uploads the images as they are
 * instead of re-tiling the pack. Replaces the offline producer
 * scripts/prepack-model.ts:28-57 for this build; the container stays WGPACK02
 * (src/prepacked/format.ts:105-144, raw storage) with metadata
 * "nemo.layout": "b200-tile-slab-v1". Host only (no GPU). With out == NULL
 * only *out_bytes (the size needed) is set; otherwise capacity must be at
 * least that size. */
int nemo_pack_b200(const void* wgpack, size_t bytes, void* out, size_t capacity, size_t* out_bytes);

/* Frees every replica. Plans of the model must be destroyed first. */
void nemo_model_destroy(nemo_model* model);

int nemo_model_info_get(const nemo_model* model, nemo_model_info* info);

/* Builds an execution plan for micro-batches of up to `batch` requests of up
 * to `sequence` tokens (buffers, RoPE table, one CUDA graph per device).
 * Replaces NemotronWebGPUModel.createPlan (src/webgpu/model.ts:328,73-139) and
 * EmbeddingRuntime.createPlan (src/webgpu/embedding-engine.ts:11-14).
 * batch in [1, 16], sequence in [1, NEMO_MAX_SEQUENCE]. */
int nemo_plan_create(nemo_model* model, uint32_t batch, uint32_t sequence, nemo_plan** out);

/* Plan flags for nemo_plan_create_ex. */
#define NEMO_PLAN_EXACT_ATTENTION 1u /* no layer-4 token merge, no stride-3 key sampling */

/* nemo_plan_create with flags (0 = the reference's semantics). With
 * NEMO_PLAN_EXACT_ATTENTION every layer keeps all valid tokens and attends over
 * every valid key: the reference's two approximations (model.ts:157 merge,
 * ops.ts:258-269 sampling) are off. No reference counterpart; single-request
 * runs on several devices stay on one device in this mode. */
int nemo_plan_create_ex(nemo_model* model, uint32_t batch, uint32_t sequence, uint32_t flags, nemo_plan** out);

/* Runs one micro-batch and blocks until the embeddings are in `out`.
 * Replaces NemotronExecutionPlan.run (src/webgpu/model.ts:146-176) /
 * EmbeddingPlan.run (src/webgpu/embedding-engine.ts:7-9).
 * ids: n_ids == batch * sequence token ids, row b padded after lengths[b];
 * lengths: n_lengths == batch values in [1, sequence] (BOS included);
 * out: batch * NEMO_HIDDEN floats, L2-normalised, caller-owned.
 * Errors: NEMO_ERR_ARGS with "token buffer does not match execution plan"
 * (model.ts:147) for a wrong n_ids; ids >= vocab and lengths outside
 * [1, sequence] are rejected as well. Requests are spread over the model's
 * devices when it has more than one. */
int nemo_plan_run(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths,
                  size_t n_lengths, float* out);

/* Same forward on inputs already resident on the plan's (first) device:
 * d_ids [batch*sequence] u32, d_lengths [batch] u32, d_out [batch*2048] f32,
 * all device pointers. Enqueued asynchronously on the plan's stream (see
 * nemo_plan_stream); the caller synchronises with nemo_plan_synchronize.
 * Inputs are not validated (lengths are clamped to [1, sequence], ids to the
 * vocabulary); single-device plans only. */
int nemo_plan_run_device(nemo_plan* plan, const uint32_t* d_ids, const uint32_t* d_lengths,
                         float* d_out);

/* cudaStream_t of the plan's first device, as void*. */
void* nemo_plan_stream(nemo_plan* plan);

/* 1 when every device of the plan runs the forward as one persistent launch
 * (plans whose batch x sequence is at most 16 tokens), 0 when it runs one
 * kernel per op, NEMO_ERR_ARGS for a null plan. Build-specific introspection;
 * the reference has no counterpart. */
int nemo_plan_single_launch(nemo_plan* plan);

/* For a plan of batch 1 on 2, 4 or 8 devices: the request length from which
 * nemo_plan_run runs the request head-parallel across the devices (token-
 * sharded projections; the QKV and attention epilogues store into the devices
 * owning each head group / token row over peer memory); 0 when the plan has
 * no head-parallel path (also when the devices lack peer access). Default 5000 tokens, NEMO_HEAD_PARALLEL_MIN at plan
 * creation overrides. Build-specific introspection; no reference counterpart. */
int nemo_plan_head_parallel(nemo_plan* plan);

/* Waits for the plan's streams; returns NEMO_ERR_TIMEOUT if a kernel reported
 * a bounded wait giving up. */
int nemo_plan_synchronize(nemo_plan* plan);

/* Per-stage device time of one forward, summed over layers like
 * NemotronExecutionPlan.profile (src/webgpu/model.ts:178-224). stage_ms has
 * NEMO_NUM_STAGES entries in the order of nemo_stage_name(). */
int nemo_plan_profile(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths,
                      size_t n_lengths, float* stage_ms);
const char* nemo_stage_name(int stage);

/* Parity hook: runs the forward eagerly and copies, after each layer l, the
 * residual stream and the normalised state (f16 bit patterns) of the valid
 * tokens, packed request-major, to x_dump + l*batch*sequence*2048 and
 * norm_dump + ... (either may be NULL); tokens_per_layer[l] receives the row
 * count. Single-device plans only. */
int nemo_plan_run_debug(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths,
                        size_t n_lengths, float* out, uint16_t* x_dump, uint16_t* norm_dump,
                        int* tokens_per_layer);

/* Frees the plan's buffers, graphs and streams. */
void nemo_plan_destroy(nemo_plan* plan);

/* Host tokenizer (no GPU): text -> token ids for nemo_plan_run, in place of
 * the browser tokenizer the reference loads with
 * AutoTokenizer.from_pretrained('nvidia/Nemotron-3-Embed-1B-BF16')
 * (src/main.ts:164-165) and calls as tokenizer(text).input_ids
 * (src/webgpu/embedding-engine.ts:41). nemo_tokenizer_load reads a Hugging
 * Face tokenizer.json of the byte-level BPE family: added tokens, no
 * normalizer, Split(regex) + ByteLevel or ByteLevel(use_regex) pre-tokenizer
 * (the Tekken and GPT-2 patterns), BPE merges, and a TemplateProcessing,
 * Bert/Roberta or ByteLevel post-processor; other components fail with
 * NEMO_ERR_FORMAT naming them. nemo_tokenizer_encode writes the ids of a
 * UTF-8 text (post-processor special tokens included) to ids (capacity
 * entries; ids == NULL only sets *n_ids). A tokenizer is immutable after load
 * and may be shared by threads. */
typedef struct nemo_tokenizer nemo_tokenizer;
int nemo_tokenizer_load(const void* tokenizer_json, size_t bytes, nemo_tokenizer** out);
int nemo_tokenizer_encode(const nemo_tokenizer* tokenizer, const char* text, size_t len, uint32_t* ids,
                          size_t capacity, size_t* n_ids);
void nemo_tokenizer_destroy(nemo_tokenizer* tokenizer);

/* contextualMergedLength (src/webgpu/model.ts:30-32). */
uint32_t nemo_merged_length(uint32_t sequence);

/* Description of the last failure on this thread ("" if none). */
const char* nemo_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* NEMO_H */
