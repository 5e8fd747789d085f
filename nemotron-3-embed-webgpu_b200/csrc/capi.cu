// extern "C" entry points of include/nemo.h and include/nemo_ops.h.
#include <math.h>

#include "../../include/nemo.h"
#include "../../include/nemo_ops.h"
#include "runtime.h"

namespace nemo {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

int model_load(const void* data, size_t bytes, const int* devices, int ndev, nemo_model** out);
void model_destroy(nemo_model* m);
int pack_b200(const void* data, size_t bytes, void* out, size_t capacity, size_t* out_bytes);
int plan_create(nemo_model* m, uint32_t batch, uint32_t seq, uint32_t flags, nemo_plan** out);
void plan_destroy(nemo_plan* plan);
int plan_run(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
             float* out);
int plan_run_device(nemo_plan* plan, const uint32_t* d_ids, const uint32_t* d_lengths, float* d_out);
int plan_synchronize(nemo_plan* plan);
int plan_profile(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                 float* stage_ms);
int plan_run_debug(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                   float* out, uint16_t* x_dump, uint16_t* norm_dump, int* tokens_per_layer);
void rope_table_host(int sequence, float* table);
extern const char* kStageNames[12];

namespace {
int sync_and_check(cudaError_t launch) {
  if (launch != cudaSuccess) {
    set_error(std::string("kernel launch failed: ") + cudaGetErrorString(launch));
    return kErrCuda;
  }
  NEMO_CUDA_TRY(cudaDeviceSynchronize());
  return kOk;
}
}  // namespace

}  // namespace nemo

using namespace nemo;

extern "C" {

int nemo_model_load(const void* wgpack, size_t bytes, const int* devices, int ndev, nemo_model** out) {
  return model_load(wgpack, bytes, devices, ndev, out);
}

void nemo_model_destroy(nemo_model* model) { model_destroy(model); }

int nemo_pack_b200(const void* wgpack, size_t bytes, void* out, size_t capacity, size_t* out_bytes) {
  return pack_b200(wgpack, bytes, out, capacity, out_bytes);
}

int nemo_model_info_get(const nemo_model* m, nemo_model_info* info) {
  if (!m || !info) {
    set_error("nemo_model_info_get: null argument");
    return kErrArgs;
  }
  info->n_layers = m->n_layers;
  info->vocab = m->vocab;
  info->n_devices = (int)m->devs.size();
  info->compact_matrices = m->compact;
  info->kquant_matrices = m->kquant;
  info->packed_weight_bytes = m->packed_bytes;
  info->device_bytes = m->devs.empty() ? 0 : m->devs[0]->bytes;
  return kOk;
}

int nemo_plan_create(nemo_model* model, uint32_t batch, uint32_t sequence, nemo_plan** out) {
  return plan_create(model, batch, sequence, 0, out);
}

int nemo_plan_create_ex(nemo_model* model, uint32_t batch, uint32_t sequence, uint32_t flags, nemo_plan** out) {
  if (flags & ~(uint32_t)NEMO_PLAN_EXACT_ATTENTION) {
    nemo::set_error("nemo_plan_create_ex: unknown flags");
    return nemo::kErrArgs;
  }
  return plan_create(model, batch, sequence, flags, out);
}

int nemo_plan_run(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                  float* out) {
  return plan_run(plan, ids, n_ids, lengths, n_lengths, out);
}

int nemo_plan_run_device(nemo_plan* plan, const uint32_t* d_ids, const uint32_t* d_lengths, float* d_out) {
  return plan_run_device(plan, d_ids, d_lengths, d_out);
}

void* nemo_plan_stream(nemo_plan* plan) {
  return plan && !plan->devs.empty() ? (void*)plan->devs[0]->stream : nullptr;
}

int nemo_plan_synchronize(nemo_plan* plan) { return plan_synchronize(plan); }

int nemo_plan_single_launch(nemo_plan* plan) {
  if (!plan || plan->devs.empty()) {
    nemo::set_error("nemo_plan_single_launch: null plan");
    return nemo::kErrArgs;
  }
  for (const auto& d : plan->devs)
    if (!d->fgrid) return 0;
  return 1;
}

int nemo_plan_head_parallel(nemo_plan* plan) {
  if (!plan) {
    nemo::set_error("nemo_plan_head_parallel: null plan");
    return nemo::kErrArgs;
  }
  return plan->hp ? plan->hp_min : 0;
}

int nemo_plan_profile(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                      float* stage_ms) {
  return plan_profile(plan, ids, n_ids, lengths, n_lengths, stage_ms);
}

const char* nemo_stage_name(int stage) { return stage >= 0 && stage < NEMO_NUM_STAGES ? kStageNames[stage] : ""; }

int nemo_plan_run_debug(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                        float* out, uint16_t* x_dump, uint16_t* norm_dump, int* tokens_per_layer) {
  return plan_run_debug(plan, ids, n_ids, lengths, n_lengths, out, x_dump, norm_dump, tokens_per_layer);
}

void nemo_plan_destroy(nemo_plan* plan) { plan_destroy(plan); }

uint32_t nemo_merged_length(uint32_t sequence) {
  const double v = ceil((double)sequence * 0.64);
  return v < 1.0 ? 1u : (uint32_t)v;
}

const char* nemo_last_error(void) { return last_error(); }

// --- kernel-level entry points ------------------------------------------------

int nemo_op_decode(int fmt, const void* d_src, int rows, int k, void* d_out16, void* d_out32) {
  if (!d_src || !d_out16 || rows < 1 || k < 32 || k % 32 || fmt < 0 || fmt > 3 || (fmt <= 1 && k % 256)) {
    set_error("nemo_op_decode: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_decode(fmt, (const uint8_t*)d_src, rows, k, (__half*)d_out16, (float*)d_out32, 0));
}

size_t nemo_op_meta_bytes(void) { return sizeof(Meta); }

int nemo_op_meta(const void* d_lengths, int batch, int sequence, void* d_meta) {
  if (!d_lengths || !d_meta || batch < 1 || batch > kMaxBatch || sequence < 1) {
    set_error("nemo_op_meta: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_meta((const uint32_t*)d_lengths, batch, sequence, nullptr, (Meta*)d_meta, 0));
}

void* nemo_op_meta_tokens(void* d_meta, int merged) {
  Meta* m = (Meta*)d_meta;
  return merged ? (void*)&m->t1 : (void*)&m->t0;
}

int nemo_op_embedding(const void* d_ids, const void* d_table, int vocab, const void* d_meta, int max_tokens,
                      void* d_x) {
  if (!d_ids || !d_table || !d_meta || !d_x || vocab < 1 || max_tokens < 1) {
    set_error("nemo_op_embedding: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_embedding((const uint32_t*)d_ids, (const uint8_t*)d_table, vocab, (const Meta*)d_meta,
                                         max_tokens, (__half*)d_x, 0));
}

int nemo_op_rmsnorm(void* d_x, const void* d_residual, const void* d_w, void* d_norm, const void* d_rows,
                    int max_rows) {
  if (!d_x || !d_w || !d_norm || !d_rows || max_rows < 1) {
    set_error("nemo_op_rmsnorm: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_residual_rmsnorm((__half*)d_x, (const __half*)d_residual, (const float*)d_w,
                                                (__half*)d_norm, (const int*)d_rows, max_rows, 0));
}

int nemo_rope_table(int sequence, float* out) {
  if (sequence < 1 || !out) {
    set_error("nemo_rope_table: bad arguments");
    return kErrArgs;
  }
  rope_table_host(sequence, out);
  return kOk;
}

int nemo_op_rope(const void* d_qkv, const void* d_table, const void* d_meta, int merged, int max_tokens, void* d_q,
                 void* d_k) {
  if (!d_qkv || !d_table || !d_meta || !d_q || !d_k || max_tokens < 1) {
    set_error("nemo_op_rope: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_rope((const __half*)d_qkv, (const float*)d_table, (const Meta*)d_meta, merged != 0,
                                    max_tokens, (__half*)d_q, (__half*)d_k, 0));
}

int nemo_op_attention(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta, int merged, int batch,
                      int max_len, void* d_out) {
  if (!d_q || !d_k || !d_qkv || !d_meta || !d_out || batch < 1 || batch > kMaxBatch || max_len < 1) {
    set_error("nemo_op_attention: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_attention((const __half*)d_q, (const __half*)d_k, (const __half*)d_qkv,
                                         (const Meta*)d_meta, merged != 0, batch, max_len, (__half*)d_out, 0));
}

int nemo_op_attention_tc(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta, int merged,
                         int batch, int max_len, int rows, void* d_out) {
  if (!d_q || !d_k || !d_qkv || !d_meta || !d_out || batch < 1 || batch > kMaxBatch || max_len < 1 || rows < 1) {
    set_error("nemo_op_attention_tc: bad arguments");
    return kErrArgs;
  }
  AttnMaps maps;
  const int rows_c = rows / kSampleStride + batch + 1;
  __half* kc = nullptr;
  __half* vc = nullptr;
  uint32_t* err = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&kc, (size_t)rows_c * kKVWidth * 2));
  NEMO_CUDA_TRY(cudaMalloc(&vc, (size_t)rows_c * kKVWidth * 2));
  NEMO_CUDA_TRY(cudaMalloc(&err, 4));
  NEMO_CUDA_TRY(cudaMemset(kc, 0, (size_t)rows_c * kKVWidth * 2));
  NEMO_CUDA_TRY(cudaMemset(vc, 0, (size_t)rows_c * kKVWidth * 2));
  NEMO_CUDA_TRY(cudaMemset(err, 0, 4));
  int rc = kOk;
  if (make_tmap_f16(&maps.q, d_q, kQWidth, rows, 64, 128) || make_tmap_f16(&maps.k, d_k, kKVWidth, rows, 64, 128) ||
      make_tmap_f16(&maps.v, d_qkv, kQKVWidth, rows, 64, 128) ||
      make_tmap_f16(&maps.kc, kc, kKVWidth, rows_c, 64, 128) || make_tmap_f16(&maps.vc, vc, kKVWidth, rows_c, 64, 128)) {
    rc = kErrCuda;
  } else {
    rc = sync_and_check(launch_gather_sampled((const __half*)d_k, (const __half*)d_qkv, (const Meta*)d_meta,
                                              merged != 0, rows_c, kc, vc, 0));
    if (!rc)
      rc = sync_and_check(
          launch_attention_tc(maps, (const Meta*)d_meta, merged != 0, batch, max_len, (__half*)d_out, err, 0));
  }
  uint32_t h = 0;
  cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
  cudaFree(kc);
  cudaFree(vc);
  cudaFree(err);
  if (rc) return rc;
  if (h) {
    set_error("tcgen05 attention: a bounded wait timed out");
    return kErrTimeout;
  }
  return kOk;
}

int nemo_op_swiglu(const void* d_gate_up, const void* d_rows, int max_rows, void* d_out) {
  if (!d_gate_up || !d_rows || !d_out || max_rows < 1) {
    set_error("nemo_op_swiglu: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_swiglu((const __half*)d_gate_up, (const int*)d_rows, max_rows, (__half*)d_out, 0));
}

int nemo_op_merge(const void* d_x, const void* d_norm, const void* d_meta, int max_out, void* d_xm, void* d_nm) {
  if (!d_x || !d_norm || !d_meta || !d_xm || !d_nm || max_out < 1) {
    set_error("nemo_op_merge: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_merge((const __half*)d_x, (const __half*)d_norm, (const Meta*)d_meta, max_out,
                                     (__half*)d_xm, (__half*)d_nm, 0));
}

int nemo_op_pool(const void* d_norm, const void* d_meta, int batch, void* d_out) {
  if (!d_norm || !d_meta || !d_out || batch < 1 || batch > kMaxBatch) {
    set_error("nemo_op_pool: bad arguments");
    return kErrArgs;
  }
  return sync_and_check(launch_mean_pool((const __half*)d_norm, (const Meta*)d_meta, batch, (float*)d_out, 0));
}

int nemo_op_gemm(int impl, const void* d_x, const void* d_w, void* d_y, const void* d_rows, int max_rows, int n, int k,
                 int bn) {
  if (!d_x || !d_w || !d_y || !d_rows || max_rows < 1 || n < 64 || n % 64 || k < 64 || k % 64) {
    set_error("nemo_op_gemm: bad arguments");
    return kErrArgs;
  }
  if (impl == 0) {
    return sync_and_check(
        launch_gemm_simt((const __half*)d_x, (const __half*)d_w, (__half*)d_y, nullptr, (const int*)d_rows, max_rows,
                         n, k, 0));
  }
  if (bn != 64 && bn != 128 && bn != 256) {
    set_error("nemo_op_gemm: bn must be 64, 128 or 256");
    return kErrArgs;
  }
  if (n % bn) {
    set_error("nemo_op_gemm: n must be a multiple of bn");
    return kErrArgs;
  }
  const int rows_pad = (max_rows + kGemmTileM - 1) / kGemmTileM * kGemmTileM;
  CUtensorMap ma, mb;
  if (int rc = make_tmap_f16(&ma, d_x, (uint64_t)k, (uint64_t)rows_pad, 64, kGemmTileM)) return rc;
  if (int rc = make_tmap_f16(&mb, d_w, (uint64_t)k, (uint64_t)n, 64, bn)) return rc;
  uint32_t* err = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&err, 4));
  NEMO_CUDA_TRY(cudaMemset(err, 0, 4));
  int rc = sync_and_check(launch_gemm_tc(&ma, &mb, (__half*)d_y, n, (const int*)d_rows, max_rows, n, k, bn, err, 0));
  uint32_t h = 0;
  cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
  cudaFree(err);
  if (rc) return rc;
  if (h) {
    set_error("tcgen05 GEMM: a bounded wait timed out");
    return kErrTimeout;
  }
  return kOk;
}

size_t nemo_op_qmatmul_image_bytes(int fmt, int n, int k) { return qmatmul_image_bytes(fmt, n, k); }

int nemo_op_qmatmul_image(int fmt, const void* d_packed, int n, int k, void* d_image) {
  if (!d_packed || !d_image || !qmatmul_image_bytes(fmt, n, k) || ((uintptr_t)d_image & 255) ||
      ((uintptr_t)d_packed & 15)) {
    set_error("nemo_op_qmatmul_image: bad arguments (n a multiple of 128, K divisible by 256, aligned buffers)");
    return kErrArgs;
  }
  return sync_and_check(launch_qmatmul_retile(fmt, (const uint8_t*)d_packed, n, k, (uint8_t*)d_image, 0));
}

int nemo_op_qmatmul_image_decode(int fmt, const void* d_image, int n, int k, void* d_w16) {
  if (!d_image || !d_w16 || !qmatmul_image_bytes(fmt, n, k) || ((uintptr_t)d_image & 255) || ((uintptr_t)d_w16 & 15)) {
    set_error("nemo_op_qmatmul_image_decode: bad arguments (n a multiple of 128, K divisible by 256, aligned buffers)");
    return kErrArgs;
  }
  return sync_and_check(launch_qmatmul_image_decode(fmt, (const uint8_t*)d_image, n, k, (__half*)d_w16, 0));
}

int nemo_op_qmatmul_enqueue(int fmt, const void* d_image, const void* d_x, int m, int n, int k, void* d_y, void* d_err,
                            void* stream) {
  if (!d_image || !d_x || !d_y || !d_err || m < 1 || ((uintptr_t)d_image & 255) || ((uintptr_t)d_x & 15) ||
      ((uintptr_t)d_y & 15)) {
    set_error("nemo_op_qmatmul_enqueue: bad arguments");
    return kErrArgs;
  }
  return qmatmul_enqueue(fmt, (const uint8_t*)d_image, (const __half*)d_x, m, n, k, (float*)d_y, (uint32_t*)d_err,
                         (cudaStream_t)stream);
}

int nemo_op_qmatmul(int fmt, const void* d_packed, const void* d_x, int m, int n, int k, void* d_y) {
  if (!d_packed || !d_x || !d_y || m < 1) {
    set_error("nemo_op_qmatmul: bad arguments");
    return kErrArgs;
  }
  const size_t bytes = qmatmul_image_bytes(fmt, n, k);
  if (!bytes) {
    set_error("quantized matmul K must be divisible by 256 and n by 128");
    return kErrArgs;
  }
  uint8_t* image = nullptr;
  uint32_t* err = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&image, bytes));
  if (cudaMalloc(&err, 4) != cudaSuccess || cudaMemset(err, 0, 4) != cudaSuccess) {
    cudaFree(image);
    cudaFree(err);
    set_error("nemo_op_qmatmul: device allocation failed");
    return kErrCuda;
  }
  int rc = nemo_op_qmatmul_image(fmt, d_packed, n, k, image);
  if (!rc) rc = nemo_op_qmatmul_enqueue(fmt, image, d_x, m, n, k, d_y, err, nullptr);
  if (!rc) rc = sync_and_check(cudaGetLastError());
  uint32_t h = 0;
  if (!rc && cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) rc = kErrCuda;
  cudaFree(image);
  cudaFree(err);
  if (rc) return rc;
  if (h) {
    set_error("quantized matmul: a bounded wait timed out");
    return kErrTimeout;
  }
  return kOk;
}

}  // extern "C"
