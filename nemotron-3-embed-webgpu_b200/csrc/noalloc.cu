// nemo_op_attention_tc_noalloc: the tcgen05 attention entry point for callers
// that must not allocate device memory. Some hosts cannot call cudaMalloc on
// the path that runs attention: a process whose device memory is owned by
// another allocator (a framework's caching allocator, or a serving engine that
// reserves its whole budget at start-up) can see an extra cudaMalloc fail or
// fragment the pool, and cudaFree synchronises the whole device, stalling every
// other stream of a latency-bound server. This variant keeps its scratch (the
// compact K/V of the every-third-key layers and the kernel error word) in one
// fixed file-scope device array instead, so a call allocates nothing.
//
// Limits and sharing rules:
//   * the array holds kNoAllocCompactRows sampled key rows (K and V, 8 heads x
//     128 f16 each): 8 MiB + 256 B per GPU that loads this library, held until
//     the process exits;
//   * the call reads the run's metadata back to the host (a blocking copy of a
//     few hundred bytes, no allocation) to learn how many sampled rows it
//     needs; a call needing more than kNoAllocCompactRows is rejected with
//     NEMO_ERR_ARGS before any device work. Exact-attention metadata samples
//     no keys, so such calls need none and are never rejected;
//   * every call shares the one array and it keeps the last call's contents.
//     Each call clears the error word, writes its sampled rows, and zeroes the
//     rows after them up to the end of the last 128-row tile the attention
//     kernel loads: key weights there are 0, but a stale non-finite V value
//     from an earlier call would still turn 0 * Inf into NaN in the P.V
//     product. Two calls that overlap on the GPU (other threads or streams)
//     race on the array;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress with that device current) and caches it; make that
//     first call before any stream capture.
#include <algorithm>
#include <mutex>

#include "../../include/nemo_ops.h"
#include "kernels.cuh"

namespace nemo {
namespace {

constexpr int kNoAllocCompactRows = 2048;
constexpr size_t kNoAllocHalfRows = (size_t)kNoAllocCompactRows * kKVWidth;  // f16 elements per buffer
constexpr size_t kNoAllocBytes = 2 * kNoAllocHalfRows * sizeof(__half) + 256;

// K rows, then V rows, then the error word.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

struct ScratchSlot {
  uint8_t* base = nullptr;
};
ScratchSlot g_slots[64];
std::mutex g_slots_mu;

int scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  NEMO_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("nemo_op_attention_tc_noalloc: device index out of range");
    return kErrArgs;
  }
  std::lock_guard<std::mutex> lock(g_slots_mu);
  if (!g_slots[dev].base) {
    void* p = nullptr;
    NEMO_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_slots[dev].base = static_cast<uint8_t*>(p);
  }
  *out = g_slots[dev].base;
  return kOk;
}

}  // namespace
}  // namespace nemo

using namespace nemo;

extern "C" int nemo_op_attention_tc_noalloc(const void* d_q, const void* d_k, const void* d_qkv, const void* d_meta,
                                            int merged, int batch, int max_len, int rows, void* d_out) {
  if (!d_q || !d_k || !d_qkv || !d_meta || !d_out || batch < 1 || batch > kMaxBatch || max_len < 1 || rows < 1) {
    set_error("nemo_op_attention_tc_noalloc: bad arguments");
    return kErrArgs;
  }
  Meta hm;
  NEMO_CUDA_TRY(cudaMemcpy(&hm, d_meta, sizeof(Meta), cudaMemcpyDeviceToHost));
  const int nb = hm.batch < 0 ? 0 : hm.batch > kMaxBatch ? kMaxBatch : hm.batch;
  const long long need = hm.samp_off[merged ? 1 : 0][nb];
  if (need < 0 || need > kNoAllocCompactRows) {
    set_error("nemo_op_attention_tc_noalloc: " + std::to_string(need) +
              " sampled key rows needed, the fixed scratch holds " + std::to_string(kNoAllocCompactRows));
    return kErrArgs;
  }
  uint8_t* base = nullptr;
  if (int rc = scratch_for_current_device(&base)) return rc;
  __half* kc = reinterpret_cast<__half*>(base);
  __half* vc = kc + kNoAllocHalfRows;
  uint32_t* err = reinterpret_cast<uint32_t*>(base + 2 * kNoAllocHalfRows * sizeof(__half));
  AttnMaps maps;
  if (make_tmap_f16(&maps.q, d_q, kQWidth, rows, 64, 128) || make_tmap_f16(&maps.k, d_k, kKVWidth, rows, 64, 128) ||
      make_tmap_f16(&maps.v, d_qkv, kQKVWidth, rows, 64, 128) ||
      make_tmap_f16(&maps.kc, kc, kKVWidth, kNoAllocCompactRows, 64, 128) ||
      make_tmap_f16(&maps.vc, vc, kKVWidth, kNoAllocCompactRows, 64, 128))
    return kErrCuda;
  NEMO_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(uint32_t), 0));
  if (need > 0) {
    NEMO_CUDA_TRY(launch_gather_sampled((const __half*)d_k, (const __half*)d_qkv, (const Meta*)d_meta, merged != 0,
                                        (int)need, kc, vc, 0));
    // rows past the sampled ones that the last 128-row K/V tile still loads
    const long long tail = std::min<long long>((need + 127) / 128 * 128, kNoAllocCompactRows);
    if (tail > need) {
      const size_t off = (size_t)need * kKVWidth, len = (size_t)(tail - need) * kKVWidth * sizeof(__half);
      NEMO_CUDA_TRY(cudaMemsetAsync(kc + off, 0, len, 0));
      NEMO_CUDA_TRY(cudaMemsetAsync(vc + off, 0, len, 0));
    }
  }
  NEMO_CUDA_TRY(launch_attention_tc(maps, (const Meta*)d_meta, merged != 0, batch, max_len, (__half*)d_out, err, 0));
  uint32_t h = 0;
  NEMO_CUDA_TRY(cudaMemcpy(&h, err, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (h) {
    set_error("nemo_op_attention_tc_noalloc: a bounded wait timed out");
    return kErrTimeout;
  }
  return kOk;
}
