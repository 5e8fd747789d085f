// Head-parallel forward of one long request across a plan's devices (the
// multi-GPU case for single requests of thousands of tokens; the reference
// runs them on one device, src/webgpu/model.ts:146-176).
//
// N devices (N in {2, 4, 8}, so the 8 KV heads and their GQA groups of 3 q
// heads split evenly) each own a contiguous token shard of ceil(S/N) tokens
// (the last one fewer) and run embedding, norms and all projections on it with
// the single-device kernels. Attention needs every token of a head, so around
// it two all-to-alls (grouped NCCL send/recv) switch layouts:
//   token-sharded [S/N x (Q|K|V) 5120]  ->  head-sharded [S x (Q|K|V)/N]
//   head-sharded  [S x 3072/N]           ->  token-sharded [S/N x 3072]
// RoPE (global positions), stride-3 key sampling and tcgen05 attention then
// run on the device's head group over the whole sequence. The layer-4 token
// merge and the final mean pool need whole rows: an all-gather of the shards
// (in place) gives every device the full sequence, each merges it and keeps
// its merged shard; the pool runs on device 0 over the gathered final rows, in
// the same order as on one device.
//
// NCCL is loaded at first use (dlopen), so the library does not depend on it
// unless this path runs. One host thread per device issues that device's
// kernels and its side of every collective (one NCCL group per exchange and
// device), so no device waits for the host to issue another device's work.
// The caller's thread then waits for every device with a host deadline; on a
// failure or a missed deadline it aborts the communicators (ncclCommAbort
// ends their kernels on every device), so nothing is left waiting on a peer,
// and the plan refuses further head-parallel runs.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>

#include "runtime.h"

namespace nemo {

namespace {

struct NcclApi {
  ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

const NcclApi* nccl_api() {
  static std::mutex mu;
  static NcclApi api;
  static int state = 0;  // 0 untried, 1 ok, -1 unavailable
  std::lock_guard<std::mutex> lock(mu);
  if (state == 0) {
    state = -1;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.CommInitAll = reinterpret_cast<decltype(api.CommInitAll)>(dlsym(h, "ncclCommInitAll"));
      api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
      api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
      api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(h, "ncclGroupStart"));
      api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
      api.Send = reinterpret_cast<decltype(api.Send)>(dlsym(h, "ncclSend"));
      api.Recv = reinterpret_cast<decltype(api.Recv)>(dlsym(h, "ncclRecv"));
      api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
      api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
      if (api.CommInitAll && api.CommDestroy && api.CommAbort && api.GroupStart && api.GroupEnd && api.Send && api.Recv &&
          api.AllGather && api.GetErrorString)
        state = 1;
    }
  }
  return state == 1 ? &api : nullptr;
}

#define HP_NCCL(expr)                                                                                 \
  do {                                                                                                \
    ncclResult_t _r = (expr);                                                                         \
    if (_r != ncclSuccess) {                                                                          \
      set_error(std::string("NCCL error: ") + nccl->GetErrorString(_r) + " (" #expr ")");           \
      return kErrNccl;                                                                                \
    }                                                                                                 \
  } while (0)

#define HP_LAUNCH(expr)                                                                               \
  do {                                                                                                \
    cudaError_t _e = (expr);                                                                          \
    if (_e != cudaSuccess) {                                                                          \
      set_error(std::string("kernel launch failed: ") + cudaGetErrorString(_e) + " (" #expr ")");     \
      return kErrCuda;                                                                                \
    }                                                                                                 \
  } while (0)

}  // namespace

// Column c of the N concatenated send blocks (block j = c / (5120 / N) holds
// the Q, K and V columns of head group j: q heads j*24/N.., kv heads j*8/N..)
// carries this column of the token's QKV row.
__host__ __device__ inline int hp_pack_source(int c, int N) {
  const int gw = kQKVWidth / N, nq = kQWidth / N, nk = kKVWidth / N;
  const int j = c / gw, w = c - j * gw;
  return w < nq ? j * nq + w : w < nq + nk ? kQWidth + j * nk + (w - nq) : kQWidth + kKVWidth + j * nk + (w - nq - nk);
}

namespace {

// Token-sharded QKV [T x 5120] -> N send blocks [T x 5120/N].
__global__ void __launch_bounds__(256) hp_pack_kernel(const __half* __restrict__ qkv, int T, int N, int stride_rows,
                                                      __half* __restrict__ send) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int kChunks = kQKVWidth / 8;
  const int t = (int)(idx / kChunks);
  if (t >= T) return;
  const int c = (int)(idx - (long long)t * kChunks) * 8;
  const int gw = kQKVWidth / N, j = c / gw, w = c - j * gw;
  *reinterpret_cast<uint4*>(send + ((size_t)j * stride_rows + t) * gw + w) =
      *reinterpret_cast<const uint4*>(qkv + (size_t)t * kQKVWidth + hp_pack_source(c, N));
}

// N received blocks [T x 3072/N] (block j: this shard's tokens, head group j)
// -> token-sharded attention output [T x 3072].
__global__ void __launch_bounds__(256) hp_unpack_kernel(const __half* __restrict__ back, int T, int N, int stride_rows,
                                                        __half* __restrict__ attn) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int kChunks = kQWidth / 8;
  const int t = (int)(idx / kChunks);
  if (t >= T) return;
  const int c = (int)(idx - (long long)t * kChunks) * 8;
  const int gq = kQWidth / N, j = c / gq, w = c - j * gq;
  *reinterpret_cast<uint4*>(attn + (size_t)t * kQWidth + c) =
      *reinterpret_cast<const uint4*>(back + ((size_t)j * stride_rows + t) * gq + w);
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

int pick_bn(int rows, int n) {
  const int mt = (rows + kGemmTileM - 1) / kGemmTileM;
  if ((long long)mt * (n / 256) >= 148) return 2;
  if ((long long)mt * (n / 128) >= 148) return 1;
  return 0;
}

}  // namespace

struct HeadParDevice {
  int device = 0;
  DevicePlan* dp = nullptr;  // stream, rope table and error word of the plan on this device
  ncclComm_t comm = nullptr;
  Meta *meta_loc = nullptr, *meta_full = nullptr;
  __half *x = nullptr, *norm = nullptr;       // [sh0 rows] token shard before the merge
  __half *qkv = nullptr, *attn = nullptr, *delta = nullptr, *gu = nullptr, *ffn = nullptr;  // [shard rows]
  __half *send = nullptr, *grp = nullptr;     // N x [sh0 x 5120/N]; [N*sh0 x 5120/N] head group, all tokens
  __half *qg = nullptr, *kg = nullptr, *kc = nullptr, *vc = nullptr, *attn_g = nullptr, *back = nullptr;
  __half *x_full = nullptr, *n_full = nullptr, *xm_full = nullptr, *nm_full = nullptr;
  float* out = nullptr;
  std::vector<void*> allocations;
};

struct HeadPar {
  int N = 0;
  int seq = 0;         // the plan's sequence: largest S
  int sh0_max = 0;     // ceil(seq / N)
  int sh1_max = 0;     // ceil(merged(seq) / N)
  int rows_c = 0;      // compact sampled rows
  bool aborted = false;  // communicators aborted after a failure: no further runs
  std::vector<HeadParDevice> d;
  // Per request length: run once eagerly (NCCL sets up its peer connections),
  // then captured as one CUDA graph per device and replayed; lengths whose
  // capture failed stay eager.
  std::set<int> warmed, eager_only;
  std::map<int, std::vector<cudaGraphExec_t>> graphs;
};

namespace {

template <typename T>
int hp_alloc(HeadParDevice& d, T** p, size_t bytes) {
  void* v = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&v, std::max<size_t>(bytes, 256)));
  NEMO_CUDA_TRY(cudaMemset(v, 0, std::max<size_t>(bytes, 256)));
  d.allocations.push_back(v);
  *p = reinterpret_cast<T*>(v);
  return kOk;
}

int merged_len(int s) { return std::max(1, (int)ceil(s * 0.64)); }

Meta make_meta(int len0, int len1, int seq) {
  Meta m = {};
  m.batch = 1;
  m.seq = seq;
  m.merged_seq = len1;
  m.t0 = len0;
  m.t1 = len1;
  m.src_len[0] = len0;
  m.tgt_len[0] = len1;
  m.src_off[1] = len0;
  m.tgt_off[1] = len1;
  m.samp_off[0][1] = len0 > kSampleThreshold ? (len0 + kSampleStride - 1) / kSampleStride : 0;
  m.samp_off[1][1] = len1 > kSampleThreshold ? (len1 + kSampleStride - 1) / kSampleStride : 0;
  return m;
}

}  // namespace

void hp_destroy(HeadPar* hp) {
  if (!hp) return;
  const NcclApi* nccl = nccl_api();
  // graphs holding NCCL kernels go before their communicators
  for (auto& kv : hp->graphs)
    for (size_t r = 0; r < kv.second.size(); ++r) {
      cudaSetDevice(hp->d[r].device);
      cudaStreamSynchronize(hp->d[r].dp->stream);
      if (kv.second[r]) cudaGraphExecDestroy(kv.second[r]);
    }
  hp->graphs.clear();
  for (auto& d : hp->d) {
    cudaSetDevice(d.device);
    if (d.dp) cudaStreamSynchronize(d.dp->stream);
    if (d.comm && nccl) nccl->CommDestroy(d.comm);
    for (void* v : d.allocations) cudaFree(v);
  }
  delete hp;
}

// Sets up head-parallel state for plans of batch 1 on 2, 4 or 8 devices.
int hp_create(nemo_plan* plan, HeadPar** out) {
  *out = nullptr;
  const int N = (int)plan->devs.size();
  if (plan->batch != 1 || (N != 2 && N != 4 && N != 8)) return kOk;
  const NcclApi* nccl = nccl_api();
  if (!nccl) {
    set_error("head-parallel attention needs NCCL (libnccl.so.2 could not be loaded)");
    return kErrNccl;
  }
  auto* hp = new HeadPar();
  hp->N = N;
  hp->seq = plan->seq;
  hp->sh0_max = (plan->seq + N - 1) / N;
  hp->sh1_max = (merged_len(plan->seq) + N - 1) / N;
  hp->rows_c = plan->seq / kSampleStride + 2;
  hp->d.resize(N);
  std::vector<int> devs(N);
  for (int r = 0; r < N; ++r) devs[r] = plan->devs[r]->device;
  std::vector<ncclComm_t> comms(N);
  auto fail = [&](int rc) {
    hp_destroy(hp);
    return rc;
  };
  {
    const ncclResult_t r = nccl->CommInitAll(comms.data(), N, devs.data());
    if (r != ncclSuccess) {
      set_error(std::string("NCCL error: ") + nccl->GetErrorString(r) + " (ncclCommInitAll)");
      delete hp;
      return kErrNccl;
    }
  }
  const int sh = round_up(hp->sh0_max, kGemmTileM);  // GEMM row tiles read whole 128-row blocks
  const int full = N * hp->sh0_max, fullp = round_up(full, kGemmTileM);
  const int mfull = N * hp->sh1_max;
  for (int r = 0; r < N; ++r) {
    HeadParDevice& d = hp->d[r];
    d.device = devs[r];
    d.dp = plan->devs[r].get();
    d.comm = comms[r];
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(kErrCuda);
    if (hp_alloc(d, &d.meta_loc, sizeof(Meta)) || hp_alloc(d, &d.meta_full, sizeof(Meta)) ||
        hp_alloc(d, &d.x, (size_t)sh * kHidden * 2) || hp_alloc(d, &d.norm, (size_t)sh * kHidden * 2) ||
        hp_alloc(d, &d.qkv, (size_t)sh * kQKVWidth * 2) || hp_alloc(d, &d.attn, (size_t)sh * kQWidth * 2) ||
        hp_alloc(d, &d.delta, (size_t)sh * kHidden * 2) || hp_alloc(d, &d.gu, (size_t)sh * 2 * kInter * 2) ||
        hp_alloc(d, &d.ffn, (size_t)sh * kInter * 2) ||
        hp_alloc(d, &d.send, (size_t)N * hp->sh0_max * (kQKVWidth / N) * 2) ||
        hp_alloc(d, &d.grp, (size_t)fullp * (kQKVWidth / N) * 2) ||
        hp_alloc(d, &d.qg, (size_t)fullp * (kQWidth / N) * 2) || hp_alloc(d, &d.kg, (size_t)fullp * (kKVWidth / N) * 2) ||
        hp_alloc(d, &d.kc, (size_t)round_up(hp->rows_c, 128) * (kKVWidth / N) * 2) ||
        hp_alloc(d, &d.vc, (size_t)round_up(hp->rows_c, 128) * (kKVWidth / N) * 2) ||
        hp_alloc(d, &d.attn_g, (size_t)fullp * (kQWidth / N) * 2) ||
        hp_alloc(d, &d.back, (size_t)N * hp->sh0_max * (kQWidth / N) * 2) ||
        hp_alloc(d, &d.x_full, (size_t)full * kHidden * 2) || hp_alloc(d, &d.n_full, (size_t)full * kHidden * 2) ||
        // + one tile: the post-merge A map of the last shard spans whole 128-row tiles
        hp_alloc(d, &d.xm_full, (size_t)(mfull + kGemmTileM) * kHidden * 2) ||
        hp_alloc(d, &d.nm_full, (size_t)(mfull + kGemmTileM) * kHidden * 2) ||
        hp_alloc(d, &d.out, (size_t)kHidden * 4))
      return fail(kErrCuda);
  }
  *out = hp;
  return kOk;
}

namespace {

struct RunMaps {
  CUtensorMap a_norm0, a_norm1, a_attn, a_ffn;
  AttnMaps g;
};

// Device r's whole share of one head-parallel forward, issued by its own host
// thread: kernels on the device's plan stream, and this device's side of every
// collective. `stop` is raised by a thread that failed; the others then issue
// no further collective (the caller aborts the communicators).
int hp_run_device(nemo_plan* plan, HeadPar* hp, int r, const RunMaps& m, int S0, std::atomic<bool>& stop) {
  const NcclApi* nccl = nccl_api();
  const int N = hp->N, L = plan->model->n_layers;
  const int S1 = merged_len(S0);
  const int sh0 = (S0 + N - 1) / N, sh1 = (S1 + N - 1) / N;
  const int gw = kQKVWidth / N, gq = kQWidth / N, gk = kKVWidth / N;
  const int nqh = kQHeads / N, nkh = kKVHeads / N;
  auto shard = [](int S, int sh, int i) { return std::max(0, std::min(sh, S - i * sh)); };
  HeadParDevice& d = hp->d[r];
  NEMO_CUDA_TRY(cudaSetDevice(d.device));
  DeviceModel& dm = *d.dp->dm;
  cudaStream_t s = d.dp->stream;
  auto halt = [&]() -> int {
    if (!stop.load()) return kOk;
    set_error("head-parallel run stopped: another device failed");
    return kErrNccl;
  };

  // ---- embedding + first norm on the shard ----
  HP_LAUNCH(launch_embedding(d.dp->ids, dm.embd, dm.vocab, d.meta_loc, sh0, d.x, s));
  HP_LAUNCH(launch_residual_rmsnorm(d.x, nullptr, dm.attn_norm[0], d.norm, &d.meta_loc->t0, sh0, s));

  for (int l = 0; l < L; ++l) {
    const bool merged = l >= kMergeAfterLayer;
    const int S = merged ? S1 : S0, sh = merged ? sh1 : sh0;
    if (l == kMergeAfterLayer) {
      // all-gather x and the normalised state, merge the whole sequence on
      // every device (ops.ts:629-661), keep the merged shard
      if (int rc = halt()) return rc;
      HP_NCCL(nccl->GroupStart());
      HP_NCCL(nccl->AllGather(d.x, d.x_full, (size_t)sh0 * kHidden, ncclHalf, d.comm, s));
      HP_NCCL(nccl->AllGather(d.norm, d.n_full, (size_t)sh0 * kHidden, ncclHalf, d.comm, s));
      HP_NCCL(nccl->GroupEnd());
      HP_LAUNCH(launch_merge(d.x_full, d.n_full, d.meta_full, S1, d.xm_full, d.nm_full, s));
    }
    __half* X = merged ? d.xm_full + (size_t)r * sh1 * kHidden : d.x;
    __half* Nrm = merged ? d.nm_full + (size_t)r * sh1 * kHidden : d.norm;
    const int* rows = merged ? &d.meta_loc->t1 : &d.meta_loc->t0;
    const int T = shard(S, sh, r);

    // QKV on the shard, packed per head group
    int bn = pick_bn(sh, kQKVWidth);
    HP_LAUNCH(launch_gemm_tc(merged ? &m.a_norm1 : &m.a_norm0, &dm.proj[l][kProjQKV].map[bn], d.qkv, kQKVWidth, rows,
                             sh, kQKVWidth, kHidden, kBnChoices[bn], d.dp->err, s));
    if (T > 0) {
      const long long threads = (long long)T * (kQKVWidth / 8);
      hp_pack_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(d.qkv, T, N, sh, d.send);
      HP_LAUNCH(cudaGetLastError());
    }
    // all-to-all: head group j of this shard -> device j; every shard's rows of
    // this device's head group <- their devices, in token order
    if (int rc = halt()) return rc;
    HP_NCCL(nccl->GroupStart());
    for (int j = 0; j < N; ++j) {
      if (T > 0) HP_NCCL(nccl->Send(d.send + (size_t)j * sh * gw, (size_t)T * gw, ncclHalf, j, d.comm, s));
      const int Tj = shard(S, sh, j);
      if (Tj > 0) HP_NCCL(nccl->Recv(d.grp + (size_t)j * sh * gw, (size_t)Tj * gw, ncclHalf, j, d.comm, s));
    }
    HP_NCCL(nccl->GroupEnd());
    // RoPE (global positions), sampled keys, attention on the head group
    HP_LAUNCH(launch_rope_group(d.grp, gw, nqh, nkh, d.dp->rope, d.meta_full, merged, S, d.qg, d.kg, s));
    if (S > kSampleThreshold)
      HP_LAUNCH(launch_gather_sampled_group(d.kg, d.grp, gw, gq + gk, gk, d.meta_full, merged, hp->rows_c, d.kc, d.vc,
                                            s));
    HP_LAUNCH(launch_attention_tc_group(m.g, d.meta_full, merged, 1, S, nqh, gq + gk, gq, d.attn_g, d.dp->err, s));
    // all-to-all back: this head group's rows of shard i -> device i
    if (int rc = halt()) return rc;
    HP_NCCL(nccl->GroupStart());
    for (int i = 0; i < N; ++i) {
      const int Ti = shard(S, sh, i);
      if (Ti > 0) HP_NCCL(nccl->Send(d.attn_g + (size_t)i * sh * gq, (size_t)Ti * gq, ncclHalf, i, d.comm, s));
      if (T > 0) HP_NCCL(nccl->Recv(d.back + (size_t)i * sh * gq, (size_t)T * gq, ncclHalf, i, d.comm, s));
    }
    HP_NCCL(nccl->GroupEnd());
    // O, norms, MLP on the shard
    if (T > 0) {
      const long long threads = (long long)T * (kQWidth / 8);
      hp_unpack_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(d.back, T, N, sh, d.attn);
      HP_LAUNCH(cudaGetLastError());
    }
    bn = pick_bn(sh, kHidden);
    HP_LAUNCH(launch_gemm_tc(&m.a_attn, &dm.proj[l][kProjO].map[bn], d.delta, kHidden, rows, sh, kHidden, kQWidth,
                             kBnChoices[bn], d.dp->err, s));
    HP_LAUNCH(launch_residual_rmsnorm(X, d.delta, dm.ffn_norm[l], Nrm, rows, sh, s));
    bn = pick_bn(sh, 2 * kInter);
    HP_LAUNCH(launch_gemm_tc(merged ? &m.a_norm1 : &m.a_norm0, &dm.proj[l][kProjGateUp].map[bn], d.gu, 2 * kInter,
                             rows, sh, 2 * kInter, kHidden, kBnChoices[bn], d.dp->err, s));
    HP_LAUNCH(launch_swiglu(d.gu, rows, sh, d.ffn, s));
    bn = pick_bn(sh, kHidden);
    HP_LAUNCH(launch_gemm_tc(&m.a_ffn, &dm.proj[l][kProjDown].map[bn], d.delta, kHidden, rows, sh, kHidden, kInter,
                             kBnChoices[bn], d.dp->err, s));
    const float* next = l + 1 < L ? dm.attn_norm[l + 1] : dm.output_norm;
    HP_LAUNCH(launch_residual_rmsnorm(X, d.delta, next, Nrm, rows, sh, s));
  }

  // ---- pool on device 0 over the gathered final rows (same order as one device) ----
  if (int rc = halt()) return rc;
  HP_NCCL(nccl->GroupStart());
  HP_NCCL(nccl->AllGather(d.nm_full + (size_t)r * sh1 * kHidden, d.nm_full, (size_t)sh1 * kHidden, ncclHalf, d.comm,
                          s));
  HP_NCCL(nccl->GroupEnd());
  if (r == 0) HP_LAUNCH(launch_mean_pool(d.nm_full, d.meta_full, 1, d.out, s));
  NEMO_CUDA_TRY(cudaMemcpyAsync(d.dp->h_err, d.dp->err, 4, cudaMemcpyDeviceToHost, s));
  return kOk;
}

// Waits for device d's stream with a host deadline (polling, no blocking sync).
int hp_wait(HeadParDevice& d, std::chrono::steady_clock::time_point deadline) {
  NEMO_CUDA_TRY(cudaSetDevice(d.device));
  for (uint32_t i = 0;; ++i) {
    const cudaError_t e = cudaStreamQuery(d.dp->stream);
    if (e == cudaSuccess) return kOk;
    if (e != cudaErrorNotReady) {
      set_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " on device " + std::to_string(d.device));
      return kErrCuda;
    }
    if ((i & 63u) == 63u) {
      if (std::chrono::steady_clock::now() > deadline) {
        set_error("head-parallel run: host deadline passed waiting for device " + std::to_string(d.device));
        return kErrTimeout;
      }
      std::this_thread::yield();
    }
  }
}

}  // namespace

// One request of `len` tokens (len <= plan sequence); out: 2048 floats.
int hp_run(nemo_plan* plan, HeadPar* hp, const uint32_t* ids, int len, float* out) {
  const NcclApi* nccl = nccl_api();
  if (!nccl) {
    set_error("NCCL unavailable");
    return kErrNccl;
  }
  if (hp->aborted) {
    set_error("head-parallel communicators were aborted after an earlier failure; create a new plan");
    return kErrState;
  }
  const int N = hp->N;
  const int S0 = len, S1 = merged_len(len);
  const int sh0 = (S0 + N - 1) / N, sh1 = (S1 + N - 1) / N;
  const int gw = kQKVWidth / N, gq = kQWidth / N, gk = kKVWidth / N;
  auto shard = [](int S, int sh, int r) { return std::max(0, std::min(sh, S - r * sh)); };

  // ---- per-run metadata, maps and inputs (host, before any device work) ----
  std::vector<RunMaps> maps(N);
  for (int r = 0; r < N; ++r) {
    HeadParDevice& d = hp->d[r];
    NEMO_CUDA_TRY(cudaSetDevice(d.device));
    const Meta ml = make_meta(shard(S0, sh0, r), shard(S1, sh1, r), sh0);
    const Meta mf = make_meta(S0, S1, S0);
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.meta_loc, &ml, sizeof(Meta), cudaMemcpyHostToDevice, d.dp->stream));
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.meta_full, &mf, sizeof(Meta), cudaMemcpyHostToDevice, d.dp->stream));
    const int T0 = shard(S0, sh0, r);
    // the plan's own ids buffer is reused as staging for this shard's ids
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.dp->ids, ids + (size_t)r * sh0, (size_t)std::max(T0, 1) * 4,
                                  cudaMemcpyHostToDevice, d.dp->stream));
    NEMO_CUDA_TRY(cudaMemsetAsync(d.dp->err, 0, 4, d.dp->stream));
    // the pageable host sources above are read before these calls return
    const int sh = round_up(hp->sh0_max, kGemmTileM);
    const int fullp = round_up(N * hp->sh0_max, kGemmTileM);
    RunMaps& m = maps[r];
    __half* nm_shard = d.nm_full + (size_t)r * sh1 * kHidden;
    if (make_tmap_f16(&m.a_norm0, d.norm, kHidden, sh, 64, kGemmTileM) ||
        make_tmap_f16(&m.a_norm1, nm_shard, kHidden, round_up(sh1, kGemmTileM), 64, kGemmTileM) ||
        make_tmap_f16(&m.a_attn, d.attn, kQWidth, sh, 64, kGemmTileM) ||
        make_tmap_f16(&m.a_ffn, d.ffn, kInter, sh, 64, kGemmTileM) ||
        make_tmap_f16(&m.g.q, d.qg, gq, fullp, 64, 128) || make_tmap_f16(&m.g.k, d.kg, gk, fullp, 64, 128) ||
        make_tmap_f16(&m.g.v, d.grp, gw, fullp, 64, 128) ||
        make_tmap_f16(&m.g.kc, d.kc, gk, round_up(hp->rows_c, 128), 64, 128) ||
        make_tmap_f16(&m.g.vc, d.vc, gk, round_up(hp->rows_c, 128), 64, 128))
      return kErrCuda;
  }
  // The post-merge map of shard r starts at row r*sh1 and spans
  // round_up(sh1, 128) rows: inside the xm/nm allocation (N*sh1_max + 128 rows).

  // ---- every device's work: replay this length's graphs, or issue it
  // concurrently with one thread per device (capturing it the second time) ----
  int rc = kOk;
  std::string msg;
  auto git = hp->graphs.find(len);
  if (git == hp->graphs.end()) {
    bool capture = hp->warmed.count(len) && !hp->eager_only.count(len);
    std::vector<cudaGraph_t> graphs(N, nullptr);
    std::vector<bool> captured(N, false);
    if (capture) {
      // Every device's stream enters capture before any thread issues work,
      // or none does: a device running its collectives for real while its
      // peers only record theirs would wait for them forever.
      int began = 0;
      for (; began < N; ++began) {
        HeadParDevice& d = hp->d[began];
        if (cudaSetDevice(d.device) != cudaSuccess ||
            cudaStreamBeginCapture(d.dp->stream, cudaStreamCaptureModeRelaxed) != cudaSuccess)
          break;
      }
      if (began < N) {
        for (int r = 0; r < began; ++r) {
          cudaGraph_t g = nullptr;
          cudaSetDevice(hp->d[r].device);
          cudaStreamEndCapture(hp->d[r].dp->stream, &g);
          if (g) cudaGraphDestroy(g);
        }
        cudaGetLastError();
        hp->eager_only.insert(len);
        capture = false;
      }
    }
    std::atomic<bool> stop(false);
    std::vector<int> rcs(N, kOk);
    std::vector<std::string> msgs(N);
    {
      std::vector<std::thread> threads;
      for (int r = 0; r < N; ++r)
        threads.emplace_back([&, r]() {
          rcs[r] = hp_run_device(plan, hp, r, maps[r], S0, stop);
          if (rcs[r]) {
            msgs[r] = last_error();
            stop.store(true);
          }
        });
      for (auto& t : threads) t.join();
    }
    if (capture)
      for (int r = 0; r < N; ++r) {
        cudaSetDevice(hp->d[r].device);
        captured[r] = cudaStreamEndCapture(hp->d[r].dp->stream, &graphs[r]) == cudaSuccess && graphs[r];
      }
    for (int r = 0; r < N; ++r)
      if (rcs[r] && !rc) {
        rc = rcs[r];
        msg = msgs[r];
      }
    if (capture) {
      // All devices' graphs or none: a partial set would leave collectives
      // without their peers. Nothing ran during the capture.
      bool all = !rc;
      std::vector<cudaGraphExec_t> execs(N, nullptr);
      for (int r = 0; r < N && all; ++r) {
        all = captured[r] && cudaSetDevice(hp->d[r].device) == cudaSuccess &&
              cudaGraphInstantiate(&execs[r], graphs[r], 0) == cudaSuccess;
      }
      for (int r = 0; r < N; ++r)
        if (graphs[r]) cudaGraphDestroy(graphs[r]);
      if (!all) {
        for (int r = 0; r < N; ++r)
          if (execs[r]) cudaGraphExecDestroy(execs[r]);
        hp->eager_only.insert(len);
        if (rc) {
          set_error(msg);
          return rc;
        }
        cudaGetLastError();  // clear a failed capture's error; run this length eagerly from now on
        return hp_run(plan, hp, ids, len, out);
      }
      git = hp->graphs.emplace(len, std::move(execs)).first;
    } else if (!rc) {
      hp->warmed.insert(len);
    }
  }
  if (!rc && git != hp->graphs.end()) {
    for (int r = 0; r < N && !rc; ++r) {
      HeadParDevice& d = hp->d[r];
      if (cudaSetDevice(d.device) != cudaSuccess || cudaGraphLaunch(git->second[r], d.dp->stream) != cudaSuccess) {
        rc = kErrCuda;
        msg = "head-parallel graph launch failed on device " + std::to_string(d.device);
      }
    }
  }
  // ---- wait for every device (host deadline), then the output ----
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(plan->host_deadline_ns);
  for (int r = 0; r < N && !rc; ++r)
    if (int e = hp_wait(hp->d[r], deadline)) {
      rc = e;
      msg = last_error();
    }
  if (rc) {
    // Collectives may be left without their peers: end them on every device.
    for (auto& d : hp->d)
      if (d.comm) {
        cudaSetDevice(d.device);
        nccl->CommAbort(d.comm);
        d.comm = nullptr;
      }
    hp->aborted = true;
    set_error(msg);
    return rc;
  }
  for (int r = 0; r < N; ++r)
    if (*hp->d[r].dp->h_err) {
      set_error("a device-side bounded wait timed out (error word " + std::to_string(*hp->d[r].dp->h_err) + ")");
      rc = kErrTimeout;
    }
  HeadParDevice& d0 = hp->d[0];
  NEMO_CUDA_TRY(cudaSetDevice(d0.device));
  NEMO_CUDA_TRY(cudaMemcpy(out, d0.out, kHidden * 4, cudaMemcpyDeviceToHost));
  return rc;
}

}  // namespace nemo

extern "C" int nemo_hp_pack_columns(int n_devices, int* columns) {
  if (!columns || (n_devices != 2 && n_devices != 4 && n_devices != 8)) {
    nemo::set_error("nemo_hp_pack_columns: n_devices must be 2, 4 or 8");
    return nemo::kErrArgs;
  }
  for (int c = 0; c < nemo::kQKVWidth; ++c) columns[c] = nemo::hp_pack_source(c, n_devices);
  return nemo::kOk;
}
