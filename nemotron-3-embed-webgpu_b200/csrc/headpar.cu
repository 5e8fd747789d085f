// Head-parallel forward of one long request across a plan's devices (the
// multi-GPU case for single requests of thousands of tokens; the reference
// runs them on one device, src/webgpu/model.ts:146-176).
//
// N devices (N in {2, 4, 8}, so the 8 KV heads and their GQA groups of 3 q
// heads split evenly) each own a contiguous token shard of ceil(S/N) tokens
// (the last one fewer) and run embedding, norms and all projections on it with
// the single-device kernels and epilogues. Attention needs every token of a
// head, so the layout switches twice per layer, and each switch is fused into
// the kernel that produces the data, over NVLink peer memory:
//   - the QKV GEMM's epilogue applies RoPE (global positions) and stores every
//     32-column chunk of a token row into the Q, K or V buffer of the device
//     owning that chunk's head group (hp_qkv_route), and the K/V of every third
//     position also into that device's compact sampled-key buffers;
//   - the attention kernel (one head group over the whole sequence) stores
//     each output row into the attention buffer of the device owning the
//     row's token shard, at the group's columns.
// No kernel waits for another device: the order between devices comes from
// CUDA events (all QKV epilogues before any attention, all attention stores
// before any O projection), which also orders every buffer's reuse one layer
// later. The layer-4 token merge and the final mean pool need whole rows: each
// device copies every shard's rows from its peers (copy engines, NVLink),
// merges the whole sequence and keeps its merged shard; the pool runs on
// device 0 over the gathered final rows, in the same order as on one device.
//
// One host thread issues every device's work. The first run of a request
// length is issued directly; the second is captured from device 0's stream
// (the other devices' streams join through events) into one multi-device CUDA
// graph that later runs of that length replay with a single launch. The caller
// waits with a host deadline; after a failure the plan refuses further
// head-parallel runs.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <map>
#include <set>
#include <string>
#include <thread>

#include "runtime.h"

namespace nemo {

namespace {

#define HP_LAUNCH(expr)                                                                               \
  do {                                                                                                \
    cudaError_t _e = (expr);                                                                          \
    if (_e != cudaSuccess) {                                                                          \
      set_error(std::string("head-parallel: ") + cudaGetErrorString(_e) + " (" #expr ")");             \
      return kErrCuda;                                                                                \
    }                                                                                                 \
  } while (0)

int round_up(int v, int m) { return (v + m - 1) / m * m; }

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

struct HeadParDevice {
  int device = 0;
  DevicePlan* dp = nullptr;  // stream, ids, rope table and error word of the plan on this device
  Meta *meta_loc = nullptr, *meta_full = nullptr;
  __half *x = nullptr, *norm = nullptr;                       // token shard before the merge
  __half *attn = nullptr, *ffn = nullptr, *delta = nullptr;  // token shard
  float* part = nullptr;                                     // K-split partial sums of O / down
  int* ksplit_used = nullptr;
  __half *qg = nullptr, *kg = nullptr, *vg = nullptr;  // this device's head group, every token
  __half *kc = nullptr, *vc = nullptr;                 // ... its sampled keys (every third position)
  __half *x_full = nullptr, *n_full = nullptr, *xm_full = nullptr, *nm_full = nullptr;
  float* out = nullptr;
  cudaEvent_t ev_in = nullptr, ev_qkv = nullptr, ev_attn = nullptr, ev_layer = nullptr, ev_join = nullptr;
  std::vector<void*> allocations;
};

struct HeadPar {
  int N = 0;
  int seq = 0;       // the plan's sequence: largest S
  int sh0_max = 0;   // ceil(seq / N)
  int sh1_max = 0;   // ceil(merged(seq) / N)
  int rows_c = 0;    // compact sampled rows
  int sh_rows = 0;   // allocated shard rows (whole 128-row GEMM tiles)
  bool failed = false;  // a run failed or missed its deadline: no further runs
  std::vector<HeadParDevice> d;
  // Per request length: issued directly once, then captured as one
  // multi-device graph and replayed; lengths whose capture failed stay direct.
  std::set<int> warmed, eager_only;
  std::map<int, cudaGraphExec_t> graphs;
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

// Bytes of K-split partial sums the O and down GEMMs can need for up to
// `rows` valid rows (the same split rule the kernel evaluates on the device).
size_t part_bytes(int rows, int sms) {
  size_t need = 0;
  for (int mt = 1; mt <= (rows + kGemmTileM - 1) / kGemmTileM; ++mt)
    for (const int kt : {kQWidth / 64, kInter / 64}) {
      const int sp = gemm_ksplit(mt, kHidden / 256, kt, sms);
      if (sp > 1) need = std::max(need, (size_t)sp * mt * kGemmTileM * kHidden * 4);
    }
  return need;
}

}  // namespace

void hp_destroy(HeadPar* hp) {
  if (!hp) return;
  if (!hp->d.empty()) {
    cudaSetDevice(hp->d[0].device);
    cudaStreamSynchronize(hp->d[0].dp->stream);
  }
  for (auto& kv : hp->graphs)
    if (kv.second) cudaGraphExecDestroy(kv.second);
  hp->graphs.clear();
  for (auto& d : hp->d) {
    cudaSetDevice(d.device);
    if (d.dp) cudaStreamSynchronize(d.dp->stream);
    for (cudaEvent_t e : {d.ev_in, d.ev_qkv, d.ev_attn, d.ev_layer, d.ev_join})
      if (e) cudaEventDestroy(e);
    for (void* v : d.allocations) cudaFree(v);
  }
  delete hp;
}

// Sets up head-parallel state for plans of batch 1 on 2, 4 or 8 devices with
// peer access between every pair (the epilogues store into peers' buffers).
// Without it the plan stays request-sharded (*out null).
int hp_create(nemo_plan* plan, HeadPar** out) {
  *out = nullptr;
  const int N = (int)plan->devs.size();
  if (plan->batch != 1 || (N != 2 && N != 4 && N != 8)) return kOk;
  for (int a = 0; a < N; ++a)
    for (int b = 0; b < N; ++b) {
      if (a == b) continue;
      int ok = 0;
      NEMO_CUDA_TRY(cudaDeviceCanAccessPeer(&ok, plan->devs[a]->device, plan->devs[b]->device));
      if (!ok) return kOk;
    }
  for (int a = 0; a < N; ++a) {
    NEMO_CUDA_TRY(cudaSetDevice(plan->devs[a]->device));
    for (int b = 0; b < N; ++b) {
      if (a == b) continue;
      const cudaError_t e = cudaDeviceEnablePeerAccess(plan->devs[b]->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        set_error(std::string("head-parallel: enabling peer access failed: ") + cudaGetErrorString(e));
        return kErrCuda;
      }
    }
  }
  auto* hp = new HeadPar();
  hp->N = N;
  hp->seq = plan->seq;
  hp->sh0_max = (plan->seq + N - 1) / N;
  hp->sh1_max = (merged_len(plan->seq) + N - 1) / N;
  hp->rows_c = plan->seq / kSampleStride + 2;
  hp->sh_rows = round_up(hp->sh0_max, kGemmTileM);  // GEMM row tiles read whole 128-row blocks
  hp->d.resize(N);
  auto fail = [&](int rc) {
    hp_destroy(hp);
    return rc;
  };
  const int sh = hp->sh_rows;
  const int full = N * hp->sh0_max, fullp = round_up(full, kGemmTileM);
  const int mfull = N * hp->sh1_max;
  const int gq = kQWidth / N, gk = kKVWidth / N;
  for (int r = 0; r < N; ++r) {
    HeadParDevice& d = hp->d[r];
    d.dp = plan->devs[r].get();
    d.device = d.dp->device;
    if (cudaSetDevice(d.device) != cudaSuccess) return fail(kErrCuda);
    for (cudaEvent_t* e : {&d.ev_in, &d.ev_qkv, &d.ev_attn, &d.ev_layer, &d.ev_join})
      if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return fail(kErrCuda);
    const size_t part = part_bytes(sh, d.dp->sms);
    if (hp_alloc(d, &d.meta_loc, sizeof(Meta)) || hp_alloc(d, &d.meta_full, sizeof(Meta)) ||
        hp_alloc(d, &d.x, (size_t)sh * kHidden * 2) || hp_alloc(d, &d.norm, (size_t)sh * kHidden * 2) ||
        hp_alloc(d, &d.attn, (size_t)sh * kQWidth * 2) || hp_alloc(d, &d.delta, (size_t)sh * kHidden * 2) ||
        hp_alloc(d, &d.ffn, (size_t)sh * kInter * 2) ||
        (part && (hp_alloc(d, &d.part, part) || hp_alloc(d, &d.ksplit_used, 2 * sizeof(int)))) ||
        hp_alloc(d, &d.qg, (size_t)fullp * gq * 2) || hp_alloc(d, &d.kg, (size_t)fullp * gk * 2) ||
        hp_alloc(d, &d.vg, (size_t)fullp * gk * 2) ||
        hp_alloc(d, &d.kc, (size_t)round_up(hp->rows_c, 128) * gk * 2) ||
        hp_alloc(d, &d.vc, (size_t)round_up(hp->rows_c, 128) * gk * 2) ||
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

// Every device's share of one head-parallel forward of S0 tokens, issued from
// this thread in phase order (all devices' QKV, then all attention, then all
// O / MLP), so each cudaStreamWaitEvent names the current phase's record.
// Starts and ends on device 0's stream: the other streams fork from it and
// join back into it (which is what lets the sequence be captured as one graph).
int hp_issue(nemo_plan* plan, HeadPar* hp, const std::vector<RunMaps>& m, int S0) {
  const int N = hp->N, L = plan->model->n_layers;
  const int S1 = merged_len(S0);
  const int sh0 = (S0 + N - 1) / N, sh1 = (S1 + N - 1) / N;
  const int gq = kQWidth / N, nqh = kQHeads / N;
  auto shard = [](int S, int sh, int i) { return std::max(0, std::min(sh, S - i * sh)); };
  auto on = [&](int r) -> cudaStream_t {
    cudaSetDevice(hp->d[r].device);
    return hp->d[r].dp->stream;
  };
  // stream r waits for event `ev` of every other device
  auto wait_all = [&](int r, cudaEvent_t HeadParDevice::*ev) -> int {
    cudaStream_t s = on(r);
    for (int j = 0; j < N; ++j)
      if (j != r) HP_LAUNCH(cudaStreamWaitEvent(s, hp->d[j].*ev, 0));
    return kOk;
  };

  HP_LAUNCH(cudaEventRecord(hp->d[0].ev_join, on(0)));  // fork
  for (int r = 1; r < N; ++r) HP_LAUNCH(cudaStreamWaitEvent(on(r), hp->d[0].ev_join, 0));

  for (int r = 0; r < N; ++r) {
    HeadParDevice& d = hp->d[r];
    cudaStream_t s = on(r);
    DeviceModel& dm = *d.dp->dm;
    HP_LAUNCH(launch_embedding(d.dp->ids, dm.embd, dm.vocab, d.meta_loc, sh0, d.x, s));
    HP_LAUNCH(launch_residual_rmsnorm(d.x, nullptr, dm.attn_norm[0], d.norm, &d.meta_loc->t0, sh0, s));
  }

  for (int l = 0; l < L; ++l) {
    const bool merged = l >= kMergeAfterLayer;
    const int S = merged ? S1 : S0, sh = merged ? sh1 : sh0;
    if (l == kMergeAfterLayer) {
      // every shard's x and normalised rows to every device, then the merge
      // of the whole sequence on each (ops.ts:629-661); each keeps its shard
      for (int r = 0; r < N; ++r) HP_LAUNCH(cudaEventRecord(hp->d[r].ev_layer, on(r)));
      for (int r = 0; r < N; ++r) {
        HeadParDevice& d = hp->d[r];
        if (int rc = wait_all(r, &HeadParDevice::ev_layer)) return rc;
        cudaStream_t s = on(r);
        for (int j = 0; j < N; ++j) {
          const size_t off = (size_t)j * sh0 * kHidden, bytes = (size_t)shard(S0, sh0, j) * kHidden * 2;
          if (!bytes) continue;
          HP_LAUNCH(cudaMemcpyPeerAsync(d.x_full + off, d.device, hp->d[j].x, hp->d[j].device, bytes, s));
          HP_LAUNCH(cudaMemcpyPeerAsync(d.n_full + off, d.device, hp->d[j].norm, hp->d[j].device, bytes, s));
        }
        HP_LAUNCH(launch_merge(d.x_full, d.n_full, d.meta_full, S1, d.xm_full, d.nm_full, s));
      }
    }

    // QKV on each shard: RoPE, then peer stores into the owners' head-group
    // buffers (and compact sampled K/V)
    for (int r = 0; r < N; ++r) {
      HeadParDevice& d = hp->d[r];
      cudaStream_t s = on(r);
      DeviceModel& dm = *d.dp->dm;
      GemmEpi ep;
      ep.mode = kSkinnyRope;
      ep.meta = d.meta_loc;
      ep.merged = merged ? 1 : 0;
      ep.rope = d.dp->rope;
      ep.hp.n_dev = N;
      ep.hp.row0 = r * sh;
      ep.hp.sample = S > kSampleThreshold ? 1 : 0;
      for (int j = 0; j < N; ++j) {
        ep.hp.q[j] = hp->d[j].qg;
        ep.hp.k[j] = hp->d[j].kg;
        ep.hp.v[j] = hp->d[j].vg;
        ep.hp.kc[j] = hp->d[j].kc;
        ep.hp.vc[j] = hp->d[j].vc;
      }
      const int bn = pick_bn(sh, kQKVWidth);
      HP_LAUNCH(launch_gemm_tc_epi(merged ? &m[r].a_norm1 : &m[r].a_norm0, &dm.proj[l][kProjQKV].map[bn], nullptr,
                                   kQKVWidth, merged ? &d.meta_loc->t1 : &d.meta_loc->t0, sh, kQKVWidth, kHidden,
                                   kBnChoices[bn], ep, d.dp->err, s));
      HP_LAUNCH(cudaEventRecord(d.ev_qkv, s));
    }
    // attention of each head group over the whole sequence; output rows to
    // the devices owning them
    for (int j = 0; j < N; ++j) {
      HeadParDevice& d = hp->d[j];
      if (int rc = wait_all(j, &HeadParDevice::ev_qkv)) return rc;
      cudaStream_t s = on(j);
      AttnScatter sc = {};
      for (int i = 0; i < N; ++i) sc.dst[i] = hp->d[i].attn;
      sc.n_dev = N;
      sc.rows_per_dev = sh;
      sc.col0 = j * gq;
      HP_LAUNCH(launch_attention_tc_group(m[j].g, d.meta_full, merged, 1, S, nqh, 0, gq, d.attn, d.dp->err, s, &sc));
      HP_LAUNCH(cudaEventRecord(d.ev_attn, s));
    }
    // O, norms, MLP on each shard
    for (int r = 0; r < N; ++r) {
      HeadParDevice& d = hp->d[r];
      if (int rc = wait_all(r, &HeadParDevice::ev_attn)) return rc;
      cudaStream_t s = on(r);
      DeviceModel& dm = *d.dp->dm;
      __half* X = merged ? d.xm_full + (size_t)r * sh1 * kHidden : d.x;
      __half* Nrm = merged ? d.nm_full + (size_t)r * sh1 * kHidden : d.norm;
      const int* rows = merged ? &d.meta_loc->t1 : &d.meta_loc->t0;
      GemmEpi eo;
      eo.part = d.part;
      eo.splits_out = d.part ? d.ksplit_used : nullptr;
      HP_LAUNCH(launch_gemm_tc_epi(&m[r].a_attn, &dm.proj[l][kProjO].map[2], d.delta, kHidden, rows, sh, kHidden,
                                   kQWidth, 256, eo, d.dp->err, s));
      if (d.part)
        HP_LAUNCH(launch_residual_rmsnorm_parts(X, d.delta, d.part, d.ksplit_used, dm.ffn_norm[l], Nrm, rows, sh, s));
      else
        HP_LAUNCH(launch_residual_rmsnorm(X, d.delta, dm.ffn_norm[l], Nrm, rows, sh, s));
      // SwiGLU in the gate/up epilogue (tensor map box bn/2, so bn >= 128)
      const int bi = std::max(1, pick_bn(sh, 2 * kInter));
      GemmEpi eg;
      eg.mode = kSkinnySwiglu;
      HP_LAUNCH(launch_gemm_tc_epi(merged ? &m[r].a_norm1 : &m[r].a_norm0, &dm.proj[l][kProjGateUp].map[bi - 1], d.ffn,
                                   kInter, rows, sh, 2 * kInter, kHidden, kBnChoices[bi], eg, d.dp->err, s));
      GemmEpi ed;
      ed.part = d.part;
      ed.splits_out = d.part ? d.ksplit_used + 1 : nullptr;
      HP_LAUNCH(launch_gemm_tc_epi(&m[r].a_ffn, &dm.proj[l][kProjDown].map[2], d.delta, kHidden, rows, sh, kHidden,
                                   kInter, 256, ed, d.dp->err, s));
      const float* next = l + 1 < L ? dm.attn_norm[l + 1] : dm.output_norm;
      if (d.part)
        HP_LAUNCH(launch_residual_rmsnorm_parts(X, d.delta, d.part, d.ksplit_used + 1, next, Nrm, rows, sh, s));
      else
        HP_LAUNCH(launch_residual_rmsnorm(X, d.delta, next, Nrm, rows, sh, s));
    }
  }

  // ---- pool on device 0 over every shard's final rows (same order as one device) ----
  for (int r = 1; r < N; ++r) HP_LAUNCH(cudaEventRecord(hp->d[r].ev_layer, on(r)));
  HeadParDevice& d0 = hp->d[0];
  if (int rc = wait_all(0, &HeadParDevice::ev_layer)) return rc;
  cudaStream_t s0 = on(0);
  for (int j = 1; j < N; ++j) {
    const size_t off = (size_t)j * sh1 * kHidden, bytes = (size_t)shard(S1, sh1, j) * kHidden * 2;
    if (bytes)
      HP_LAUNCH(cudaMemcpyPeerAsync(d0.nm_full + off, d0.device, hp->d[j].nm_full + off, hp->d[j].device, bytes, s0));
  }
  HP_LAUNCH(launch_mean_pool(d0.nm_full, d0.meta_full, 1, d0.out, s0));
  for (int r = 0; r < N; ++r) {
    cudaStream_t s = on(r);
    HP_LAUNCH(cudaMemcpyAsync(hp->d[r].dp->h_err, hp->d[r].dp->err, 4, cudaMemcpyDeviceToHost, s));
    if (r) HP_LAUNCH(cudaEventRecord(hp->d[r].ev_join, s));
  }
  if (int rc = wait_all(0, &HeadParDevice::ev_join)) return rc;  // join
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
  if (hp->failed) {
    set_error("an earlier head-parallel run failed on this plan; create a new plan");
    return kErrState;
  }
  const int N = hp->N;
  const int S0 = len, S1 = merged_len(len);
  const int sh0 = (S0 + N - 1) / N, sh1 = (S1 + N - 1) / N;
  const int gq = kQWidth / N, gk = kKVWidth / N;
  auto shard = [](int S, int sh, int r) { return std::max(0, std::min(sh, S - r * sh)); };
  const int fullp = round_up(N * hp->sh0_max, kGemmTileM);

  // ---- per-run metadata, maps and inputs (outside any graph) ----
  std::vector<RunMaps> maps(N);
  for (int r = 0; r < N; ++r) {
    HeadParDevice& d = hp->d[r];
    NEMO_CUDA_TRY(cudaSetDevice(d.device));
    const Meta ml = make_meta(shard(S0, sh0, r), shard(S1, sh1, r), sh0);
    const Meta mf = make_meta(S0, S1, S0);
    const int T0 = shard(S0, sh0, r);
    // pinned staging of the plan on this device: this shard's ids
    memcpy(d.dp->h_ids, ids + (size_t)r * sh0, (size_t)std::max(T0, 0) * 4);
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.meta_loc, &ml, sizeof(Meta), cudaMemcpyHostToDevice, d.dp->stream));
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.meta_full, &mf, sizeof(Meta), cudaMemcpyHostToDevice, d.dp->stream));
    NEMO_CUDA_TRY(cudaMemcpyAsync(d.dp->ids, d.dp->h_ids, (size_t)std::max(T0, 1) * 4, cudaMemcpyHostToDevice,
                                  d.dp->stream));
    NEMO_CUDA_TRY(cudaMemsetAsync(d.dp->err, 0, 4, d.dp->stream));
    NEMO_CUDA_TRY(cudaEventRecord(d.ev_in, d.dp->stream));
    RunMaps& m = maps[r];
    __half* nm_shard = d.nm_full + (size_t)r * sh1 * kHidden;
    if (make_tmap_f16(&m.a_norm0, d.norm, kHidden, hp->sh_rows, 64, kGemmTileM) ||
        make_tmap_f16(&m.a_norm1, nm_shard, kHidden, round_up(sh1, kGemmTileM), 64, kGemmTileM) ||
        make_tmap_f16(&m.a_attn, d.attn, kQWidth, hp->sh_rows, 64, kGemmTileM) ||
        make_tmap_f16(&m.a_ffn, d.ffn, kInter, hp->sh_rows, 64, kGemmTileM) ||
        make_tmap_f16(&m.g.q, d.qg, gq, fullp, 64, 128) || make_tmap_f16(&m.g.k, d.kg, gk, fullp, 64, 128) ||
        make_tmap_f16(&m.g.v, d.vg, gk, fullp, 64, 128) ||
        make_tmap_f16(&m.g.kc, d.kc, gk, round_up(hp->rows_c, 128), 64, 128) ||
        make_tmap_f16(&m.g.vc, d.vc, gk, round_up(hp->rows_c, 128), 64, 128))
      return kErrCuda;
  }
  // The post-merge map of shard r starts at row r*sh1 and spans
  // round_up(sh1, 128) rows: inside the xm/nm allocation (N*sh1_max + 128 rows).
  // Device 0's stream (where the forward starts) after every device's inputs:
  NEMO_CUDA_TRY(cudaSetDevice(hp->d[0].device));
  for (int r = 1; r < N; ++r) NEMO_CUDA_TRY(cudaStreamWaitEvent(hp->d[0].dp->stream, hp->d[r].ev_in, 0));

  int rc = kOk;
  auto git = hp->graphs.find(len);
  if (git == hp->graphs.end() && hp->warmed.count(len) && !hp->eager_only.count(len)) {
    // capture this length once (nothing runs during the capture)
    cudaStream_t s0 = hp->d[0].dp->stream;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool ok = cudaStreamBeginCapture(s0, cudaStreamCaptureModeRelaxed) == cudaSuccess;
    if (ok) {
      const int irc = hp_issue(plan, hp, maps, S0);
      cudaSetDevice(hp->d[0].device);
      ok = cudaStreamEndCapture(s0, &g) == cudaSuccess && g && !irc;
      ok = ok && cudaGraphInstantiate(&exec, g, 0) == cudaSuccess;
      if (g) cudaGraphDestroy(g);
    }
    if (ok) {
      git = hp->graphs.emplace(len, exec).first;
    } else {
      if (exec) cudaGraphExecDestroy(exec);
      cudaGetLastError();  // a failed capture: this length is issued directly from now on
      hp->eager_only.insert(len);
    }
  }
  if (git != hp->graphs.end()) {
    NEMO_CUDA_TRY(cudaSetDevice(hp->d[0].device));
    if (cudaGraphLaunch(git->second, hp->d[0].dp->stream) != cudaSuccess) {
      set_error("head-parallel graph launch failed");
      rc = kErrCuda;
    }
  } else {
    rc = hp_issue(plan, hp, maps, S0);
    if (!rc) hp->warmed.insert(len);
  }
  // ---- wait for device 0 (every device's work joins into its stream), then
  // every stream, with a host deadline ----
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(plan->host_deadline_ns);
  std::string msg = rc ? last_error() : std::string();
  for (int r = 0; r < N; ++r)
    if (int e = hp_wait(hp->d[r], deadline)) {
      if (!rc) {
        rc = e;
        msg = last_error();
      }
      if (e == kErrTimeout) break;
    }
  if (rc) {
    hp->failed = true;
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

extern "C" int nemo_hp_qkv_route(int n_devices, int* device, int* buffer, int* column) {
  if (!device || !buffer || !column || (n_devices != 2 && n_devices != 4 && n_devices != 8)) {
    nemo::set_error("nemo_hp_qkv_route: n_devices must be 2, 4 or 8 and the arrays non-null");
    return nemo::kErrArgs;
  }
  for (int c = 0; c < nemo::kQKVWidth; ++c) nemo::hp_qkv_route(c, n_devices, device + c, buffer + c, column + c);
  return nemo::kOk;
}

extern "C" int nemo_hp_row_owner(int n_devices, int rows_per_device, int n_positions, int* device) {
  if (!device || (n_devices != 2 && n_devices != 4 && n_devices != 8) || rows_per_device < 1 || n_positions < 0) {
    nemo::set_error("nemo_hp_row_owner: n_devices must be 2, 4 or 8, rows_per_device >= 1, device non-null");
    return nemo::kErrArgs;
  }
  for (int p = 0; p < n_positions; ++p) device[p] = nemo::hp_row_owner(p, rows_per_device, n_devices);
  return nemo::kOk;
}
