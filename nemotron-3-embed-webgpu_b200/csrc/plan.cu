// Execution plans: the B200 counterpart of NemotronExecutionPlan
// (src/webgpu/model.ts:58-234). A plan owns, per device, buffers sized for its
// worst case (capacity batch x sequence tokens), the RoPE table, and two CUDA
// graphs captured once at creation:
//   graph_host    H2D ids/lengths from pinned staging -> forward -> D2H output
//   graph_device  forward only (inputs already resident)
// Kernels read the run's token counts from device metadata, so one graph
// serves every run of the plan whatever the request lengths (only valid
// tokens are computed; padding rows are skipped, not masked).
#include <math.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <numeric>
#include <thread>

#include "runtime.h"

namespace nemo {

int model_load(const void* data, size_t bytes, const int* devices, int ndev, nemo_model** out);
void model_destroy(nemo_model* m);

const char* kStageNames[12] = {"embedding_norm", "token_merge",  "qkv",         "rope_attention",
                               "attention_output", "post_attention_norm", "ffn_up_gate", "swiglu",
                               "ffn_down",         "post_ffn_norm",       "pool",        "forward_fused"};
constexpr int kStageFused = 11;  // the whole forward as one persistent launch

struct Profile {
  std::vector<cudaEvent_t> events;
  std::vector<int> ids;
};

struct Dump {
  uint16_t* x = nullptr;
  uint16_t* norm = nullptr;
  int* tokens = nullptr;
  size_t stride = 0;
};

// Split-K factor and weight-ring depth of the small-T kernel. The splits of a
// tile form one cluster (at most 16 CTAs) and each needs >= 1 slab. Among the
// choices that fit shared memory, pick the one whose grid fills the GPU's CTA
// slots best in whole waves (two CTAs per SM when a CTA fits in half the SM's
// shared memory), preferring the deeper ring, then fewer splits.
void pick_splits(int tiles, int slabs, int np, int chunk_max, int* splits_out, int* rstages_out) {
  double best = -1.0;
  *splits_out = 1;
  *rstages_out = 2;
  for (int rs = 3; rs >= 2; --rs)
    for (int s = 1; s <= std::min(slabs, 16); ++s) {
      const size_t smem = skinny_smem_bytes(np, (slabs + s - 1) / s, chunk_max, rs);
      const int per_sm = smem <= 113 * 1024 ? 2 : smem <= 226 * 1024 ? 1 : 0;
      if (!per_sm) continue;
      const int slots = 148 * per_sm;
      const int ctas = tiles * s;
      const int waves = (ctas + slots - 1) / slots;
      // work per CTA ~ slabs/s; a wave costs the slowest CTA's slabs
      const double time = waves * (double)((slabs + s - 1) / s) + 0.05 * s;
      const double score = 1.0 / time;
      if (score > best + 1e-9) {
        best = score;
        *splits_out = s;
        *rstages_out = rs;
      }
    }
}

namespace {

int env_int(const char* name, int fallback) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : fallback;
}

// Bound of every wait inside the single-launch forward: 2 s, or shorter for a
// test that makes one run out (NEMO_TEST_WAIT_LIMIT_MS at plan creation).
int test_wait_limit_ms() { return std::min(2000, std::max(1, env_int("NEMO_TEST_WAIT_LIMIT_MS", 2000))); }

// Before each run of a plan created with NEMO_TEST_FAULTS set: the grid
// barrier the next run stalls at (NEMO_TEST_STALL_BARRIER, 0 = none).
int stage_test_stall(DevicePlan& p) {
  if (!p.test_stall) return kOk;
  *p.h_test_stall = (uint32_t)std::max(0, env_int("NEMO_TEST_STALL_BARRIER", 0));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.test_stall, p.h_test_stall, 4, cudaMemcpyHostToDevice, p.stream));
  return kOk;
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

template <typename T>
int plan_alloc(DevicePlan& p, T** ptr, size_t bytes) {
  void* v = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&v, bytes));
  NEMO_CUDA_TRY(cudaMemset(v, 0, bytes));
  p.allocations.push_back(v);
  *ptr = reinterpret_cast<T*>(v);
  return kOk;
}

template <typename T>
int plan_upload(DevicePlan& p, T** ptr, const std::vector<T>& host) {
  if (int rc = plan_alloc(p, ptr, std::max<size_t>(host.size() * sizeof(T), 16))) return rc;
  NEMO_CUDA_TRY(cudaMemcpy(*ptr, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice));
  return kOk;
}

// Sets up the persistent single-launch forward when the plan's worst case fits
// kFwdNP tokens (leaves p.fgrid = 0 otherwise). Weight work of QKV, O and
// down is split per projection into grid-many contiguous ranges of the
// tile-major (tile, slab) sequence; a range that crosses a tile boundary
// becomes two segments. Gate/up tiles are not split (one CTA each). Slots
// of a tile are numbered in K order, so the partial sums of a tile are always
// added in the same order. The CTA that takes range 0 rotates per projection
// so the CTAs with one extra slab differ from projection to projection.
int setup_forward(nemo_model* m, DeviceModel* dm, DevicePlan& p) {
  const int L = m->n_layers;
  if (p.tmax0 > kFwdNP || L <= kMergeAfterLayer) return kOk;
  const char* env = getenv("NEMO_FORWARD");
  if (env && strcmp(env, "per_op") == 0) return kOk;
  int chunk_max = 0;
  for (int l = 0; l < L; ++l)
    for (int w = 0; w < 4; ++w) {
      const Projection& P = dm->proj[l][w];
      if (P.tiles > kFwdMaxTiles || P.slabs > 255 || !P.packed) return kOk;
      chunk_max = std::max(chunk_max, P.chunk_max);
    }
  int G = 0;
  NEMO_CUDA_TRY(cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, p.device));
  if (G < 1) return kOk;

  // NEMO_FORWARD_GATE_UP=split: gate/up split over the whole grid like the
  // other projections (tile counters + SwiGLU by the CTA finishing a tile).
  const char* gu_env = getenv("NEMO_FORWARD_GATE_UP");
  const bool split_gate_up = gu_env && strcmp(gu_env, "split") == 0;
  std::vector<std::vector<FwdSeg>> per(G);
  std::vector<uint8_t> nslots((size_t)L * 4 * kFwdMaxTiles, 0);
  int max_slots = 1;
  std::vector<SkinnyTile> tiles;
  for (int pi = 0; pi < L * 4; ++pi) {
    const Projection& P = dm->proj[pi / 4][pi % 4];
    tiles.resize(P.tiles);
    NEMO_CUDA_TRY(cudaMemcpy(tiles.data(), P.d_tiles, P.tiles * sizeof(SkinnyTile), cudaMemcpyDeviceToHost));
    const long long U = (long long)P.tiles * P.slabs;
    const int rot = (int)(((long long)pi * 37) % G);
    auto add = [&](int c, int tile, int s0, int s1) -> bool {
      uint8_t& n = nslots[(size_t)pi * kFwdMaxTiles + tile];
      if (n == 255) return false;
      FwdSeg sg = {};
      sg.chunk0 = P.packed + tiles[tile].offset;
      sg.chunk_bytes = tiles[tile].chunk_bytes;
      sg.proj = (uint16_t)pi;
      sg.tile = (uint16_t)tile;
      sg.s0 = (uint8_t)s0;
      sg.s1 = (uint8_t)s1;
      sg.slot = n++;
      sg.fmt[0] = tiles[tile].fmt[0];
      sg.fmt[1] = tiles[tile].fmt[1];
      max_slots = std::max(max_slots, (int)n);
      per[c].push_back(sg);
      return true;
    };
    if (pi % 4 == 2 && P.tiles <= G && !split_gate_up) {
      // Gate/up: every tile whole on one CTA (spread evenly over the grid).
      // Its SwiGLU epilogue then runs straight from TMEM, with no partial
      // sums in global memory and no tile counter; the CTAs left over start
      // decoding their down-projection slabs early.
      for (int tile = 0; tile < P.tiles; ++tile)
        if (!add((int)(((long long)tile * G / P.tiles + rot) % G), tile, 0, P.slabs)) return kOk;
      continue;
    }
    for (int ce = 0; ce < G; ++ce) {
      const int u0 = (int)(ce * U / G), u1 = (int)((ce + 1) * U / G);
      const int c = (ce + rot) % G;
      // a CTA runs the epilogues of at most 4 tiles per projection
      if (u1 > u0 && (u1 - 1) / P.slabs - u0 / P.slabs + 1 > 4) return kOk;
      for (int u = u0; u < u1;) {
        const int tile = u / P.slabs, s0 = u % P.slabs;
        const int s1 = std::min(P.slabs, s0 + (u1 - u));
        if (!add(c, tile, s0, s1)) return kOk;
        u += s1 - s0;
      }
    }
  }
  // Items of the small phases that pause their CTA's decoders (attention and
  // the two norms of each layer) go first to the CTAs with the fewest slabs in
  // the projection that follows the phase.
  if (G > 255) return kOk;
  std::vector<uint8_t> small_rank((size_t)L * 3 * G, 0);
  {
    std::vector<int> order(G);
    for (int l = 0; l < L; ++l)
      for (int k = 0; k < 3; ++k) {
        const int next = k == 0 ? l * 4 + 1 : k == 1 ? l * 4 + 2 : (l + 1 < L ? (l + 1) * 4 : -1);
        std::vector<int> load(G, 0);
        if (next >= 0)
          for (int c = 0; c < G; ++c)
            for (const FwdSeg& sg : per[c])
              if (sg.proj == next) load[c] += sg.s1 - sg.s0;
        for (int c = 0; c < G; ++c) order[c] = c;
        std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return load[x] < load[y]; });
        for (int i = 0; i < G; ++i) small_rank[((size_t)l * 3 + k) * G + order[i]] = (uint8_t)i;
      }
  }
  std::vector<FwdSeg> segs;
  std::vector<int> start(G + 1, 0);
  int max_segs = 1;
  for (int c = 0; c < G; ++c) {
    start[c] = (int)segs.size();
    segs.insert(segs.end(), per[c].begin(), per[c].end());
    max_segs = std::max(max_segs, (int)per[c].size());
  }
  start[G] = (int)segs.size();
  std::vector<int> sstride((size_t)L * 4, 1);
  for (int pi = 0; pi < L * 4; ++pi)
    for (int t = 0; t < kFwdMaxTiles; ++t) sstride[pi] = std::max(sstride[pi], (int)nslots[(size_t)pi * kFwdMaxTiles + t]);
  // The gate/up epilogue pulls all slots of a tile into shared memory at once,
  // and the norms stage all O or down slots of a row.
  int gu_slots = 1, res_slots = 1;
  for (int l = 0; l < L; ++l) {
    gu_slots = std::max(gu_slots, sstride[(size_t)l * 4 + 2]);
    res_slots = std::max({res_slots, sstride[(size_t)l * 4 + 1], sstride[(size_t)l * 4 + 3]});
  }
  const int scratch_slots = forward_scratch_slots(gu_slots, res_slots);
  const size_t smem = forward_smem_bytes(chunk_max, scratch_slots, max_segs, L);
  if (smem > 227 * 1024) return kOk;
  int resident = 0;
  NEMO_CUDA_TRY(forward_max_grid(smem, &resident));
  if (resident != G) return kOk;

  FwdArgs& a = p.fargs;
  a = FwdArgs();
  int* d_sstride = nullptr;
  FwdSeg* d_segs = nullptr;
  int* d_start = nullptr;
  uint8_t* d_nslots = nullptr;
  uint8_t* d_small = nullptr;
  if (plan_upload(p, &d_sstride, sstride) || plan_upload(p, &d_segs, segs) || plan_upload(p, &d_start, start) ||
      plan_upload(p, &d_nslots, nslots) || plan_upload(p, &d_small, small_rank))
    return kErrCuda;
  p.fsync_bytes = (size_t)(1 + L * 4 * kFwdMaxTiles) * 4;
  if (plan_alloc(p, &p.fsync, p.fsync_bytes) ||
      plan_alloc(p, &a.part, (size_t)kFwdMaxTiles * max_slots * kFwdNP * 128 * 4))
    return kErrCuda;
  a.sstride = d_sstride;
  a.segs = d_segs;
  a.seg_start = d_start;
  a.nslots = d_nslots;
  a.small_rank = d_small;
  a.sync = p.fsync;
  a.err = p.err;
  a.ids = p.ids;
  a.embd = dm->embd;
  a.vocab = dm->vocab;
  for (int l = 0; l < L; ++l) {
    a.attn_norm[l] = dm->attn_norm[l];
    a.ffn_norm[l] = dm->ffn_norm[l];
  }
  a.output_norm = dm->output_norm;
  a.meta = p.meta;
  a.rope = p.rope;
  a.x = p.x;
  a.nrm = p.norm;
  a.xm = p.xm;
  a.nm = p.nm;
  a.qkv = p.qkv;
  a.q = p.q;
  a.k = p.k;
  a.attn = p.attn;
  a.delta = p.delta;
  a.ffn = p.ffn;
  a.max_slots = max_slots;
  a.scratch_slots = scratch_slots;
  a.max_segs = max_segs;
  a.rope_rows = p.seq;
  a.out = p.out;
  a.n_layers = L;
  a.chunk_max = chunk_max;
  a.exact = p.exact ? 1 : 0;
  a.wait_ns = (uint64_t)test_wait_limit_ms() * 1000000ull;
  a.test_stall = p.test_stall;
  // X operands by TMA; the small-T maps (box 64 x 16) exist because tmax0 <= 16.
  a.xmap[0] = p.xmap_norm[0];
  a.xmap[1] = p.xmap_norm[1];
  a.xmap[2] = p.xmap_attn[0];
  a.xmap[3] = p.xmap_ffn[0];
  p.fgrid = G;
  return kOk;
}

void free_device_plan(DevicePlan& p) {
  cudaSetDevice(p.device);
  if (p.graph_host) cudaGraphExecDestroy(p.graph_host);
  if (p.graph_device) cudaGraphExecDestroy(p.graph_device);
  for (void* v : p.allocations) cudaFree(v);
  if (p.h_ids) cudaFreeHost(p.h_ids);
  if (p.h_lengths) cudaFreeHost(p.h_lengths);
  if (p.h_out) cudaFreeHost(p.h_out);
  if (p.h_err) cudaFreeHost(p.h_err);
  if (p.h_test_stall) cudaFreeHost(p.h_test_stall);
  if (p.stream) cudaStreamDestroy(p.stream);
  p = DevicePlan();
}

}  // namespace

#define NEMO_LAUNCH(expr)                                                                              \
  do {                                                                                                 \
    cudaError_t _e = (expr);                                                                           \
    if (_e != cudaSuccess) {                                                                           \
      set_error(std::string("kernel launch failed: ") + cudaGetErrorString(_e) + " (" #expr ")");      \
      return kErrCuda;                                                                                 \
    }                                                                                                  \
  } while (0)

// Enqueues one forward pass (model.ts:152-168) on stream s.
int enqueue_forward(DevicePlan& p, int n_layers, cudaStream_t s, Profile* prof, Dump* dump) {
  DeviceModel& dm = *p.dm;
  auto stage = [&](int id) {
    if (!prof) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, s);
    prof->events.push_back(e);
    prof->ids.push_back(id);
  };
  const int* t0 = &p.meta->t0;
  const int* t1 = &p.meta->t1;
  NEMO_LAUNCH(launch_meta(p.lengths, p.cap_batch, p.seq, p.lengths + p.cap_batch, p.meta, s, p.exact ? 1 : 0));
  Meta host_meta;
  if (dump) {
    NEMO_CUDA_TRY(cudaMemcpyAsync(&host_meta, p.meta, sizeof(Meta), cudaMemcpyDeviceToHost, s));
    NEMO_CUDA_TRY(cudaStreamSynchronize(s));
  }
  if (p.fgrid && !dump) {
    NEMO_CUDA_TRY(cudaMemsetAsync(p.fsync, 0, p.fsync_bytes, s));
    stage(kStageFused);
    NEMO_LAUNCH(launch_forward(p.fargs, p.fgrid, s));
    stage(-1);
    return kOk;
  }
  stage(0);
  NEMO_LAUNCH(launch_embedding(p.ids, dm.embd, dm.vocab, p.meta, p.tmax0, p.x, s));
  NEMO_LAUNCH(launch_residual_rmsnorm(p.x, nullptr, dm.attn_norm[0], p.norm, t0, p.tmax0, s));
  for (int l = 0; l < n_layers; ++l) {
    const bool merged = !p.exact && l >= kMergeAfterLayer;
    if (l == kMergeAfterLayer && !p.exact) {
      stage(1);
      NEMO_LAUNCH(launch_merge(p.x, p.norm, p.meta, p.tmax1, p.xm, p.nm, s));
    }
    __half* X = merged ? p.xm : p.x;
    __half* N = merged ? p.nm : p.norm;
    const CUtensorMap* mapN = merged ? &p.map_norm1 : &p.map_norm0;
    const int* rows = merged ? t1 : t0;
    const int maxr = merged ? p.tmax1 : p.tmax0;
    Projection* pr = dm.proj[l];
    const int ph = merged ? 1 : 0;
    const int np = p.np[ph];
    // Small token counts: fused-dequant split-K kernel on the packed weights,
    // with RoPE fused into QKV and SwiGLU into gate/up.
    auto skinny = [&](int which, const CUtensorMap* xmap, int mode, __half* out, int ldo) -> int {
      const Projection& P = pr[which];
      SkinnyArgs a = {};
      a.packed = P.packed;
      a.tiles = P.d_tiles;
      a.err = p.err;
      a.d_tokens = rows;
      a.meta = p.meta;
      a.merged = merged ? 1 : 0;
      a.n = P.n;
      a.slabs = P.slabs;
      a.splits = p.splits[l][which];
      a.slabs_max = (P.slabs + a.splits - 1) / a.splits;
      a.chunk_max = P.chunk_max;
      a.rstages = p.rstages[l][which];
      a.mode = mode;
      a.out = out;
      a.ldo = ldo;
      a.q = p.q;
      a.k = p.k;
      a.rope = p.rope;
      a.pdl = 1;
      NEMO_LAUNCH(launch_skinny(xmap, a, np, P.tiles, s));
      return kOk;
    };
    // Batched token counts: dequant-fused tcgen05 GEMM over the packed weights.
    auto gemm_q = [&](int which, const CUtensorMap* xmap, int mode, __half* out, int ldo) -> int {
      const Projection& P = pr[which];
      NEMO_LAUNCH(launch_gemm_q(xmap, P.packed, P.d_tiles, P.tiles, P.slabs, P.chunk_max, mode, out, ldo, rows, maxr,
                                p.err, s));
      return kOk;
    };
    stage(2);
    if (np) {
      if (int rc = skinny(kProjQKV, &p.xmap_norm[ph], kSkinnyRope, p.qkv, kQKVWidth)) return rc;
      stage(3);
    } else {
      if (p.batched_f16) {
        // RoPE in the GEMM epilogue: Q/K straight into the attention inputs
        GemmEpi ep;
        ep.mode = kSkinnyRope;
        ep.meta = p.meta;
        ep.merged = merged ? 1 : 0;
        ep.rope = p.rope;
        ep.q = p.q;
        ep.k = p.k;
        NEMO_LAUNCH(launch_gemm_tc_epi(mapN, &pr[kProjQKV].map[p.bn[l][0]], p.qkv, kQKVWidth, rows, maxr, kQKVWidth,
                                       kHidden, kBnChoices[p.bn[l][0]], ep, p.err, s));
        stage(3);
      } else {
        if (int rc = gemm_q(kProjQKV, mapN, kSkinnyPlain, p.qkv, kQKVWidth)) return rc;
        stage(3);
        NEMO_LAUNCH(launch_rope(p.qkv, p.rope, p.meta, merged, maxr, p.q, p.k, s));
      }
    }
    if (p.gather[ph]) NEMO_LAUNCH(launch_gather_sampled(p.k, p.qkv, p.meta, merged, p.rows_c, p.kc, p.vc, s));
    NEMO_LAUNCH(launch_attention_tc(p.amaps, p.meta, merged, p.cap_batch, merged ? p.mseq : p.seq, p.attn, p.err, s));
    stage(4);
    if (np) {
      if (int rc = skinny(kProjO, &p.xmap_attn[ph], kSkinnyPlain, p.delta, kHidden)) return rc;
    } else if (p.batched_f16) {
      GemmEpi ep;
      ep.part = p.part;
      ep.splits_out = p.part ? p.ksplit_used : nullptr;
      NEMO_LAUNCH(launch_gemm_tc_epi(&p.map_attn, &pr[kProjO].map[2], p.delta, kHidden, rows, maxr, kHidden, kQWidth,
                                     256, ep, p.err, s));
    } else if (int rc = gemm_q(kProjO, &p.map_attn, kSkinnyPlain, p.delta, kHidden)) {
      return rc;
    }
    stage(5);
    // the batched f16 O and down GEMMs may leave K-split partial sums
    const bool parts = !np && p.batched_f16 && p.part;
    if (parts)
      NEMO_LAUNCH(
          launch_residual_rmsnorm_parts(X, p.delta, p.part, p.ksplit_used, dm.ffn_norm[l], N, rows, maxr, s));
    else
      NEMO_LAUNCH(launch_residual_rmsnorm(X, p.delta, dm.ffn_norm[l], N, rows, maxr, s));
    stage(6);
    if (np) {
      if (int rc = skinny(kProjGateUp, &p.xmap_norm[ph], kSkinnySwiglu, p.ffn, kInter)) return rc;
      stage(7);
    } else if (p.batched_f16) {
      // SwiGLU in the GEMM epilogue: each CTA multiplies bn/2 gate rows and
      // the matching up rows (tensor map box bn/2), so bn >= 128
      const int bi = std::max(1, p.bn[l][2]);
      GemmEpi ep;
      ep.mode = kSkinnySwiglu;
      NEMO_LAUNCH(launch_gemm_tc_epi(mapN, &pr[kProjGateUp].map[bi - 1], p.ffn, kInter, rows, maxr, 2 * kInter,
                                     kHidden, kBnChoices[bi], ep, p.err, s));
      stage(7);
    } else {
      // SwiGLU fused into the epilogue (tiles interleave 64 gate + 64 up rows)
      if (int rc = gemm_q(kProjGateUp, mapN, kSkinnySwiglu, p.ffn, kInter)) return rc;
      stage(7);
    }
    stage(8);
    if (np) {
      if (int rc = skinny(kProjDown, &p.xmap_ffn[ph], kSkinnyPlain, p.delta, kHidden)) return rc;
    } else if (p.batched_f16) {
      GemmEpi ep;
      ep.part = p.part;
      ep.splits_out = p.part ? p.ksplit_used + 1 : nullptr;
      NEMO_LAUNCH(launch_gemm_tc_epi(&p.map_ffn, &pr[kProjDown].map[2], p.delta, kHidden, rows, maxr, kHidden, kInter,
                                     256, ep, p.err, s));
    } else if (int rc = gemm_q(kProjDown, &p.map_ffn, kSkinnyPlain, p.delta, kHidden)) {
      return rc;
    }
    stage(9);
    const float* next = l + 1 < n_layers ? dm.attn_norm[l + 1] : dm.output_norm;
    if (parts)
      NEMO_LAUNCH(launch_residual_rmsnorm_parts(X, p.delta, p.part, p.ksplit_used + 1, next, N, rows, maxr, s));
    else
      NEMO_LAUNCH(launch_residual_rmsnorm(X, p.delta, next, N, rows, maxr, s));
    if (dump) {
      const int T = merged ? host_meta.t1 : host_meta.t0;
      if (dump->tokens) dump->tokens[l] = T;
      if (dump->x)
        NEMO_CUDA_TRY(cudaMemcpyAsync(dump->x + (size_t)l * dump->stride, X, (size_t)T * kHidden * 2,
                                      cudaMemcpyDeviceToHost, s));
      if (dump->norm)
        NEMO_CUDA_TRY(cudaMemcpyAsync(dump->norm + (size_t)l * dump->stride, N, (size_t)T * kHidden * 2,
                                      cudaMemcpyDeviceToHost, s));
      NEMO_CUDA_TRY(cudaStreamSynchronize(s));
    }
  }
  stage(10);
  NEMO_LAUNCH(launch_mean_pool(p.exact ? p.norm : p.nm, p.meta, p.cap_batch, p.out, s));
  stage(-1);
  return kOk;
}

namespace {

int capture(DevicePlan& p, int n_layers, bool host_io, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  NEMO_CUDA_TRY(cudaStreamBeginCapture(p.stream, cudaStreamCaptureModeThreadLocal));
  int rc = kOk;
  auto body = [&]() -> int {
    NEMO_CUDA_TRY(cudaMemsetAsync(p.err, 0, 4, p.stream));
    if (host_io) {
      NEMO_CUDA_TRY(cudaMemcpyAsync(p.ids, p.h_ids, (size_t)p.cap_batch * p.seq * 4, cudaMemcpyHostToDevice, p.stream));
      NEMO_CUDA_TRY(cudaMemcpyAsync(p.lengths, p.h_lengths, (size_t)(p.cap_batch + 1) * 4, cudaMemcpyHostToDevice,
                                    p.stream));
    }
    if (int r = enqueue_forward(p, n_layers, p.stream, nullptr, nullptr)) return r;
    if (host_io) {
      NEMO_CUDA_TRY(cudaMemcpyAsync(p.h_out, p.out, (size_t)p.cap_batch * kHidden * 4, cudaMemcpyDeviceToHost,
                                    p.stream));
    }
    NEMO_CUDA_TRY(cudaMemcpyAsync(p.h_err, p.err, 4, cudaMemcpyDeviceToHost, p.stream));
    return kOk;
  };
  rc = body();
  cudaError_t e = cudaStreamEndCapture(p.stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) {
    set_error(std::string("graph capture failed: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error(std::string("graph instantiate failed: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  return kOk;
}

int create_device_plan(nemo_model* m, DeviceModel* dm, int cap_batch, int seq, bool exact, DevicePlan& p) {
  p.exact = exact;
  {
    const char* env = getenv("NEMO_BATCHED");
    p.batched_f16 = !(env && strcmp(env, "fused") == 0);
  }
  p.device = dm->device;
  p.dm = dm;
  p.cap_batch = cap_batch;
  p.seq = seq;
  p.mseq = exact ? seq : (int)std::max(1.0, ceil(seq * 0.64));
  p.tmax0 = cap_batch * seq;
  p.tmax1 = cap_batch * p.mseq;
  p.rows0 = round_up(p.tmax0, kGemmTileM);
  p.rows1 = round_up(p.tmax1, kGemmTileM);
  NEMO_CUDA_TRY(cudaSetDevice(p.device));
  NEMO_CUDA_TRY(cudaStreamCreateWithFlags(&p.stream, cudaStreamNonBlocking));
  const size_t r0 = p.rows0, r1 = p.rows1;
  if (plan_alloc(p, &p.ids, (size_t)p.tmax0 * 4) || plan_alloc(p, &p.lengths, (size_t)(cap_batch + 1) * 4) ||
      plan_alloc(p, &p.meta, sizeof(Meta)) || plan_alloc(p, &p.err, 256) ||
      plan_alloc(p, &p.rope, (size_t)seq * 128 * 4) || plan_alloc(p, &p.x, r0 * kHidden * 2) ||
      plan_alloc(p, &p.norm, r0 * kHidden * 2) || plan_alloc(p, &p.xm, r1 * kHidden * 2) ||
      plan_alloc(p, &p.nm, r1 * kHidden * 2) || plan_alloc(p, &p.qkv, r0 * kQKVWidth * 2) ||
      plan_alloc(p, &p.q, r0 * kQWidth * 2) || plan_alloc(p, &p.k, r0 * kKVWidth * 2) ||
      plan_alloc(p, &p.attn, r0 * kQWidth * 2) || plan_alloc(p, &p.delta, r0 * kHidden * 2) ||
      plan_alloc(p, &p.gu, r0 * 2 * kInter * 2) || plan_alloc(p, &p.ffn, r0 * kInter * 2) ||
      plan_alloc(p, &p.out, (size_t)cap_batch * kHidden * 4))
    return kErrCuda;
  NEMO_CUDA_TRY(cudaMallocHost(&p.h_ids, (size_t)p.tmax0 * 4));
  NEMO_CUDA_TRY(cudaMallocHost(&p.h_lengths, (size_t)(cap_batch + 1) * 4));
  NEMO_CUDA_TRY(cudaMallocHost(&p.h_out, (size_t)cap_batch * kHidden * 4));
  NEMO_CUDA_TRY(cudaMallocHost(&p.h_err, 4));
  for (int i = 0; i < p.tmax0; ++i) p.h_ids[i] = 0;
  for (int b = 0; b < cap_batch; ++b) p.h_lengths[b] = 1;
  p.h_lengths[cap_batch] = cap_batch;
  *p.h_err = 0;
  // model.ts:95-107 (f64 math, stored f32).
  std::vector<float> rope((size_t)seq * 128);
  rope_table_host(seq, rope.data());
  NEMO_CUDA_TRY(cudaMemcpy(p.rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice));
  if (make_tmap_f16(&p.map_norm0, p.norm, kHidden, r0, 64, kGemmTileM) ||
      make_tmap_f16(&p.map_norm1, p.nm, kHidden, r1, 64, kGemmTileM) ||
      make_tmap_f16(&p.map_attn, p.attn, kQWidth, r0, 64, kGemmTileM) ||
      make_tmap_f16(&p.map_ffn, p.ffn, kInter, r0, 64, kGemmTileM))
    return kErrCuda;
  // Attention: compact sampled K/V only when a phase can exceed 2048 keys.
  p.gather[0] = !exact && p.seq > kSampleThreshold;
  p.gather[1] = !exact && p.mseq > kSampleThreshold;
  p.rows_c = (p.gather[0] || p.gather[1]) ? p.tmax0 / kSampleStride + cap_batch + 1 : kGemmTileM;
  if (plan_alloc(p, &p.kc, (size_t)p.rows_c * kKVWidth * 2) || plan_alloc(p, &p.vc, (size_t)p.rows_c * kKVWidth * 2))
    return kErrCuda;
  if (make_tmap_f16(&p.amaps.q, p.q, kQWidth, r0, 64, 128) || make_tmap_f16(&p.amaps.k, p.k, kKVWidth, r0, 64, 128) ||
      make_tmap_f16(&p.amaps.v, p.qkv, kQKVWidth, r0, 64, 128) ||
      make_tmap_f16(&p.amaps.kc, p.kc, kKVWidth, p.rows_c, 64, 128) ||
      make_tmap_f16(&p.amaps.vc, p.vc, kKVWidth, p.rows_c, 64, 128))
    return kErrCuda;
  for (int l = 0; l < m->n_layers; ++l) {
    const int rows = l >= kMergeAfterLayer ? p.rows1 : p.rows0;
    for (int w = 0; w < 4; ++w) p.bn[l][w] = pick_bn(rows, kProjN[w]);
  }
  // Batched O and down (f16 weights): 2048 / 256 n tiles, K split on the
  // device by gemm_ksplit for the valid token count; the partial-sum buffer
  // covers every count up to the plan's rows.
  NEMO_CUDA_TRY(cudaDeviceGetAttribute(&p.sms, cudaDevAttrMultiProcessorCount, p.device));
  {
    size_t need = 0;
    for (int mt = 1; mt <= (int)(r0 / kGemmTileM); ++mt)
      for (const int kt : {kQWidth / 64, kInter / 64}) {
        const int sp = gemm_ksplit(mt, kHidden / 256, kt, p.sms);
        if (sp > 1) need = std::max(need, (size_t)sp * mt * kGemmTileM * kHidden * 4);
      }
    if (need && (plan_alloc(p, &p.part, need) || plan_alloc(p, &p.ksplit_used, 2 * sizeof(int)))) return kErrCuda;
  }
  // Small-T path: worst-case tokens of the phase padded to the MMA N size.
  const int tmax[2] = {p.tmax0, p.tmax1};
  for (int ph = 0; ph < 2; ++ph) {
    p.np[ph] = tmax[ph] <= 16 ? 16 : tmax[ph] <= 32 ? 32 : tmax[ph] <= 64 ? 64 : 0;
    if (!p.np[ph]) continue;
    if (make_tmap_f16(&p.xmap_norm[ph], ph ? (void*)p.nm : (void*)p.norm, kHidden, ph ? r1 : r0, 64, p.np[ph]) ||
        make_tmap_f16(&p.xmap_attn[ph], p.attn, kQWidth, r0, 64, p.np[ph]) ||
        make_tmap_f16(&p.xmap_ffn[ph], p.ffn, kInter, r0, 64, p.np[ph]))
      return kErrCuda;
  }
  for (int l = 0; l < m->n_layers; ++l) {
    const int ph = l >= kMergeAfterLayer ? 1 : 0;
    if (!p.np[ph]) continue;
    for (int w = 0; w < 4; ++w) {
      const Projection& P = dm->proj[l][w];
      pick_splits(P.tiles, P.slabs, p.np[ph], P.chunk_max, &p.splits[l][w], &p.rstages[l][w]);
      if (skinny_smem_bytes(p.np[ph], (P.slabs + p.splits[l][w] - 1) / p.splits[l][w], P.chunk_max,
                            p.rstages[l][w]) > 227 * 1024) {
        set_error("small-T projection does not fit shared memory");
        return kErrState;
      }
    }
  }

  // The lengths buffer must hold a valid run before the first launch.
  NEMO_CUDA_TRY(cudaMemcpy(p.lengths, p.h_lengths, (size_t)(cap_batch + 1) * 4, cudaMemcpyHostToDevice));
  if (env_int("NEMO_TEST_FAULTS", 0)) {
    if (plan_alloc(p, &p.test_stall, 4)) return kErrCuda;
    NEMO_CUDA_TRY(cudaMallocHost(&p.h_test_stall, 4));
    *p.h_test_stall = 0;
  }
  if (int rc = setup_forward(m, dm, p)) return rc;
  if (int rc = capture(p, m->n_layers, true, &p.graph_host)) return rc;
  if (int rc = capture(p, m->n_layers, false, &p.graph_device)) return rc;
  return kOk;
}

}  // namespace

void rope_table_host(int sequence, float* table) {
  const double frequency_scale = 1.0 / 16.0;
  auto correction = [](double beta) {
    return 128.0 * log(16384.0 / (beta * 2.0 * M_PI)) / (2.0 * log(kRopeTheta));
  };
  const double low = floor(correction(32.0));
  const double high = ceil(correction(1.0));
  for (int pos = 0; pos < sequence; ++pos)
    for (int d = 0; d < 64; ++d) {
      double t = (d - low) / fmax(0.001, high - low);
      t = fmin(1.0, fmax(0.0, t));
      const double ramp = 1.0 - t;
      const double frequency = frequency_scale * (1.0 - ramp) + ramp;
      const double angle = pos * pow(kRopeTheta, -d / 64.0) * frequency;
      table[((size_t)pos * 64 + d) * 2] = (float)cos(angle);
      table[((size_t)pos * 64 + d) * 2 + 1] = (float)sin(angle);
    }
}

int plan_create(nemo_model* m, uint32_t batch, uint32_t seq, uint32_t flags, nemo_plan** out) {
  if (!m || !out) {
    set_error("nemo_plan_create: null argument");
    return kErrArgs;
  }
  *out = nullptr;
  if (batch < 1 || batch > (uint32_t)kMaxBatch) {
    set_error("batch must be between 1 and 16");
    return kErrArgs;
  }
  if (seq < 1 || seq > 32768u) {
    set_error("sequence must be between 1 and 32768");
    return kErrArgs;
  }
  auto* plan = new nemo_plan();
  plan->model = m;
  plan->batch = (int)batch;
  plan->seq = (int)seq;
  plan->exact = (flags & 1u) != 0;
  plan->host_deadline_ns = (int64_t)std::max(1, env_int("NEMO_HOST_DEADLINE_MS", 60000)) * 1000000ll;
  plan->fail_device = env_int("NEMO_TEST_FAIL_DEVICE", -1);
  for (auto& dm : m->devs) {
    auto dp = std::make_unique<DevicePlan>();
    int rc = create_device_plan(m, dm.get(), (int)batch, (int)seq, plan->exact, *dp);
    plan->devs.push_back(std::move(dp));
    if (rc) {
      for (auto& d : plan->devs) free_device_plan(*d);
      delete plan;
      return rc;
    }
  }
  // Multi-device plans of one request: from hp_min tokens on (default 5000,
  // NEMO_HEAD_PARALLEL_MIN overrides) the request runs head-parallel.
  if (plan->devs.size() >= 2 && batch == 1 && !plan->exact) {
    const char* env = getenv("NEMO_HEAD_PARALLEL_MIN");
    plan->hp_min = env ? std::max(1, atoi(env)) : 5000;
    if ((int)seq >= plan->hp_min) {
      if (int rc = hp_create(plan, &plan->hp)) {
        for (auto& d : plan->devs) free_device_plan(*d);
        delete plan;
        return rc;
      }
    }
  }
  *out = plan;
  return kOk;
}

void plan_destroy(nemo_plan* plan) {
  if (!plan) return;
  hp_destroy(plan->hp);
  plan->hp = nullptr;
  for (auto& d : plan->devs) {
    cudaSetDevice(d->device);
    cudaStreamSynchronize(d->stream);
    free_device_plan(*d);
  }
  delete plan;
}

namespace {

int validate_inputs(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths) {
  if (!ids || !lengths) {
    set_error("null ids or lengths");
    return kErrArgs;
  }
  if (n_ids != (size_t)plan->batch * plan->seq) {
    set_error("token buffer does not match execution plan");  // model.ts:147
    return kErrArgs;
  }
  if (n_lengths != (size_t)plan->batch) {
    set_error("lengths buffer does not match execution plan batch");
    return kErrArgs;
  }
  for (int b = 0; b < plan->batch; ++b)
    if (lengths[b] < 1 || lengths[b] > (uint32_t)plan->seq) {
      set_error("lengths[" + std::to_string(b) + "] = " + std::to_string(lengths[b]) + " is outside [1, sequence]");
      return kErrArgs;
    }
  const uint32_t vocab = (uint32_t)plan->model->vocab;
  for (int b = 0; b < plan->batch; ++b)
    for (uint32_t i = 0; i < lengths[b]; ++i)
      if (ids[(size_t)b * plan->seq + i] >= vocab) {
        set_error("token id " + std::to_string(ids[(size_t)b * plan->seq + i]) + " is outside the vocabulary");
        return kErrArgs;
      }
  return kOk;
}

// Waits for the device's stream with a host-side deadline: polls the stream
// instead of blocking in cudaStreamSynchronize, so a caller never waits longer
// than the plan's deadline (the device-side waits are bounded as well).
int wait_stream(DevicePlan& d, int64_t deadline_ns) {
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0;; ++i) {
    const cudaError_t e = cudaStreamQuery(d.stream);
    if (e == cudaSuccess) return kOk;
    if (e != cudaErrorNotReady) {
      set_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " while waiting for device " +
                std::to_string(d.device));
      return kErrCuda;
    }
    if ((i & 63u) == 63u) {
      if (std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count() >
          deadline_ns) {
        set_error("host deadline of " + std::to_string(deadline_ns / 1000000) + " ms passed waiting for device " +
                  std::to_string(d.device));
        return kErrTimeout;
      }
      std::this_thread::yield();
    }
  }
}

int check_err(DevicePlan& d) {
  if (*d.h_err) {
    set_error("a device-side bounded wait timed out (error word " + std::to_string(*d.h_err) + ")");
    return kErrTimeout;
  }
  return kOk;
}

}  // namespace

int plan_run(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
             float* out) {
  if (!plan || !out) {
    set_error("nemo_plan_run: null argument");
    return kErrArgs;
  }
  if (int rc = validate_inputs(plan, ids, n_ids, lengths, n_lengths)) return rc;
  const int ndev = (int)plan->devs.size();
  if (plan->hp && (int)lengths[0] >= plan->hp_min) return hp_run(plan, plan->hp, ids, (int)lengths[0], out);
  // Request sharding: longest first onto the device with the fewest tokens.
  std::vector<std::vector<int>> assign(ndev);
  if (ndev == 1) {
    assign[0].resize(plan->batch);
    std::iota(assign[0].begin(), assign[0].end(), 0);
  } else {
    std::vector<int> order(plan->batch);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lengths[a] > lengths[b]; });
    std::vector<long long> load(ndev, 0);
    for (int r : order) {
      const int d = (int)(std::min_element(load.begin(), load.end()) - load.begin());
      assign[d].push_back(r);
      load[d] += lengths[r];
    }
  }
  // A failure on any device rejects the whole micro-batch (the caller's
  // engine rejects every request of it, embedding-engine.ts:84-89); the other
  // devices' work is still waited for, so nothing is in flight on return.
  int rc = kOk;
  std::vector<bool> launched(ndev, false);
  for (int d = 0; d < ndev; ++d) {
    DevicePlan& p = *plan->devs[d];
    if (assign[d].empty()) continue;
    if (d == plan->fail_device) {
      set_error("injected failure of device " + std::to_string(p.device) + "'s share (NEMO_TEST_FAIL_DEVICE)");
      rc = kErrCuda;
      continue;
    }
    for (size_t j = 0; j < assign[d].size(); ++j) {
      const int r = assign[d][j];
      memcpy(p.h_ids + j * p.seq, ids + (size_t)r * plan->seq, (size_t)plan->seq * 4);
      p.h_lengths[j] = lengths[r];
    }
    p.h_lengths[p.cap_batch] = (uint32_t)assign[d].size();
    cudaError_t e = cudaSetDevice(p.device);
    if (e == cudaSuccess && stage_test_stall(p) != kOk) e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaGraphLaunch(p.graph_host, p.stream);
    if (e != cudaSuccess) {
      set_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " launching device " + std::to_string(p.device));
      rc = kErrCuda;
      continue;
    }
    launched[d] = true;
  }
  const std::string first_error = rc ? last_error() : "";
  for (int d = 0; d < ndev; ++d) {
    DevicePlan& p = *plan->devs[d];
    if (!launched[d]) continue;
    int e = cudaSetDevice(p.device) == cudaSuccess ? wait_stream(p, plan->host_deadline_ns) : kErrCuda;
    if (!e) e = check_err(p);
    if (e) {
      if (!rc) rc = e;
      continue;
    }
    for (size_t j = 0; j < assign[d].size(); ++j)
      memcpy(out + (size_t)assign[d][j] * kHidden, p.h_out + j * kHidden, kHidden * 4);
  }
  if (!first_error.empty()) set_error(first_error);
  return rc;
}

int plan_run_device(nemo_plan* plan, const uint32_t* d_ids, const uint32_t* d_lengths, float* d_out) {
  if (!plan || !d_ids || !d_lengths || !d_out) {
    set_error("nemo_plan_run_device: null argument");
    return kErrArgs;
  }
  if (plan->devs.size() != 1) {
    set_error("nemo_plan_run_device needs a single-device plan");
    return kErrState;
  }
  DevicePlan& p = *plan->devs[0];
  NEMO_CUDA_TRY(cudaSetDevice(p.device));
  p.h_lengths[p.cap_batch] = (uint32_t)p.cap_batch;
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.ids, d_ids, (size_t)p.cap_batch * p.seq * 4, cudaMemcpyDeviceToDevice, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.lengths, d_lengths, (size_t)p.cap_batch * 4, cudaMemcpyDeviceToDevice, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.lengths + p.cap_batch, p.h_lengths + p.cap_batch, 4, cudaMemcpyHostToDevice,
                                p.stream));
  if (int rc = stage_test_stall(p)) return rc;
  NEMO_CUDA_TRY(cudaGraphLaunch(p.graph_device, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(d_out, p.out, (size_t)p.cap_batch * kHidden * 4, cudaMemcpyDeviceToDevice, p.stream));
  return kOk;
}

int plan_synchronize(nemo_plan* plan) {
  if (!plan) return kErrArgs;
  int rc = kOk;
  for (auto& d : plan->devs) {
    NEMO_CUDA_TRY(cudaSetDevice(d->device));
    NEMO_CUDA_TRY(cudaStreamSynchronize(d->stream));
    if (int e = check_err(*d)) rc = e;
  }
  return rc;
}

static int stage_host_inputs(nemo_plan* plan, DevicePlan& p, const uint32_t* ids, const uint32_t* lengths) {
  memcpy(p.h_ids, ids, (size_t)plan->batch * plan->seq * 4);
  for (int b = 0; b < plan->batch; ++b) p.h_lengths[b] = lengths[b];
  p.h_lengths[p.cap_batch] = (uint32_t)plan->batch;
  NEMO_CUDA_TRY(cudaSetDevice(p.device));
  NEMO_CUDA_TRY(cudaMemsetAsync(p.err, 0, 4, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.ids, p.h_ids, (size_t)p.tmax0 * 4, cudaMemcpyHostToDevice, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.lengths, p.h_lengths, (size_t)(p.cap_batch + 1) * 4, cudaMemcpyHostToDevice,
                                p.stream));
  return kOk;
}

int plan_profile(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                 float* stage_ms) {
  if (!plan || !stage_ms) {
    set_error("nemo_plan_profile: null argument");
    return kErrArgs;
  }
  if (int rc = validate_inputs(plan, ids, n_ids, lengths, n_lengths)) return rc;
  DevicePlan& p = *plan->devs[0];
  if (int rc = stage_host_inputs(plan, p, ids, lengths)) return rc;
  Profile prof;
  int rc = enqueue_forward(p, plan->model->n_layers, p.stream, &prof, nullptr);
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.h_err, p.err, 4, cudaMemcpyDeviceToHost, p.stream));
  NEMO_CUDA_TRY(cudaStreamSynchronize(p.stream));
  for (int i = 0; i <= kStageFused; ++i) stage_ms[i] = 0.f;
  for (size_t i = 0; i + 1 < prof.events.size(); ++i) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, prof.events[i], prof.events[i + 1]);
    if (prof.ids[i] >= 0) stage_ms[prof.ids[i]] += ms;
  }
  for (cudaEvent_t e : prof.events) cudaEventDestroy(e);
  if (rc) return rc;
  return check_err(p);
}

int plan_run_debug(nemo_plan* plan, const uint32_t* ids, size_t n_ids, const uint32_t* lengths, size_t n_lengths,
                   float* out, uint16_t* x_dump, uint16_t* norm_dump, int* tokens_per_layer) {
  if (!plan || !out) {
    set_error("nemo_plan_run_debug: null argument");
    return kErrArgs;
  }
  if (plan->devs.size() != 1) {
    set_error("nemo_plan_run_debug needs a single-device plan");
    return kErrState;
  }
  if (int rc = validate_inputs(plan, ids, n_ids, lengths, n_lengths)) return rc;
  DevicePlan& p = *plan->devs[0];
  if (int rc = stage_host_inputs(plan, p, ids, lengths)) return rc;
  Dump dump;
  dump.x = x_dump;
  dump.norm = norm_dump;
  dump.tokens = tokens_per_layer;
  dump.stride = (size_t)plan->batch * plan->seq * kHidden;
  if (int rc = enqueue_forward(p, plan->model->n_layers, p.stream, nullptr, &dump)) return rc;
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.h_out, p.out, (size_t)plan->batch * kHidden * 4, cudaMemcpyDeviceToHost, p.stream));
  NEMO_CUDA_TRY(cudaMemcpyAsync(p.h_err, p.err, 4, cudaMemcpyDeviceToHost, p.stream));
  NEMO_CUDA_TRY(cudaStreamSynchronize(p.stream));
  memcpy(out, p.h_out, (size_t)plan->batch * kHidden * 4);
  return check_err(p);
}

}  // namespace nemo
