// Host-side objects behind the C ABI: per-device model replicas and plans.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "wgpack.h"

struct nemo_model;
struct nemo_plan;

namespace nemo {

constexpr int kProjQKV = 0, kProjO = 1, kProjGateUp = 2, kProjDown = 3;
constexpr int kProjN[4] = {kQKVWidth, kHidden, 2 * kInter, kHidden};
constexpr int kProjK[4] = {kHidden, kQWidth, kHidden, kInter};
constexpr int kNumBn = 3;
constexpr int kBnChoices[kNumBn] = {64, 128, 256};

// BN of a batched projection GEMM: the one that needs the fewest waves of
// output tiles over the 148 SMs, the narrowest on a tie. A tile's fixed cost
// (pipeline fill, X loads, epilogue) is about that of 64-100 columns of its
// weight stream, so a second, nearly empty wave of narrow tiles costs more
// than one wave of wide ones that leaves SMs idle (16 x 15 tokens: QKV
// 0.557 -> 0.414 ms and gate/up 0.622 -> 0.490 ms per forward against
// choosing the widest BN that still fills every SM).
inline int pick_bn(int rows, int n) {
  const long long mt = (rows + kGemmTileM - 1) / kGemmTileM;
  int best = 2;
  long long best_waves = -1;
  for (int b = 0; b < 3; ++b) {
    const long long tiles = mt * (n / kBnChoices[b]);
    const long long waves = (tiles + 147) / 148;
    if (best_waves < 0 || waves < best_waves) {
      best = b;
      best_waves = waves;
    }
  }
  return best;
}


// A row range of a projection stored in one quantised format.
struct Segment {
  int fmt = 0;        // SegFormat
  int row0 = 0;
  int rows = 0;
  size_t bytes = 0;  // the pack's block bytes (decoded at load, not kept on the device)
};

struct Projection {
  int n = 0, k = 0;
  __half* w16 = nullptr;     // effective f16 weights, [n x k] row-major
  CUtensorMap map[kNumBn];   // TMA maps over w16, box 64 x bn
  std::vector<Segment> segs;
  // Tile-slab packed copy for the fused-dequant small-T kernel (k_skinny.cu).
  // Gate/up tiles interleave 64 gate rows with the matching 64 up rows.
  uint8_t* packed = nullptr;
  SkinnyTile* d_tiles = nullptr;
  int tiles = 0;
  int slabs = 0;
  int chunk_max = 0;
  size_t packed_bytes = 0;
};

// Host-side tile-slab image of one projection, built once per model.
struct TileSlabImage {
  std::vector<uint8_t> bytes;
  std::vector<SkinnyTile> tiles;
  int chunk_max = 0;
};

struct DeviceModel {
  int device = 0;
  uint8_t* embd = nullptr;   // Q6_K token table, vocab x 8 blocks x 210 B
  int vocab = 0;
  float* attn_norm[kMaxLayers] = {};
  float* ffn_norm[kMaxLayers] = {};
  float* output_norm = nullptr;
  Projection proj[kMaxLayers][4];
  std::vector<void*> allocations;
  size_t bytes = 0;
};

// One device's share of a plan: buffers sized for the plan's worst case
// (capacity batch x sequence), pinned staging, and the captured graph.
struct DevicePlan {
  int device = 0;
  DeviceModel* dm = nullptr;
  int cap_batch = 0, seq = 0, mseq = 0;
  int tmax0 = 0, tmax1 = 0;  // worst-case valid tokens before / after merge
  int rows0 = 0, rows1 = 0;  // tmax rounded up to the GEMM M tile
  cudaStream_t stream = nullptr;
  // device buffers
  uint32_t* ids = nullptr;
  uint32_t* lengths = nullptr;
  Meta* meta = nullptr;
  uint32_t* err = nullptr;
  float* rope = nullptr;
  __half *x = nullptr, *norm = nullptr, *xm = nullptr, *nm = nullptr;
  __half *qkv = nullptr, *q = nullptr, *k = nullptr, *attn = nullptr, *delta = nullptr;
  __half *gu = nullptr, *ffn = nullptr;
  float* out = nullptr;
  // K-split f32 partial sums of the batched O and down GEMMs (gemm_ksplit),
  // sized for the largest split x rows any valid token count can use; sms is
  // the grid of those GEMMs.
  float* part = nullptr;
  int* ksplit_used = nullptr;  // [2]: the K splits the last O and down GEMMs used
  int sms = 0;
  // pinned host staging
  uint32_t* h_ids = nullptr;
  uint32_t* h_lengths = nullptr;
  float* h_out = nullptr;
  uint32_t* h_err = nullptr;
  CUtensorMap map_norm0, map_norm1, map_attn, map_ffn;
  int bn[kMaxLayers][4] = {};
  // Small-T fused-dequant path: tokens padded to np (16/32/64) per phase
  // (0 = layers 0-3, 1 = layers 4+); 0 selects the batched tcgen05 GEMM.
  int np[2] = {0, 0};
  CUtensorMap xmap_norm[2], xmap_attn[2], xmap_ffn[2];  // box 64 x np[phase]
  // tcgen05 attention: maps over q / k / qkv and the compact sampled K/V
  // (filled only for phases whose worst-case length exceeds 2048).
  AttnMaps amaps;
  __half *kc = nullptr, *vc = nullptr;
  int rows_c = 0;
  bool gather[2] = {false, false};
  bool exact = false;  // exact-attention plan: no token merge, no key sampling
  // Batched projections (> 64 tokens): tcgen05 GEMM over the f16 weights
  // decoded at load (default: measured faster at every batched size here), or
  // the dequant-fused tcgen05 GEMM over the packed blocks (NEMO_BATCHED=fused
  // at plan creation).
  bool batched_f16 = true;
  int splits[kMaxLayers][4] = {};
  int rstages[kMaxLayers][4] = {};
  // Persistent single-launch forward (k_forward.cu) when the plan's worst case
  // fits kFwdNP tokens: grid size (0 = per-op kernels), its arguments and the
  // barrier / tile-counter block zeroed before each launch.
  int fgrid = 0;
  FwdArgs fargs = {};
  uint32_t* fsync = nullptr;
  size_t fsync_bytes = 0;
  // Test hooks, off unless NEMO_TEST_FAULTS is set when the plan is created:
  // a device word the single-launch forward reads for the grid barrier to
  // stall (NEMO_TEST_STALL_BARRIER, read at every run) and its pinned staging.
  uint32_t* test_stall = nullptr;
  uint32_t* h_test_stall = nullptr;
  cudaGraphExec_t graph_host = nullptr;    // H2D inputs -> forward -> D2H output
  cudaGraphExec_t graph_device = nullptr;  // forward only
  std::vector<void*> allocations;
  int run_batch = 0;
};

struct Profile;
struct Dump;
int enqueue_forward(DevicePlan& p, int n_layers, cudaStream_t s, Profile* prof, Dump* dump);
void rope_table_host(int sequence, float* table);

}  // namespace nemo

struct nemo_model {
  std::vector<std::unique_ptr<nemo::DeviceModel>> devs;
  int n_layers = 0;
  int vocab = 0;
  int compact = 0;
  int kquant = 0;
  uint64_t packed_bytes = 0;
};

namespace nemo {
// Head-parallel forward of one long request across a plan's devices (headpar.cu).
struct HeadPar;
int hp_create(nemo_plan* plan, HeadPar** out);
int hp_run(nemo_plan* plan, HeadPar* hp, const uint32_t* ids, int len, float* out);
void hp_destroy(HeadPar* hp);
}  // namespace nemo

struct nemo_plan {
  nemo_model* model = nullptr;
  int batch = 0, seq = 0;
  std::vector<std::unique_ptr<nemo::DevicePlan>> devs;
  // Multi-device plans of batch 1: requests of at least hp_min tokens run
  // head-parallel over all devices (peer memory); shorter ones run on one device.
  nemo::HeadPar* hp = nullptr;
  int hp_min = 0;
  bool exact = false;  // NEMO_PLAN_EXACT_ATTENTION
  // Host-side bound on every wait for a device's stream in nemo_plan_run
  // (NEMO_HOST_DEADLINE_MS at creation, default 60 s): past it the call
  // returns NEMO_ERR_TIMEOUT instead of blocking.
  int64_t host_deadline_ns = 60000000000ll;
  // Test hook (NEMO_TEST_FAIL_DEVICE at creation, -1 = off): the plan's device
  // with this index fails its share of every nemo_plan_run before launching
  // anything, so the whole micro-batch is rejected.
  int fail_device = -1;
};
