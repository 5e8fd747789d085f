// Launch wrappers for every device kernel of the encoder forward pass. Token
// rows are packed: the valid tokens of request 0, then request 1, ... (padding
// rows of the reference's [batch x sequence] layout are never computed).
#pragma once

#include "common.cuh"

namespace nemo {

// Per-run token bookkeeping, built on the device from the request lengths.
struct Meta {
  int batch;
  int seq;         // plan input sequence
  int merged_seq;  // contextualMergedLength(seq)
  int t0;          // valid tokens, layers 0..3
  int t1;          // valid tokens after the layer-4 merge
  int src_len[kMaxBatch];
  int tgt_len[kMaxBatch];
  int src_off[kMaxBatch + 1];
  int tgt_off[kMaxBatch + 1];
  // Rows of the compact sampled K/V buffer per request and phase (requests
  // whose valid length exceeds 2048 keep every third key, ops.ts:258-269).
  int samp_off[2][kMaxBatch + 1];
  // Exact-attention plans: no layer-4 merge (t1 = t0, tgt = src) and no
  // stride-3 key sampling.
  int exact;
};

constexpr int kSampleThreshold = 2048;
constexpr int kSampleStride = 3;

// Weight segment formats accepted by the decoders.
enum SegFormat { kSegQ4K = 0, kSegQ6K = 1, kSegQ40 = 2, kSegQ40Tile32 = 3 };

// Decodes `rows` rows of a [rows x k] quantised matrix to f16 (the effective
// weights f16(decode)) and, if out32 != nullptr, to exact f32 values.
cudaError_t launch_decode(int fmt, const uint8_t* src, int rows, int k, __half* out16, float* out32,
                          cudaStream_t s);

// model.ts:226-233 on the device: lengths -> Meta. `batch` is the capacity;
// when run_batch is non-null the run uses min(*run_batch, batch) requests.
cudaError_t launch_meta(const uint32_t* lengths, int batch, int seq, const uint32_t* run_batch, Meta* meta,
                        cudaStream_t s, int exact = 0);

// ops.ts:680-725. ids: [batch x seq] padded rows; output packed rows.
cudaError_t launch_embedding(const uint32_t* ids, const uint8_t* table, int vocab, const Meta* meta,
                             int max_tokens, __half* x, cudaStream_t s);

// ops.ts:21-72. rows = *d_rows (device int). residual may be null.
cudaError_t launch_residual_rmsnorm(__half* x, const __half* residual, const float* w, __half* norm,
                                    const int* d_rows, int max_rows, cudaStream_t s);
// The same after a persistent GEMM with GemmEpi::part: with one split
// (*d_splits, the GEMM's GemmEpi::splits_out) the residual is its f16
// output, else f16(sum of its f32 parts, in split order).
cudaError_t launch_residual_rmsnorm_parts(__half* x, const __half* residual, const float* part, const int* d_splits,
                                          const float* w, __half* norm, const int* d_rows, int max_rows,
                                          cudaStream_t s);

// ops.ts:168-194. merged selects the post-merge offsets for positions.
cudaError_t launch_rope(const __half* qkv, const float* table, const Meta* meta, bool merged,
                        int max_tokens, __half* q, __half* k, cudaStream_t s);
// Same for a head group: Q at columns [0, nq*128), K at [nq*128, (nq+nk)*128)
// of qkv rows qkv_ld wide; q out [T x nq x 128], k out [T x nk x 128].
cudaError_t launch_rope_group(const __half* qkv, int qkv_ld, int nq, int nk, const float* table, const Meta* meta,
                              bool merged, int max_tokens, __half* q, __half* k, cudaStream_t s);

// ops.ts:213-362. q [T x 24 x 128], k [T x 8 x 128], v read from qkv at column
// 4096 (row stride 5120); out [T x 3072].
cudaError_t launch_attention(const __half* q, const __half* k, const __half* qkv, const Meta* meta,
                             bool merged, int batch, int max_len, __half* out, cudaStream_t s);

// tcgen05 flash attention (k_attention_tc.cu). Tensor maps (box 64 x 128,
// 128B swizzle): q over Q [rows x 3072], k over K [rows x 1024], v over the
// QKV buffer [rows x 5120] (V at column 4096), kc/vc over the compact sampled
// K/V [rows_c x 1024] filled by launch_gather_sampled.
struct AttnMaps {
  CUtensorMap q, k, v, kc, vc;
};
cudaError_t launch_attention_tc(const AttnMaps& maps, const Meta* meta, bool merged, int batch, int max_len,
                                __half* out, uint32_t* err, cudaStream_t s);
cudaError_t launch_gather_sampled(const __half* k, const __half* qkv, const Meta* meta, bool merged, int max_rows,
                                  __half* kc, __half* vc, cudaStream_t s);
// Head-group variants (head-parallel attention): q_heads q heads with their
// q_heads/3 kv heads; V at column v_col0 of the v map's rows; out rows out_ld
// wide, or, with scatter (batch 1), row p stored at
// dst[p / rows_per_dev] + (p % rows_per_dev) * 3072 + col0 + head * 128: the
// attention buffer of the device owning the row (peer memory).
// Head-parallel routing over n devices (2, 4 or 8). Device j owns head group
// j: q heads j*24/n.. (QKV columns [j*3072/n, (j+1)*3072/n)) and kv heads
// j*8/n.. (K and V columns [j*1024/n, (j+1)*1024/n) after their offsets), so
// each GQA group of 3 q heads stays with its kv head. QKV column c goes to
// buffer *buf (0 Q, 1 K, 2 V) of device *dev at column *dcol (Q rows 3072/n
// wide, K and V rows 1024/n wide).
__host__ __device__ inline void hp_qkv_route(int c, int n, int* dev, int* buf, int* dcol) {
  const int gq = kQWidth / n, gk = kKVWidth / n;
  if (c < kQWidth) {
    *dev = c / gq, *buf = 0, *dcol = c - *dev * gq;
  } else if (c < kQWidth + kKVWidth) {
    c -= kQWidth;
    *dev = c / gk, *buf = 1, *dcol = c - *dev * gk;
  } else {
    c -= kQWidth + kKVWidth;
    *dev = c / gk, *buf = 2, *dcol = c - *dev * gk;
  }
}
// Token position pos of a request sharded in rows_per_dev-row shards (the last
// one shorter) belongs to this device.
__host__ __device__ inline int hp_row_owner(int pos, int rows_per_dev, int n) {
  const int o = pos / rows_per_dev;
  return o < n - 1 ? o : n - 1;
}

struct AttnScatter {
  __half* dst[8];
  int n_dev;
  int rows_per_dev;
  int col0;
};
cudaError_t launch_attention_tc_group(const AttnMaps& maps, const Meta* meta, bool merged, int batch, int max_len,
                                      int q_heads, int v_col0, int out_ld, __half* out, uint32_t* err,
                                      cudaStream_t s, const AttnScatter* scatter = nullptr);
cudaError_t launch_gather_sampled_group(const __half* k, const __half* qkv, int qkv_ld, int v_col0, int kv_w,
                                        const Meta* meta, bool merged, int max_rows, __half* kc, __half* vc,
                                        cudaStream_t s);

// ops.ts:74-89 over [rows x 12288] -> [rows x 6144].
cudaError_t launch_swiglu(const __half* gate_up, const int* d_rows, int max_rows, __half* out,
                          cudaStream_t s);

// ops.ts:629-661, applied to x and normalized in one launch.
cudaError_t launch_merge(const __half* x, const __half* norm, const Meta* meta, int max_out,
                         __half* xm, __half* nm, cudaStream_t s);

// ops.ts:596-616.
cudaError_t launch_mean_pool(const __half* norm, const Meta* meta, int batch, float* out,
                             cudaStream_t s);

// Plain CUDA-core f16 GEMM, f32 accumulate: Y[M x N] = X[M x K] . W[N x K]^T,
// M = *d_rows. A validation kernel for the tensor-core GEMM.
cudaError_t launch_gemm_simt(const __half* x, const __half* w, __half* y, float* y32,
                             const int* d_rows, int max_rows, int n, int k, cudaStream_t s);

// tcgen05 GEMM: A = activations via tensor map (box 64 x 128, 128B swizzle),
// B = f16 weights via tensor map (box 64 x bn). Y row-major [M x ldy] f16.
cudaError_t launch_gemm_tc(const CUtensorMap* map_a, const CUtensorMap* map_b, __half* y, int ldy,
                           const int* d_rows, int max_rows, int n, int k, int bn, uint32_t* err,
                           cudaStream_t s);
// Fused epilogues of the tcgen05 GEMM (mode: kSkinnyPlain, kSkinnyRope,
// kSkinnySwiglu). RoPE (QKV, n = 5120): Q and K columns are rotated by the
// table row of the token's position and written to q [T x 3072] and
// k [T x 1024]; V columns go to y. SwiGLU (gate/up, n = 12288, bn >= 128):
// map_b has a box of bn/2 rows; CTA x multiplies gate rows [x*bn/2, +bn/2) and
// the matching up rows and writes SwiGLU to y [T x ldy] at column x*bn/2.
struct GemmEpi {
  int mode = 0;
  const Meta* meta = nullptr;
  int merged = 0;
  const float* rope = nullptr;
  __half* q = nullptr;
  __half* k = nullptr;
  // Plain mode only: with part set, the K range is split gemm_ksplit(...)
  // ways and split s stores f32 partial sums at part[(s * M + row) * n + col]
  // (M = valid rows); launch_residual_rmsnorm_parts sums them in split order.
  // The split count used is stored at *splits_out (set with part).
  float* part = nullptr;
  int* splits_out = nullptr;
  // Head-parallel QKV (RoPE mode, hp.n_dev > 0): local row r is token position
  // hp.row0 + r of one request; each 32-column chunk is stored, Q and K
  // rotated, at that row of the Q, K or V buffer of the device owning its head
  // group (hp_qkv_route): peer memory over NVLink. With hp.sample set the K
  // and V of every third position also go to row pos / 3 of that device's
  // compact kc / vc buffers (the keys attention samples above 2048).
  struct {
    __half* q[8] = {};
    __half* k[8] = {};
    __half* v[8] = {};
    __half* kc[8] = {};
    __half* vc[8] = {};
    int n_dev = 0;
    int row0 = 0;
    int sample = 0;
  } hp;
};

// K splits of the persistent GEMM for m_tiles x n_tiles output tiles of kt
// 64-wide K steps on a grid of g CTAs. Fewer tiles than CTAs leave SMs idle
// for the whole launch (the O and down projections have 8 n tiles of 256),
// so the K range may then be split into up to 8 parts of >= 4 steps each.
// The split with the smallest modelled time wins, in thousandths of one
// full-K tile: waves of units, each 1/s of a tile plus 1/20 for its fill and
// drain, plus the consumer's reads of the f32 partial sums (one 2048-wide f32
// row per token and split, against a tile of kt steps). With a wave or more
// of tiles no split is taken: at 200-320 tiles (one 3200-5000-token request)
// splitting in two saved less in the GEMMs than the norms spent on partials.
// Host and device evaluate the same integers.
constexpr int kMaxKSplit = 8;  // most K splits gemm_ksplit picks
__host__ __device__ inline int gemm_ksplit(int m_tiles, int n_tiles, int kt, int g) {
  const int tiles = m_tiles * n_tiles;
  if (tiles <= 0 || g <= 0 || kt <= 0 || tiles >= g) return 1;
  int best = 1, best_cost = 0x7fffffff;
  for (int s = 1; s <= kMaxKSplit && kt / s >= 4; ++s) {
    const int waves = (tiles * s + g - 1) / g;
    const int cost = waves * (1000 / s + 50) + (s > 1 ? s * m_tiles * 355 / kt : 0);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}
cudaError_t launch_gemm_tc_epi(const CUtensorMap* map_a, const CUtensorMap* map_b, __half* y, int ldy,
                               const int* d_rows, int max_rows, int n, int k, int bn, const GemmEpi& ep,
                               uint32_t* err, cudaStream_t s);

// --- fused-dequant split-K projection for T <= 64 tokens (k_skinny.cu) -----
// Packed weights are re-tiled at load into 128-row tiles x 256-column slabs:
// chunk(tile, slab) at packed + tile.offset + slab * tile.chunk_bytes holds two
// 64-row regions (rows 0-63, 64-127), each in one format:
//   Q4_K : 64 x 144 B GGUF blocks
//   Q4_0 : 64 x [d[8] (16 B) | 8 x 16 quant bytes] (one 256 slab per row)
//   Q6_K : 64 x [ql 128 | qh 64 | scales 16] (208 B), then 64 x f16 d
struct SkinnyTile {
  uint32_t offset;
  uint32_t chunk_bytes;
  uint8_t fmt[2];
  uint8_t pad[6];
};

// kSkinnyF32: plain Y stored as f32 (the standalone quantised matmul entry
// point; `out` then points at floats and ldo counts floats).
enum SkinnyMode { kSkinnyPlain = 0, kSkinnyRope = 1, kSkinnySwiglu = 2, kSkinnyF32 = 3 };

struct SkinnyArgs {
  const uint8_t* packed;
  const SkinnyTile* tiles;
  uint32_t* err;
  const int* d_tokens;  // valid token rows (device int); null: `tokens` below
  int tokens;
  const Meta* meta;
  int merged;
  int n, slabs, splits, slabs_max, chunk_max;
  int rstages;  // weight ring depth, 2 or 3
  int mode;
  __half* out;  // plain: [T x ldo]; rope: qkv buffer (V columns); swiglu: [T x 6144]
  int ldo;
  __half* q;
  __half* k;
  const float* rope;
  int pdl;
};

size_t skinny_smem_bytes(int np, int slabs_max, int chunk_max, int rstages);
// Split-K factor and weight-ring depth of the small-T kernel for a projection
// of `tiles` 128-row tiles and `slabs` 256-column slabs (plan.cu).
void pick_splits(int tiles, int slabs, int np, int chunk_max, int* splits_out, int* rstages_out);
// Grid (tiles, splits), cluster (1, splits) with splits <= 16 and <= slabs;
// np = tokens padded to 16, 32 or 64; map_x box 64 x np.
cudaError_t launch_skinny(const CUtensorMap* map_x, const SkinnyArgs& a, int np, int tiles, cudaStream_t s);

// --- dequant-fused batched projection GEMM (k_gemm_q.cu) --------------------
// Y[M x 128 * n_tiles] = X . W^T with W decoded from the tile-slab image in
// shared memory; map_x box 64 x 128 (128B swizzle). mode kSkinnyPlain stores
// f16 rows (ldy wide); kSkinnySwiglu applies SwiGLU to each tile's interleaved
// gate/up rows and stores 64 columns per tile ([M x 6144]).
cudaError_t launch_gemm_q(const CUtensorMap* map_x, const uint8_t* packed, const SkinnyTile* tiles, int n_tiles,
                          int slabs, int chunk_max, int mode, __half* y, int ldy, const int* d_rows, int max_rows,
                          uint32_t* err, cudaStream_t s);

// --- standalone quantised matmul (qmatmul.cu) ------------------------------
// Bytes of the device tile-slab image of an [n x k] matrix (0 if n is not a
// multiple of 128 or k of 256), the device re-tile of GGUF / tile32 blocks into
// it, and Y[m x n] f32 = X[m x k] . W^T on the image (small-token kernel for
// m <= 64, dequant-fused GEMM above). err: device word for bounded waits.
size_t qmatmul_image_bytes(int fmt, int n, int k);
cudaError_t launch_qmatmul_retile(int fmt, const uint8_t* src, int n, int k, uint8_t* image, cudaStream_t s);
cudaError_t launch_qmatmul_image_decode(int fmt, const uint8_t* image, int n, int k, __half* w16, cudaStream_t s);
int qmatmul_enqueue(int fmt, const uint8_t* image, const __half* x, int m, int n, int k, float* y, uint32_t* err,
                    cudaStream_t s);

// Exact decode of a whole tile-slab image (device chunks + device tile table)
// to the row-major f16 matrix [n x k]; interleave: gate/up tiles (qmatmul.cu).
cudaError_t launch_decode_image(const uint8_t* chunks, const SkinnyTile* tiles, int ntiles, int slabs, bool interleave,
                                int n, int k, __half* w16, cudaStream_t s);

// --- persistent single-launch forward for <= kFwdNP tokens (k_forward.cu) ---
constexpr int kFwdNP = 16;        // token rows per projection (padded)
constexpr int kFwdMaxTiles = 96;  // 128-row tiles of the widest projection (gate/up)

// One CTA's share of one projection: a tile and a range of 256-column slabs,
// with the tile's location in the projection's tile-slab image.
struct FwdSeg {
  const uint8_t* chunk0;  // chunk (tile, slab 0); slab s at chunk0 + s * chunk_bytes
  uint32_t chunk_bytes;
  uint16_t proj;          // layer * 4 + projection (QKV, O, gate/up, down)
  uint16_t tile;
  uint8_t s0, s1;         // slabs [s0, s1)
  uint8_t slot;           // partial-sum slot within the tile (slots follow K order)
  uint8_t fmt[2];         // SegFormat of the tile's two 64-row regions
  uint8_t pad[3];
};

struct FwdArgs {
  // Activation tensor maps, box 64 x kFwdNP, 128B swizzle: normalised state
  // before / after the merge, attention output, SwiGLU output.
  CUtensorMap xmap[4];
  const int* sstride;       // [n_layers * 4] partial-slot stride (largest slot count of the projection's tiles)
  const FwdSeg* segs;       // per-CTA lists in forward order, concatenated
  const int* seg_start;     // [grid + 1]
  const uint8_t* nslots;    // [n_layers * 4][kFwdMaxTiles]
  const uint8_t* small_rank;  // [n_layers * 3][grid]: a CTA's place in the attention, post-attention
                              // norm and post-FFN norm item lists of each layer (least next-projection
                              // work first, so the CTAs that pause their decoders for these phases
                              // have the least weight work right after them)
  uint32_t* sync;           // [0] grid barrier, [1 + proj * kFwdMaxTiles + tile] tile counters; zero at launch
  uint32_t* err;
  const uint32_t* ids;      // [batch x seq]
  const uint8_t* embd;
  int vocab;
  const float* attn_norm[kMaxLayers];
  const float* ffn_norm[kMaxLayers];
  const float* output_norm;
  const Meta* meta;
  const float* rope;
  int rope_rows;            // positions in the RoPE table (the plan's sequence, <= kFwdNP here)
  __half *x, *nrm, *xm, *nm, *qkv, *q, *k, *attn, *delta, *ffn;
  float* part;              // [tile][kFwdNP tokens][sstride slots][128] f32 per projection
  int max_slots;             // most split-K slots of any tile (sizes `part`)
  int scratch_slots;         // 8 KB units of shared scratch after the X ring: the gate/up
                             // epilogue's slots and the norm phase's O/down staging
  int max_segs;             // most segments any CTA owns
  float* out;               // [batch x 2048]
  int n_layers;
  int chunk_max;
  int exact;                // no merge, pool over the unmerged rows
  uint64_t wait_ns;          // bound of every wait in the kernel (2 s; tests shorten it)
  const uint32_t* test_stall;  // test hook (null in normal plans): grid barrier number
                               // *test_stall (1-based, 0 = none) can never complete
};

size_t forward_smem_bytes(int chunk_max, int scratch_slots, int max_segs, int n_layers);
// Shared scratch (8 KB units) that the forward needs beyond its X ring, given
// the most slots of a gate/up tile and of an O or down tile.
int forward_scratch_slots(int gate_up_slots, int residual_slots);

// Largest co-resident grid (one CTA per SM) or 0 if the kernel does not fit.
cudaError_t forward_max_grid(size_t smem_bytes, int* grid);
cudaError_t launch_forward(const FwdArgs& a, int grid, cudaStream_t s);

// Host: encodes a 2-D f16 tensor map over a row-major [outer x inner] array
// with a (box_inner x box_outer) box and 128-byte swizzle.
int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                  uint32_t box_inner, uint32_t box_outer);

}  // namespace nemo
