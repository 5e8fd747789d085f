// Bidirectional GQA flash attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), the B200 counterpart of the reference's attention
// pipelines (src/webgpu/ops.ts:213-293 tiled flash, :295-362 small).
//
// Semantics kept from the reference: each query of request b attends to the
// request's valid keys of this layer; when that valid length exceeds 2048 only
// every third key (positions 0, 3, 6, ...) is used (ops.ts:258-269) -- those
// keys are gathered into a compact buffer first; queries at positions >= 16384
// get the temperature factor of ops.ts:241; scale 1/sqrt(128); GQA q_head/3.
// Scores and the softmax statistics are f32, P is rounded to f16 for the P.V
// product (the reference keeps P in f16 as well), O accumulates in f32.
//
// One CTA = two tiles of 128 queries (256) of one q head of one request, which
// share every K/V tile (320 threads):
//   warp 0      TMA producer: the two Q tiles once, then K and V tiles of 128
//               keys (double-buffered ring); V comes straight out of the QKV
//               projection buffer and is consumed MN-major
//   warp 1      TMEM allocation (512 columns: S_0, S_1, O_0, O_1, 128 each) and
//               tcgen05.mma issue (elected lane): S_t = Q_t.K_j^T, then
//               O_t += P_t.V_j with P_t read from TMEM (A operand in tensor
//               memory), interleaved over the two tiles so the tensor pipe
//               works on one tile while the other tile's softmax runs
//   warps 2..5  softmax of tile 0, warps 6..9 of tile 1 (thread = query row):
//               tcgen05.ld of the S row, online max/sum, P (f16) written back
//               over its own S columns, O rows rescaled in TMEM when the running
//               max moves (it moves only by more than 2^8); final O / l to global.
// All mbarrier waits are bounded; on a timeout every role unwinds and TMEM is
// released only after the CTA's MMAs have retired.
#include "kernels.cuh"

namespace nemo {
namespace {

constexpr int kTile = 128;
constexpr int kHalfTile = kTile * 64 * 2;  // 128 rows x 64 f16 = 16 KB (one 128B-swizzle column block)
constexpr int kTileBytes = 2 * kHalfTile;  // 128 x 128 f16
// Two shapes of the kernel: NT query tiles per CTA sharing every K/V tile,
// KVS K/V stages. <2, 2> (320 threads, 512 TMEM columns, ~197 KB) for long
// requests; <1, 1> (192 threads, 256 TMEM columns, ~97 KB, two CTAs per SM)
// for plans of short requests, whose one or two key tiles leave nothing to
// pipeline and whose CTAs are mostly set-up: a second resident CTA overlaps it.
template <int NT, int KVS>
struct AttnCfg {
  static constexpr int kThreads = 64 + 128 * NT;
  static constexpr int kSmem = 1024 + NT * kTileBytes /*Q*/ + KVS * kTileBytes /*K*/ + KVS * kTileBytes /*V*/ + 256;
  static constexpr uint32_t kTmemCols = 256 * NT;
  static constexpr uint32_t kColS = 0, kColO = 128 * NT;  // S_t at kColS + 128 t, O_t at kColO + 128 t
};
constexpr int kShortAttentionMaxLen = 256;  // plans up to this many rows use AttnCfg<1, 1>
constexpr float kMaxSlack = 8.0f;           // running-max hysteresis (log2 units): P <= 256

__device__ __forceinline__ uint32_t pack_h2f(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AttnTcArgs {
  const Meta* meta;
  int merged;
  __half* out;
  uint32_t* err;
  int v_col0;  // column of the head group's V in the rows of the v map
  int out_ld;  // output row stride (q heads of the group x 128)
  AttnScatter scatter;  // scatter.dst[0] set: rows go to the devices that own them
};

template <int NT, int KVS>
__global__ void __launch_bounds__(AttnCfg<NT, KVS>::kThreads, NT == 1 ? 2 : 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_kc,
                        const __grid_constant__ CUtensorMap map_vc, AttnTcArgs a) {
  using C = AttnCfg<NT, KVS>;
  constexpr uint32_t kColS = C::kColS, kColO = C::kColO;
  extern __shared__ uint8_t smem_raw[];
  dev::pdl_launch_dependents();
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * NT * kTile;
  const Meta* meta = a.meta;
  if (b >= meta->batch) return;
  const int ph = a.merged ? 1 : 0;
  const int len = a.merged ? meta->tgt_len[b] : meta->src_len[b];
  if (q0 >= len) return;  // uniform over the CTA
  const int nqt = NT == 2 && q0 + kTile < len ? 2 : 1;  // query tiles with valid rows
  const int base = a.merged ? meta->tgt_off[b] : meta->src_off[b];
  const int kvh = h / (kQHeads / kKVHeads);
  const bool sampled = !meta->exact && len > kSampleThreshold;
  const int nkeys = sampled ? (len + kSampleStride - 1) / kSampleStride : len;
  const int kbase = sampled ? meta->samp_off[ph][b] : base;
  const CUtensorMap* km = sampled ? &map_kc : &map_k;
  const CUtensorMap* vm = sampled ? &map_vc : &map_v;
  const int kcol = kvh * kHeadDim;
  const int vcol = sampled ? kvh * kHeadDim : a.v_col0 + kvh * kHeadDim;
  const int ntiles = (nkeys + kTile - 1) / kTile;

  const uint32_t raw_s = dev::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  uint8_t* sQ = smem;                    // Q_0 (, Q_1)
  uint8_t* sK = sQ + NT * kTileBytes;
  uint8_t* sV = sK + KVS * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KVS * kTileBytes);
  const uint32_t q_full = dev::smem_u32(bars);
  const uint32_t kv_full = q_full + 8, kv_empty = kv_full + 16;
  const uint32_t s_full = kv_empty + 16, p_ready = s_full + 16, pv_done = p_ready + 16;
  const uint32_t mma_fin = pv_done + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&map_q);
    dev::prefetch_tmap(km);
    dev::prefetch_tmap(vm);
    dev::mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(kv_full + 8 * s, 1);
      dev::mbar_init(kv_empty + 8 * s, 1);
      dev::mbar_init(s_full + 8 * s, 1);
      dev::mbar_init(p_ready + 8 * s, 128);
      dev::mbar_init(pv_done + 8 * s, 1);
    }
    dev::mbar_init(mma_fin, 1);
    dev::fence_mbar_init();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), C::kTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // Converged warp; the elected lane issues the copies.
    dev::pdl_wait();
    if (dev::elect_one()) {
      dev::mbar_arrive_expect_tx(q_full, nqt * kTileBytes);
      for (int t = 0; t < nqt; ++t) {
        dev::tma_load_2d(dev::smem_u32(sQ + t * kTileBytes), &map_q, h * kHeadDim, base + q0 + t * kTile, q_full);
        dev::tma_load_2d(dev::smem_u32(sQ + t * kTileBytes + kHalfTile), &map_q, h * kHeadDim + 64,
                         base + q0 + t * kTile, q_full);
      }
    }
    __syncwarp();
    int issued = 0;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % KVS;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(kv_empty + 8 * st, ((j / KVS) & 1) ^ 1, a.err))) break;
      const uint32_t fb = kv_full + 8 * st;
      const uint32_t dk = dev::smem_u32(sK + st * kTileBytes), dv = dev::smem_u32(sV + st * kTileBytes);
      const int row = kbase + j * kTile;
      if (dev::elect_one()) {
        dev::mbar_arrive_expect_tx(fb, 2 * kTileBytes);
        dev::tma_load_2d(dk, km, kcol, row, fb);
        dev::tma_load_2d(dk + kHalfTile, km, kcol + 64, row, fb);
        dev::tma_load_2d(dv, vm, vcol, row, fb);
        dev::tma_load_2d(dv + kHalfTile, vm, vcol + 64, row, fb);
      }
      __syncwarp();
      ++issued;
    }
    dev::mbar_wait(q_full, 0, a.err, 100000000ull);
    for (int i = issued > KVS ? issued - KVS : 0; i < issued; ++i)
      dev::mbar_wait(kv_full + 8 * (i % KVS), (i / KVS) & 1, a.err, 100000000ull);
  } else if (warp == 1) {
    // Converged warp; the elected lane (lane 0) issues every MMA and commit.
    // Order per key tile j and query tile t: PV_t(j-1) (reads P_t from the
    // S_t columns) strictly before S_t(j) (overwrites them); the tensor pipe
    // runs them in issue order.
    const uint32_t idesc_s = dev::make_idesc_f16(kTile, kTile);                  // Q.K^T, both K-major
    const uint32_t idesc_o = dev::make_idesc_f16(kTile, kHeadDim) | (1u << 16);  // P.V, V MN-major
    bool ok = __all_sync(0xffffffffu, dev::mbar_wait(q_full, 0, a.err));
    auto pv = [&](int t, int jj) -> bool {  // O_t += P_t(jj) . V(jj)
      if (!__all_sync(0xffffffffu, dev::mbar_wait(p_ready + 8 * t, jj & 1, a.err))) return false;
      dev::tc_fence_after();
      const uint32_t bv = dev::smem_u32(sV + (jj % KVS) * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        if (dev::elect_one()) {
          const uint64_t bd = dev::make_sw128_desc_mn(bv + kk * 2048, kHalfTile, 1024);
          dev::tc_mma_f16_ts(tmem + kColO + t * kTile, tmem + kColS + t * kTile + kk * 8, bd, idesc_o,
                             (jj | kk) != 0 ? 1u : 0u);
        }
        __syncwarp();
      }
      if (dev::elect_one()) dev::tc_commit(pv_done + 8 * t);
      __syncwarp();
      return true;
    };
    auto qk = [&](int t, int j) {  // S_t = Q_t . K(j)^T
      const uint32_t aq = dev::smem_u32(sQ + t * kTileBytes);
      const uint32_t bk = dev::smem_u32(sK + (j % KVS) * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kHeadDim / 16; ++kk) {
        if (dev::elect_one()) {
          const uint64_t ad = dev::make_sw128_desc(aq + (kk >> 2) * kHalfTile + (kk & 3) * 32);
          const uint64_t bd = dev::make_sw128_desc(bk + (kk >> 2) * kHalfTile + (kk & 3) * 32);
          dev::tc_mma_f16(tmem + kColS + t * kTile, ad, bd, idesc_s, kk != 0 ? 1u : 0u);
        }
        __syncwarp();
      }
      if (dev::elect_one()) dev::tc_commit(s_full + 8 * t);
      __syncwarp();
    };
    if (KVS == 1) {
      // One K/V stage: K/V tile j + 1 is loaded only after P.V(j) has read
      // V(j), so each key tile runs S, softmax, P.V in turn.
      for (int j = 0; j < ntiles && ok; ++j) {
        if (!__all_sync(0xffffffffu, dev::mbar_wait(kv_full, j & 1, a.err))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        for (int t = 0; t < nqt; ++t) qk(t, j);
        for (int t = 0; t < nqt && ok; ++t) ok = pv(t, j);
        // every MMA that reads the key/value stage has been issued
        if (ok && dev::elect_one()) dev::tc_commit(kv_empty);
        __syncwarp();
      }
    } else {
      for (int j = 0; j < ntiles && ok; ++j) {
        if (!__all_sync(0xffffffffu, dev::mbar_wait(kv_full + 8 * (j % KVS), (j / KVS) & 1, a.err))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        for (int t = 0; t < nqt && ok; ++t) {
          if (j > 0) ok = pv(t, j - 1);
          if (ok) qk(t, j);
        }
        // every MMA that reads key/value stage j - 1 has been issued
        if (ok && j > 0 && dev::elect_one()) dev::tc_commit(kv_empty + 8 * ((j - 1) % KVS));
        __syncwarp();
      }
      for (int t = 0; t < nqt && ok; ++t) ok = pv(t, ntiles - 1);
    }
    if (dev::elect_one()) dev::tc_commit(mma_fin);
    __syncwarp();
    dev::mbar_wait(mma_fin, 0, a.err, 100000000ull);  // every MMA retired before TMEM is freed
  } else {
    // ---- softmax warps: tile t, thread = query row (TMEM lane) ----
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t colS = kColS + t * kTile, colO = kColO + t * kTile;
    const int pos = q0 + t * kTile + row;
    const float temp = pos >= 16384 ? logf(floorf((float)pos / 16384.0f) + 1.0f) * 0.1f + 1.0f : 1.0f;
    // exp(x) = 2^(x log2 e): scores are kept in log2 units
    const float scale = 0.08838834764831845f * temp * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    bool ok = t < nqt;  // uniform over the warp
    for (int j = 0; j < ntiles && ok; ++j) {
      // warp-uniform outcome: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, dev::mbar_wait(s_full + 8 * t, j & 1, a.err))) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      const int valid = min(kTile, nkeys - j * kTile);
      // The S row: its four 32-column loads in flight before one wait; keys
      // past the valid ones (only on a partial last tile) masked to -inf.
      // (A macro, not a lambda: s must stay in registers.)
#define NEMO_LOAD_S_ROW()                                                                                  \
  do {                                                                                                     \
    _Pragma("unroll") for (int c = 0; c < 4; ++c)                                                          \
        dev::tmem_ld_32x32b_x32(lane_base + colS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32])); \
    dev::tc_wait_ld();                                                                                     \
    if (valid < kTile) {                                                                                   \
      _Pragma("unroll") for (int i = 0; i < kTile; ++i) s[i] = i < valid ? s[i] : -INFINITY;               \
    }                                                                                                      \
  } while (0)
      float s[kTile];
      NEMO_LOAD_S_ROW();
      // The running max of the warp's rows moves only when some row's tile
      // max exceeds it by more than kMaxSlack (log2 units). Otherwise P is
      // taken against the stale max: P <= 2^kMaxSlack, well inside f16, and
      // O / l is unchanged, while the O rows need no rescale on that tile.
      // (With the exact running max nearly every tile moves some row's max.)
      // From the second tile on the exponentials are computed against the
      // running max straight after the load, the tile max (of the raw scores,
      // scaled once: scale > 0 keeps the order) beside them; only when the max
      // moves is the row reloaded from TMEM (P has not overwritten it yet) and
      // recomputed against the new max. On the first tile the max always moves.
      // p = 2^(s * scale - m): one FMA per score on the raw value.
      float tmax = -INFINITY, rs0 = 0.f, rs1 = 0.f;  // two independent sum chains
      bool move = true;
      if (j > 0) {
        const float nm = -m;
#pragma unroll
        for (int i = 0; i < kTile; i += 2) {
          tmax = fmaxf(tmax, fmaxf(s[i], s[i + 1]));
          s[i] = ex2(fmaf(s[i], scale, nm));
          s[i + 1] = ex2(fmaf(s[i + 1], scale, nm));
          rs0 += s[i];
          rs1 += s[i + 1];
        }
        tmax *= scale;
        move = __any_sync(0xffffffffu, tmax > m + kMaxSlack);
      } else {
#pragma unroll
        for (int i = 0; i < kTile; ++i) tmax = fmaxf(tmax, s[i]);
        tmax *= scale;
      }
      const float mnew = move ? fmaxf(m, tmax) : m;
      if (move) {
        if (j > 0) NEMO_LOAD_S_ROW();
        const float nm = -mnew;
        rs0 = rs1 = 0.f;
#pragma unroll
        for (int i = 0; i < kTile; i += 2) {
          s[i] = ex2(fmaf(s[i], scale, nm));
          s[i + 1] = ex2(fmaf(s[i + 1], scale, nm));
          rs0 += s[i];
          rs1 += s[i + 1];
        }
      }
#undef NEMO_LOAD_S_ROW
      const float rsum = rs0 + rs1;
      const float alpha = ex2(m - mnew);  // 0 on the first tile, 1 while the max stays
      // P_t (f16) over its own S columns: S_t(j) has been read, and neither
      // PV_t(j) nor S_t(j + 1) is issued before p_ready
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pr[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i] = pack_h2f(s[c * 64 + 2 * i], s[c * 64 + 2 * i + 1]);
        dev::tmem_st_32x32b_x32(lane_base + colS + c * 32, pr);
      }
      if (j > 0) {
        // PV_t(j - 1) complete: O_t is stable
        if (!__all_sync(0xffffffffu, dev::mbar_wait(pv_done + 8 * t, (j - 1) & 1, a.err))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        if (move) {
          uint32_t orow[kHeadDim];  // all four loads in flight before one wait
#pragma unroll
          for (int c = 0; c < 4; ++c)
            dev::tmem_ld_32x32b_x32(lane_base + colO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&orow[c * 32]));
          dev::tc_wait_ld();
#pragma unroll
          for (int i = 0; i < kHeadDim; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            dev::tmem_st_32x32b_x32(lane_base + colO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&orow[c * 32]));
        }
      }
      dev::tc_wait_st();
      l = l * alpha + rsum;
      m = mnew;
      dev::tc_fence_before();
      dev::mbar_arrive(p_ready + 8 * t);
    }
    if (ok && __all_sync(0xffffffffu, dev::mbar_wait(pv_done + 8 * t, (ntiles - 1) & 1, a.err))) {
      dev::tc_fence_after();
      const float inv = 1.0f / l;
      auto out_unit = [&](const uint32_t (&r)[32], int v) {
        return make_uint4(pack_h2f(__uint_as_float(r[v * 8]) * inv, __uint_as_float(r[v * 8 + 1]) * inv),
                          pack_h2f(__uint_as_float(r[v * 8 + 2]) * inv, __uint_as_float(r[v * 8 + 3]) * inv),
                          pack_h2f(__uint_as_float(r[v * 8 + 4]) * inv, __uint_as_float(r[v * 8 + 5]) * inv),
                          pack_h2f(__uint_as_float(r[v * 8 + 6]) * inv, __uint_as_float(r[v * 8 + 7]) * inv));
      };
      if (a.scatter.dst[0]) {
        // Head-parallel: each output row goes to the attention buffer of the
        // device owning the row's token shard (peer memory over NVLink), at
        // this head group's columns. The warp stages its 32 rows x 128
        // columns in its quarter of the Q_t tile (every MMA reading Q_t has
        // retired) and writes each row as one 256-byte segment, 16 lanes per
        // row; 16-byte unit u of row i sits at unit u ^ (i & 7).
        uint8_t* stage = sQ + t * kTileBytes + quarter * (32 * 256);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          dev::tmem_ld_32x32b_x32(lane_base + colO + c * 32, r);
          dev::tc_wait_ld();
#pragma unroll
          for (int v = 0; v < 4; ++v)
            *reinterpret_cast<uint4*>(stage + lane * 256 + (((c * 4 + v) ^ (lane & 7)) * 16)) = out_unit(r, v);
        }
        __syncwarp();
        const int u = lane & 15;
#pragma unroll 4
        for (int it = 0; it < 16; ++it) {
          const int rr = it * 2 + (lane >> 4);
          const int p = q0 + t * kTile + quarter * 32 + rr;
          if (p < len) {
            const int owner = hp_row_owner(p, a.scatter.rows_per_dev, a.scatter.n_dev);
            __half* buf = a.scatter.dst[0];
#pragma unroll
            for (int i = 1; i < 8; ++i) buf = owner == i ? a.scatter.dst[i] : buf;  // selects, no local copy
            *reinterpret_cast<uint4*>(buf + (size_t)(p - owner * a.scatter.rows_per_dev) * kQWidth +
                                      a.scatter.col0 + h * kHeadDim + u * 8) =
                *reinterpret_cast<const uint4*>(stage + rr * 256 + ((u ^ (rr & 7)) * 16));
          }
        }
      } else {
        __half* dst = a.out + (size_t)(base + pos) * a.out_ld + h * kHeadDim;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          dev::tmem_ld_32x32b_x32(lane_base + colO + c * 32, r);
          dev::tc_wait_ld();
          if (pos < len) {
#pragma unroll
            for (int v = 0; v < 4; ++v) reinterpret_cast<uint4*>(dst + c * 32)[v] = out_unit(r, v);
          }
        }
      }
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Gathers every third key of the requests whose valid length exceeds 2048
// into compact K/V buffers (one block per compact row, 8 columns per thread).
// kv_w = KV heads of the group x 128; k rows are kv_w wide, V sits at column
// v_col0 of qkv rows qkv_ld wide.
__global__ void __launch_bounds__(128) gather_sampled_kernel(const __half* __restrict__ k,
                                                            const __half* __restrict__ qkv,
                                                            const Meta* __restrict__ meta, int merged,
                                                            __half* kc, __half* vc, int kv_w, int qkv_ld,
                                                            int v_col0) {
  const int ph = merged ? 1 : 0;
  const int row = blockIdx.x;
  if (row >= meta->samp_off[ph][meta->batch]) return;
  int b = 0;
  while (b + 1 < meta->batch && row >= meta->samp_off[ph][b + 1]) ++b;
  const int base = merged ? meta->tgt_off[b] : meta->src_off[b];
  const size_t src = (size_t)base + (size_t)(row - meta->samp_off[ph][b]) * kSampleStride;
  const int c = threadIdx.x * 8;
  if (c >= kv_w) return;
  *reinterpret_cast<uint4*>(kc + (size_t)row * kv_w + c) = *reinterpret_cast<const uint4*>(k + src * kv_w + c);
  *reinterpret_cast<uint4*>(vc + (size_t)row * kv_w + c) =
      *reinterpret_cast<const uint4*>(qkv + src * qkv_ld + v_col0 + c);
}

}  // namespace

cudaError_t launch_gather_sampled(const __half* k, const __half* qkv, const Meta* meta, bool merged, int max_rows,
                                  __half* kc, __half* vc, cudaStream_t s) {
  return launch_gather_sampled_group(k, qkv, kQKVWidth, kQWidth + kKVWidth, kKVWidth, meta, merged, max_rows, kc, vc,
                                     s);
}

cudaError_t launch_gather_sampled_group(const __half* k, const __half* qkv, int qkv_ld, int v_col0, int kv_w,
                                        const Meta* meta, bool merged, int max_rows, __half* kc, __half* vc,
                                        cudaStream_t s) {
  if (max_rows <= 0) return cudaSuccess;
  if (kv_w % 8 || kv_w > 1024 || v_col0 % 8 || qkv_ld % 8) return cudaErrorInvalidValue;
  gather_sampled_kernel<<<max_rows, 128, 0, s>>>(k, qkv, meta, merged ? 1 : 0, kc, vc, kv_w, qkv_ld, v_col0);
  return cudaGetLastError();
}

cudaError_t launch_attention_tc(const AttnMaps& maps, const Meta* meta, bool merged, int batch, int max_len,
                                __half* out, uint32_t* err, cudaStream_t s) {
  return launch_attention_tc_group(maps, meta, merged, batch, max_len, kQHeads, kQWidth + kKVWidth, kQWidth, out, err,
                                   s, nullptr);
}

cudaError_t launch_attention_tc_group(const AttnMaps& maps, const Meta* meta, bool merged, int batch, int max_len,
                                      int q_heads, int v_col0, int out_ld, __half* out, uint32_t* err,
                                      cudaStream_t s, const AttnScatter* scatter) {
  if (max_len <= 0 || batch <= 0) return cudaSuccess;
  if (q_heads <= 0 || q_heads % (kQHeads / kKVHeads) || v_col0 % 8 || out_ld % 8) return cudaErrorInvalidValue;
  if (scatter && (batch != 1 || scatter->n_dev < 1 || scatter->n_dev > 8 || scatter->rows_per_dev < 1 ||
                  scatter->col0 % 8 || !scatter->dst[0]))
    return cudaErrorInvalidValue;
  static bool configured[64][2] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64) return cudaErrorInvalidDevice;
  // NEMO_ATTENTION_SHORT_MAX overrides the row bound of the short shape
  static const int short_max = [] {
    const char* v = getenv("NEMO_ATTENTION_SHORT_MAX");
    return v && *v ? atoi(v) : kShortAttentionMaxLen;
  }();
  const bool shrt = max_len <= short_max;
  if (!configured[dev][shrt]) {
    e = shrt ? cudaFuncSetAttribute(attention_tc_kernel<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    AttnCfg<1, 1>::kSmem)
             : cudaFuncSetAttribute(attention_tc_kernel<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    AttnCfg<2, 2>::kSmem);
    if (e != cudaSuccess) return e;
    configured[dev][shrt] = true;
  }
  AttnTcArgs a{meta, merged ? 1 : 0, out, err, v_col0, out_ld, {}};
  if (scatter) a.scatter = *scatter;
  if (shrt) {
    dim3 grid((max_len + kTile - 1) / kTile, q_heads, batch);
    attention_tc_kernel<1, 1><<<grid, AttnCfg<1, 1>::kThreads, AttnCfg<1, 1>::kSmem, s>>>(maps.q, maps.k, maps.v,
                                                                                        maps.kc, maps.vc, a);
  } else {
    dim3 grid((max_len + 2 * kTile - 1) / (2 * kTile), q_heads, batch);
    attention_tc_kernel<2, 2><<<grid, AttnCfg<2, 2>::kThreads, AttnCfg<2, 2>::kSmem, s>>>(maps.q, maps.k, maps.v,
                                                                                        maps.kc, maps.vc, a);
  }
  return cudaGetLastError();
}

}  // namespace nemo
