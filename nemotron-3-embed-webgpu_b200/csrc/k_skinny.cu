// Fused-dequant projection GEMM for small token counts (T <= 64), the
// batch-1 regime of the reference's latency/subgroup matmul pipelines
// (src/webgpu/quant-matmul.ts:156-223,379-423, dispatched per
// src/webgpu/model.ts:313-320). Here the projection is weight-bandwidth bound,
// so the kernel streams the quantised bytes once and dequantises them on chip:
//
//   D[128 weight rows x NP tokens] += W_tile[128 x 16] . X^T[16 x NP]   (tcgen05, f16 in, f32 in TMEM)
//
// One CTA = one 128-row tile x one K range (split-K over the grid's y axis).
//   warp 0      producer: starts streaming its packed weight chunks (one
//               128-row x 256-column chunk per ring stage, cp.async.bulk)
//               before waiting on the previous kernel, then TMA-loads the
//               activation K range (box 64 x NP, 128B swizzle)
//   warp 1      TMEM allocation + tcgen05.mma issue (elected lane)
//   warps 2..9  decoders (thread = weight row): exact decode of the block
//               with the reference's arithmetic (quantization.ts:19-74; every
//               intermediate is exact or rounded once, as there), f16 round to
//               nearest, written in the canonical 128B-swizzled K-major layout.
//               Warps 2-5 decode the even 64-column quarters of each slab into
//               A stage 0, warps 6-9 the odd ones into stage 1, so two quarters
//               are decoded at once; warps 2-5 then move TMEM -> this CTA's
//               partial tile in shared memory.
// The split-K CTAs of one tile are one thread-block cluster: after a cluster
// barrier each CTA reduces a slice of the tile's rows from its peers' shared
// memory (DSMEM), summing the splits in rank order (deterministic), and applies
// the fused epilogue (plain f16 store, RoPE + Q/K/V split, or SwiGLU).
// All mbarrier waits are bounded (see common.cuh); every thread reaches both
// cluster barriers on every path. Shared memory is sized per projection so
// two CTAs share an SM when they fit.
#include "tile_decode.cuh"

namespace nemo {
namespace {

constexpr int kMaxRawStages = 3;
constexpr int kAStages = 2;
constexpr int kABytes = 128 * 128;  // 128 rows x 64 f16
constexpr int kMaxSplits = 16;
constexpr int kThreads = 320;  // producer, MMA issuer, two groups of four decoder warps

using namespace tsd;

template <int NP>
__global__ void __launch_bounds__(kThreads, 2)
    skinny_kernel(const __grid_constant__ CUtensorMap map_x, SkinnyArgs a) {
  extern __shared__ uint8_t smem_raw[];
  dev::pdl_launch_dependents();
  const uint32_t raw_s = dev::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  const int tile = blockIdx.x, split = blockIdx.y;
  const int RS = a.rstages;
  const int slab0 = split * a.slabs / a.splits, slab1 = (split + 1) * a.slabs / a.splits;
  const int nsl = slab1 - slab0;
  const int kr = nsl * 256;
  // shared layout: X [kr/64][NP rows x 128 B] | raw ring | A ring | barriers
  uint8_t* xs = smem;
  uint8_t* raw = xs + (size_t)(a.slabs_max * 4) * NP * 128;
  uint8_t* as = raw + ((RS * a.chunk_max + 1023) & ~1023);  // A tiles 1024-aligned (SW128)
  uint64_t* bars = reinterpret_cast<uint64_t*>(as + kAStages * kABytes);
  const uint32_t xfull = dev::smem_u32(bars);
  const uint32_t rfull = xfull + 8, rempty = rfull + 8 * kMaxRawStages;
  const uint32_t afull = rempty + 8 * kMaxRawStages, aempty = afull + 8 * kAStages;
  const uint32_t accum = aempty + 8 * kAStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 + 2 * kMaxRawStages + 2 * kAStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = NP < 32 ? 32 : NP;
  const SkinnyTile ti = a.tiles[tile];

  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&map_x);
    dev::mbar_init(xfull, 1);
    for (int s = 0; s < kMaxRawStages; ++s) {
      dev::mbar_init(rfull + 8 * s, 1);
      dev::mbar_init(rempty + 8 * s, 256);
    }
    for (int s = 0; s < kAStages; ++s) {
      dev::mbar_init(afull + 8 * s, 128);
      dev::mbar_init(aempty + 8 * s, 1);
    }
    dev::mbar_init(accum, 1);
    dev::fence_mbar_init();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), kTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint8_t* chunk0 = a.packed + ti.offset + (size_t)slab0 * ti.chunk_bytes;

  if (warp == 0) {
    // Converged warp; the elected lane issues the copies. Weights do not
    // depend on the previous kernel: start streaming them before waiting for
    // the activations (programmatic dependent launch).
    int issued = 0;
    for (int i = 0; i < nsl && i < RS; ++i) {
      if (dev::elect_one()) {
        dev::mbar_arrive_expect_tx(rfull + 8 * i, ti.chunk_bytes);
        dev::bulk_load(dev::smem_u32(raw + i * a.chunk_max), chunk0 + (size_t)i * ti.chunk_bytes, ti.chunk_bytes,
                       rfull + 8 * i);
      }
      __syncwarp();
      ++issued;
    }
    dev::pdl_wait();
    if (dev::elect_one()) {
      dev::mbar_arrive_expect_tx(xfull, (uint32_t)(kr / 64) * NP * 128);
      for (int c = 0; c < kr / 64; ++c)
        dev::tma_load_2d(dev::smem_u32(xs + c * NP * 128), &map_x, slab0 * 256 + c * 64, 0, xfull);
    }
    __syncwarp();
    for (int i = RS; i < nsl; ++i) {
      const int s = i % RS;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(rempty + 8 * s, ((i / RS) & 1) ^ 1, a.err))) break;
      if (dev::elect_one()) {
        dev::mbar_arrive_expect_tx(rfull + 8 * s, ti.chunk_bytes);
        dev::bulk_load(dev::smem_u32(raw + s * a.chunk_max), chunk0 + (size_t)i * ti.chunk_bytes, ti.chunk_bytes,
                       rfull + 8 * s);
      }
      __syncwarp();
      ++issued;
    }
    // Drain: every issued copy has landed before shared memory is reused.
    dev::mbar_wait(xfull, 0, a.err, 100000000ull);
    for (int i = issued > RS ? issued - RS : 0; i < issued; ++i)
      dev::mbar_wait(rfull + 8 * (i % RS), (i / RS) & 1, a.err, 100000000ull);
  } else if (warp == 1) {
    // Converged warp; the elected lane (lane 0) issues every MMA and commit.
    constexpr uint32_t idesc = dev::make_idesc_f16(128, NP);
    if (__all_sync(0xffffffffu, dev::mbar_wait(xfull, 0, a.err))) {
      const uint32_t xbase = dev::smem_u32(xs), abase = dev::smem_u32(as);
      int sub = 0;
      bool ok = true;
      for (int i = 0; i < nsl && ok; ++i)
        for (int q = 0; q < 4; ++q, ++sub) {
          const int s = sub % kAStages;
          if (!__all_sync(0xffffffffu, dev::mbar_wait(afull + 8 * s, (sub / kAStages) & 1, a.err))) {
            ok = false;
            break;
          }
          dev::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (dev::elect_one()) {
              const uint64_t ad = dev::make_sw128_desc(abase + s * kABytes + kk * 32);
              const uint64_t bd = dev::make_sw128_desc(xbase + (i * 4 + q) * NP * 128 + kk * 32);
              dev::tc_mma_f16(tmem, ad, bd, idesc, (sub | kk) != 0 ? 1u : 0u);
            }
            __syncwarp();
          }
          if (dev::elect_one()) dev::tc_commit(aempty + 8 * s);
          __syncwarp();
        }
    }
    if (dev::elect_one()) dev::tc_commit(accum);
    __syncwarp();
    dev::mbar_wait(accum, 0, a.err, 100000000ull);
  } else {
    // ---- decoders: thread = weight row of the tile; group grp decodes the
    // quarters q = grp, grp + 2 of every slab into A stage grp ----
    const int r = (threadIdx.x - 64) & 127, grp = (threadIdx.x - 64) >> 7;
    const int half = r >> 6, rr = r & 63;
    const int fmt = ti.fmt[half];
    const int roff = half ? region_bytes(ti.fmt[0]) : 0;
    int sub = 0;
    bool ok = true;
    for (int i = 0; i < nsl && ok; ++i) {
      const int rs = i % RS;
      if (!dev::mbar_wait(rfull + 8 * rs, (i / RS) & 1, a.err)) break;
      const uint8_t* region = raw + rs * a.chunk_max + roff;
      const uint8_t* blk = region + rr * (fmt == kSegQ6K ? 208 : 144);
      const uint16_t d6 = fmt == kSegQ6K ? *reinterpret_cast<const uint16_t*>(region + 64 * 208 + rr * 2) : 0;
      for (int q = grp; q < 4; q += kAStages) {
        sub = i * 4 + q;  // A stage sub % kAStages = grp
        const int s = sub % kAStages;
        if (!dev::mbar_wait(aempty + 8 * s, ((sub / kAStages) & 1) ^ 1, a.err)) {
          ok = false;
          break;
        }
        uint8_t* a_tile = as + s * kABytes;
        const SmemTileSink sink{a_tile, r};
        if (fmt == kSegQ4K) decode_q4k(blk, q, sink);
        else if (fmt == kSegQ6K) decode_q6k(blk, d6, q, sink);
        else decode_q40(blk, q, sink);
        dev::fence_proxy_async_smem();
        dev::mbar_arrive(afull + 8 * s);
      }
      dev::mbar_arrive(rempty + 8 * rs);
    }
    // ---- TMEM -> this CTA's partial tile in shared memory (red[t][row], f32;
    // the raw ring is free once every chunk has been decoded), by warps 2-5 ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    float* red = reinterpret_cast<float*>(raw);
    if (grp == 0 && __all_sync(0xffffffffu, dev::mbar_wait(accum, 0, a.err))) {  // warp-uniform: tcgen05.ld is collective
      dev::tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < NP; c0 += 16) {
        uint32_t v[16];
        dev::tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + c0, v);
        dev::tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) red[(c0 + j) * 128 + row] = __uint_as_float(v[j]);
      }
    }
  }
  // ---- split-K reduction over the cluster + fused epilogue ----
  dev::cluster_sync();
  {
    const int T = min(a.d_tokens ? *a.d_tokens : a.tokens, NP);
    const int S = a.splits, rank = split, n0 = tile * 128;
    const uint32_t red_addr = dev::smem_u32(raw);
    auto sum_row = [&](int t, int r) -> float {
      const uint32_t local = red_addr + (uint32_t)(t * 128 + r) * 4u;
      float v[kMaxSplits];
#pragma unroll
      for (int i = 0; i < kMaxSplits; ++i) v[i] = i < S ? dev::ld_dsmem_f32(dev::mapa(local, i)) : 0.f;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxSplits; ++i)
        if (i < S) acc = __fadd_rn(acc, v[i]);
      return acc;
    };
    if (a.mode == kSkinnyPlain || a.mode == kSkinnyF32) {
      const int r0 = rank * 128 / S, nr = (rank + 1) * 128 / S - r0;
      for (int it = threadIdx.x; it < nr * T; it += blockDim.x) {
        const int r = r0 + it % nr, t = it / nr;
        if (a.mode == kSkinnyF32) reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + n0 + r] = sum_row(t, r);
        else a.out[(size_t)t * a.ldo + n0 + r] = __float2half_rn(sum_row(t, r));
      }
    } else if (a.mode == kSkinnyRope) {
      const int* off = a.merged ? a.meta->tgt_off : a.meta->src_off;
      const int p0 = rank * 64 / S, npairs = (rank + 1) * 64 / S - p0;
      for (int it = threadIdx.x; it < npairs * T; it += blockDim.x) {
        const int r = 2 * (p0 + it % npairs), t = it / npairs;
        const int col = n0 + r;
        // the reference stores QKV in f16 before rotating (ops.ts:189)
        const float even = __half2float(__float2half_rn(sum_row(t, r)));
        const float odd = __half2float(__float2half_rn(sum_row(t, r + 1)));
        __half2 o;
        if (col < kQWidth + kKVWidth) {
          const int b = find_req(off, a.meta->batch, t);
          const int pos = t - off[b];
          const float2 cs = *reinterpret_cast<const float2*>(a.rope + ((size_t)pos * 64 + ((col & 127) >> 1)) * 2);
          o = __halves2half2(__float2half_rn(__fsub_rn(__fmul_rn(even, cs.x), __fmul_rn(odd, cs.y))),
                             __float2half_rn(__fadd_rn(__fmul_rn(even, cs.y), __fmul_rn(odd, cs.x))));
          if (col < kQWidth) *reinterpret_cast<__half2*>(a.q + (size_t)t * kQWidth + col) = o;
          else *reinterpret_cast<__half2*>(a.k + (size_t)t * kKVWidth + col - kQWidth) = o;
        } else {
          o = __halves2half2(__float2half_rn(even), __float2half_rn(odd));
          *reinterpret_cast<__half2*>(a.out + (size_t)t * kQKVWidth + col) = o;
        }
      }
    } else {
      const int g0 = rank * 64 / S, ng = (rank + 1) * 64 / S - g0;
      for (int it = threadIdx.x; it < ng * T; it += blockDim.x) {
        const int r = g0 + it % ng, t = it / ng;
        // gate/up stored f16 before SwiGLU (ops.ts:85-87)
        const float g = __half2float(__float2half_rn(sum_row(t, r)));
        const float u = __half2float(__float2half_rn(sum_row(t, r + 64)));
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        a.out[(size_t)t * kInter + tile * 64 + r] = __float2half_rn(__fmul_rn(silu, u));
      }
    }
  }
  dev::cluster_sync();  // peers may still be reading this CTA's partial tile
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

size_t skinny_smem_bytes(int np, int slabs_max, int chunk_max, int rstages) {
  return 1024 + (size_t)slabs_max * 4 * np * 128 + (((size_t)rstages * chunk_max + 1023) & ~(size_t)1023) +
         kAStages * kABytes + 256;
}

cudaError_t launch_skinny(const CUtensorMap* map_x, const SkinnyArgs& a, int np, int tiles, cudaStream_t s) {
  if (a.splits < 1 || a.splits > kMaxSplits || a.splits > a.slabs || a.rstages < 2 || a.rstages > kMaxRawStages)
    return cudaErrorInvalidValue;
  const size_t smem = skinny_smem_bytes(np, a.slabs_max, a.chunk_max, a.rstages);
  static bool configured[64][3] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int ni = np == 16 ? 0 : np == 32 ? 1 : np == 64 ? 2 : -1;
  if (ni < 0 || dev >= 64) return cudaErrorInvalidValue;
  const void* fn = ni == 0 ? (const void*)skinny_kernel<16> : ni == 1 ? (const void*)skinny_kernel<32>
                                                                       : (const void*)skinny_kernel<64>;
  if (!configured[dev][ni]) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured[dev][ni] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, a.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // the split-K CTAs of a tile
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = a.splits;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (ni == 0) return cudaLaunchKernelEx(&cfg, skinny_kernel<16>, *map_x, a);
  if (ni == 1) return cudaLaunchKernelEx(&cfg, skinny_kernel<32>, *map_x, a);
  return cudaLaunchKernelEx(&cfg, skinny_kernel<64>, *map_x, a);
}

}  // namespace nemo
