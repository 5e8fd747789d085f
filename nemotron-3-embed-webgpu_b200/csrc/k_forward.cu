// Persistent single-launch encoder forward for small token counts (at most
// kFwdNP valid tokens per run, the batch-1 regime of the reference's
// latency-bound path: src/webgpu/model.ts:146-176 with the subgroup / latency
// matmul pipelines of src/webgpu/quant-matmul.ts:156-223,379-423).
//
// At a handful of tokens every projection is a weight stream: ~33 MB of
// quantised weights per layer against a few KB of activations. A launch per
// op leaves the SMs idle between kernels and caps each projection at its own
// pipeline fill. Here one cooperative grid (one CTA per SM) runs the whole
// forward. Each CTA owns a fixed list of weight segments, (projection, 128-row
// tile, K range of 256-column slabs), in forward order, and streams and
// decodes them independently of the activations, running ahead across
// layer boundaries as far as its rings allow. Only the tensor-core step waits
// for activations.
//
//   warp 0      producer: cp.async.bulk of packed 128 x 256 weight chunks
//               into a 4-stage ring, for all segments back to back
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer:
//               D[128 rows x NP tokens] (+)= A[128 x 64] . X^T[64 x NP] per
//               substage, D double-buffered in TMEM across segments
//   warps 2-5   phase warps: the activation side of every phase (below)
//   warps 6-13  decoders (tile_decode.cuh): warps 6-9 fill substages 0 and 2
//               of each slab, warps 10-13 substages 1 and 3, into an A ring.
//               They hold the highest warp numbers of the CTA: with any
//               higher-numbered warp resident on their scheduler, waiting or
//               not, the same decoders ran at half the rate (measured).
//     - projection phases: stage X slabs (f16, 128B-swizzled) into an X
//       ring, drain each finished segment from TMEM to an f32 partial slot in
//       global memory, and count the tile's finished segments; the CTA that
//       finishes a tile last sums its slots in K order (deterministic) and
//       applies the epilogue: RoPE + Q/K/V split (QKV), f16 store (O, down)
//       or SwiGLU (gate/up, rows interleaved 64 gate + 64 up per tile)
//     - small phases: embedding + RMSNorm, attention, residual + RMSNorm,
//       token merge, mean pool, each spread over the grid by item
//   and a grid barrier between phases (release/acquire on a global counter).
//
// Every wait is bounded (%globaltimer) and also gives up as soon as any
// thread has raised the error word, so a failure unwinds the whole grid
// within microseconds; the host reads the word after the run. Loops of the
// phase warps never exit early, so their named barriers always match.
#include <math.h>

#include "tile_decode.cuh"

namespace nemo {
namespace {

using namespace tsd;

constexpr int kThreads = 448;
constexpr int kPhaseThread0 = 64;   // warps 2..5
constexpr int kDecThread0 = 192;    // warps 6..13
constexpr int kRawStages = 4;   // packed weight chunks in shared memory
constexpr int kASlabs = 3;     // decoded A slabs in TMEM (128 x 256 f16 = 128 columns each)
constexpr int kXStages = 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDevErrGridBarrier = 4u;

__device__ __forceinline__ uint32_t ld_err(const uint32_t* e) { return *reinterpret_cast<const volatile uint32_t*>(e); }

// Bounded mbarrier wait (limit_ns) that also returns false once the error
// word is set.
__device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, uint32_t* err, uint64_t limit_ns) {
  if (dev::mbar_try_wait(bar, parity)) return true;
  if (ld_err(err)) return false;
  const uint64_t t0 = dev::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (dev::mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (ld_err(err)) return false;
      if (dev::globaltimer() - t0 > limit_ns) {
        atomicOr(err, kDevErrMbarTimeout);
        return false;
      }
    }
  }
}


__device__ __forceinline__ void pw_sync() { dev::named_barrier(1, 128); }

// Release/acquire hand-offs between CTAs. A sequentially consistent fence
// (__threadfence) costs 1.5-3 us here while the weight stream is in flight;
// these need only release (publish this CTA's writes, ordered before by the
// named barrier) and acquire (see the other CTAs' writes).
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __halves2half2(__float2half_rn(v[2 * i]), __float2half_rn(v[2 * i + 1]));
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row sum over 256 virtual threads (8 values each) with the reduction tree of
// the 256-thread row kernels in k_misc.cu (butterfly per 32 virtual lanes,
// then a butterfly over the 8 warp totals): phase thread p holds virtual
// threads p (s0) and 128 + p (s1), so the result is bit-identical.
__device__ __forceinline__ float row_sum_256(float s0, float s1, float* red) {
  const int pt = threadIdx.x - kPhaseThread0, w = pt >> 5, lane = pt & 31;
  s0 = warp_sum(s0);
  s1 = warp_sum(s1);
  if (lane == 0) {
    red[w] = s0;
    red[4 + w] = s1;
  }
  pw_sync();
  float t = lane < 8 ? red[lane] : 0.f;
  t = warp_sum(t);
  pw_sync();  // red is reused by the next call
  return t;
}

struct Shared {
  uint32_t tmem;
  int flag;
  int quiet;  // set while the phase warps run a latency-critical small phase
  float red[8];
};

template <int NP>
__global__ void __launch_bounds__(kThreads, 1) forward_kernel(const __grid_constant__ FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = dev::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  constexpr int kXBytes = 4 * NP * 128;      // one 256-column slab of X: 4 x [NP rows x 64 f16]
  constexpr int kSlotBytes = NP * 128 * 4;   // slot-buffer unit: [NP][128] f32
  const int CM = a.chunk_max;
  // shared layout: X ring | epilogue slots | raw weight ring | barriers
  uint8_t* xring = smem;
  float* ebuf = reinterpret_cast<float*>(xring + kXStages * kXBytes);
  uint8_t* raw = reinterpret_cast<uint8_t*>(ebuf) + (size_t)a.scratch_slots * kSlotBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + ((kRawStages * CM + 15) & ~15));
  const uint32_t rfull = dev::smem_u32(bars), rempty = rfull + 8 * kRawStages;
  const uint32_t afull = rempty + 8 * kRawStages, aempty = afull + 8 * kASlabs;
  const uint32_t xfull = aempty + 8 * kASlabs, xempty = xfull + 8 * kXStages;
  const uint32_t dfull = xempty + 8 * kXStages, dempty = dfull + 16, fin = dempty + 16, ebar = fin + 8;
  const uint32_t rowbar = ebar + 8;  // the norm phase's bulk loads
  Shared* sh = reinterpret_cast<Shared*>(bars + 2 * kRawStages + 2 * kASlabs + 2 * kXStages + 7);
  // Run metadata copied to shared memory once: this CTA's segments, slot
  // counts and strides, the run's Meta and the RoPE rows of positions < NP.
  FwdSeg* segs = reinterpret_cast<FwdSeg*>(reinterpret_cast<uint8_t*>(sh) + ((sizeof(Shared) + 15) & ~15));
  Meta* meta = reinterpret_cast<Meta*>(segs + a.max_segs);
  float* rope = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(meta + 1) + 15) & ~(uintptr_t)15);
  int* sstride = reinterpret_cast<int*>(rope + NP * 128);
  uint8_t* nslots = reinterpret_cast<uint8_t*>(sstride + a.n_layers * 4);
  uint8_t* srank = nslots + a.n_layers * 4 * kFwdMaxTiles;  // [n_layers * 3] this CTA's small-phase ranks
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  const int seg0 = a.seg_start[cta];
  const int nseg = a.seg_start[cta + 1] - seg0;
  uint32_t* err = a.err;
  const uint64_t lim = a.wait_ns;  // bound of every wait (2 s unless a test shortens it)
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.segs + seg0);
    uint32_t* dst = reinterpret_cast<uint32_t*>(segs);
    for (int i = threadIdx.x; i < nseg * (int)(sizeof(FwdSeg) / 4); i += kThreads) dst[i] = src[i];
    for (int i = threadIdx.x; i < (int)(sizeof(Meta) / 4); i += kThreads)
      reinterpret_cast<int*>(meta)[i] = reinterpret_cast<const int*>(a.meta)[i];
    for (int i = threadIdx.x; i < NP * 128; i += kThreads) rope[i] = i < a.rope_rows * 128 ? a.rope[i] : 0.f;
    for (int i = threadIdx.x; i < a.n_layers * 4; i += kThreads) sstride[i] = a.sstride[i];
    for (int i = threadIdx.x; i < a.n_layers * 4 * kFwdMaxTiles; i += kThreads) nslots[i] = a.nslots[i];
    for (int i = threadIdx.x; i < a.n_layers * 3; i += kThreads) srank[i] = a.small_rank[(size_t)i * G + cta];
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) dev::prefetch_tmap(&a.xmap[i]);
    for (int s = 0; s < kRawStages; ++s) {
      dev::mbar_init(rfull + 8 * s, 1);
      dev::mbar_init(rempty + 8 * s, 256);
    }
    for (int s = 0; s < kASlabs; ++s) {
      dev::mbar_init(afull + 8 * s, 256);
      dev::mbar_init(aempty + 8 * s, 1);
    }
    for (int s = 0; s < kXStages; ++s) {
      dev::mbar_init(xfull + 8 * s, 1);
      dev::mbar_init(xempty + 8 * s, 1);
    }
    for (int d = 0; d < 2; ++d) {
      dev::mbar_init(dfull + 8 * d, 1);
      dev::mbar_init(dempty + 8 * d, 128);
    }
    dev::mbar_init(fin, 1);
    dev::mbar_init(ebar, 1);
    dev::mbar_init(rowbar, 1);
    dev::fence_mbar_init();
    sh->flag = 0;
    sh->quiet = 0;
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(&sh->tmem), kTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = sh->tmem;
  // TMEM columns: two D accumulators of NP columns (segments alternate; every
  // substage of a segment accumulates into its D), then the A slabs.
  const uint32_t tm_a = tmem + 8 * NP;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the schedule; one elected lane issues each copy.
    // Weights are read once per forward: L2 evict-first keeps them from
    // displacing the activations and partial sums the phases exchange.
    const uint64_t policy = dev::l2_evict_first_policy();
    int it = 0;
    bool ok = true;
    for (int si = 0; si < nseg && ok; ++si) {
      const FwdSeg sg = segs[si];
      for (int sl = sg.s0; sl < sg.s1; ++sl, ++it) {
        if (*reinterpret_cast<volatile int*>(&sh->quiet)) {
          const uint64_t t0 = dev::globaltimer();
          while (*reinterpret_cast<volatile int*>(&sh->quiet) && dev::globaltimer() - t0 < lim) __nanosleep(128);
        }
        const int s = it % kRawStages;
        if (!__all_sync(0xffffffffu, wait(rempty + 8 * s, ((it / kRawStages) & 1) ^ 1, err, lim))) {
          ok = false;
          break;
        }
        if (dev::elect_one()) {
          dev::mbar_arrive_expect_tx(rfull + 8 * s, sg.chunk_bytes);
          dev::bulk_load_hint(dev::smem_u32(raw + s * CM), sg.chunk0 + (size_t)sl * sg.chunk_bytes, sg.chunk_bytes,
                              rfull + 8 * s, policy);
        }
        __syncwarp();
      }
    }
    // Every issued copy lands before the CTA may exit.
    for (int j = it > kRawStages ? it - kRawStages : 0; j < it; ++j)
      dev::mbar_wait(rfull + 8 * (j % kRawStages), (j / kRawStages) & 1, err, 100000000ull);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Converged warp, elected lane 0 issues every MMA and commit.
    constexpr uint32_t idesc = dev::make_idesc_f16(128, NP);
    const uint32_t xbase = dev::smem_u32(xring);
    int it = 0;
    bool ok = true;
    for (int si = 0; si < nseg && ok; ++si) {
      const FwdSeg sg = segs[si];
      const int d = si & 1;
      if (!__all_sync(0xffffffffu, wait(dempty + 8 * d, ((si >> 1) & 1) ^ 1, err, lim))) break;
      dev::tc_fence_after();
      for (int sl = sg.s0; sl < sg.s1; ++sl, ++it) {
        const int xs = it % kXStages, s = it % kASlabs;
        if (!__all_sync(0xffffffffu, wait(xfull + 8 * xs, (it / kXStages) & 1, err, lim) &&
                                         wait(afull + 8 * s, (it / kASlabs) & 1, err, lim))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (dev::elect_one()) {
              const uint64_t bd = dev::make_sw128_desc(xbase + xs * kXBytes + q * NP * 128 + kk * 32);
              dev::tc_mma_f16_ts(tmem + d * NP, tm_a + s * 128 + q * 32 + kk * 8, bd, idesc,
                                 (sl != sg.s0 || q != 0 || kk != 0) ? 1u : 0u);
            }
            __syncwarp();
          }
        if (dev::elect_one()) {
          dev::tc_commit(aempty + 8 * s);
          dev::tc_commit(xempty + 8 * xs);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (dev::elect_one()) dev::tc_commit(dfull + 8 * d);
      __syncwarp();
    }
    // All issued MMAs complete before the TMEM is released.
    if (dev::elect_one()) dev::tc_commit(fin);
    __syncwarp();
    dev::mbar_wait(fin, 0, err, 100000000ull);
  } else if (threadIdx.x >= kDecThread0) {
    // ------------------------------------------------------------ decoders
    // Warp w writes TMEM lanes 32 * (w % 4) .. + 31, so its threads own those
    // weight rows; warps 6-9 fill substages 0 and 2 of every slab, warps 10-13
    // substages 1 and 3. A slab is handed to the MMA once both halves are in.
    const int quarter = warp & 3, grp = (warp - kDecThread0 / 32) >> 2;
    const int r = quarter * 32 + lane;
    const int half = r >> 6, rr = r & 63;  // half is uniform within a warp
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int si = 0; si < nseg && ok; ++si) {
      const FwdSeg sg = segs[si];
      const int fmt = sg.fmt[half];
      const int roff = half ? region_bytes(sg.fmt[0]) : 0;
      for (int sl = sg.s0; sl < sg.s1; ++sl, ++it) {
        // Yield the SM's issue slots to the phase warps during small phases
        // (attention, norms); bounded like every other wait.
        if (*reinterpret_cast<volatile int*>(&sh->quiet)) {
          const uint64_t t0 = dev::globaltimer();
          while (*reinterpret_cast<volatile int*>(&sh->quiet) && dev::globaltimer() - t0 < lim) __nanosleep(128);
        }
        const int rs = it % kRawStages;
        if (!__all_sync(0xffffffffu, wait(rfull + 8 * rs, (it / kRawStages) & 1, err, lim))) {
          ok = false;
          break;
        }
        const uint8_t* region = raw + rs * CM + roff;
        const uint8_t* blk = region + rr * (fmt == kSegQ6K ? 208 : 144);
        const uint16_t d6 = fmt == kSegQ6K ? *reinterpret_cast<const uint16_t*>(region + 64 * 208 + rr * 2) : 0;
        const int s = it % kASlabs;
        if (!__all_sync(0xffffffffu, wait(aempty + 8 * s, ((it / kASlabs) & 1) ^ 1, err, lim))) {
          ok = false;
          break;
        }
        // Both quarters are decoded into separate registers before either
        // TMEM store (two independent chains per thread).
        {
          uint32_t ha[32], hb[32];
          const RegSink sa{ha}, sb{hb};
          if (fmt == kSegQ4K) {
            decode_q4k(blk, grp, sa);
            decode_q4k(blk, grp + 2, sb);
          } else if (fmt == kSegQ6K) {
            decode_q6k(blk, d6, grp, sa);
            decode_q6k(blk, d6, grp + 2, sb);
          } else {
            decode_q40(blk, grp, sa);
            decode_q40(blk, grp + 2, sb);
          }
          dev::tmem_st_32x32b_x32(tm_a + lane_base + s * 128 + grp * 32, ha);
          dev::tmem_st_32x32b_x32(tm_a + lane_base + s * 128 + (grp + 2) * 32, hb);
        }
        dev::tc_wait_st();
        dev::tc_fence_before();
        dev::mbar_arrive(afull + 8 * s);
        dev::mbar_arrive(rempty + 8 * rs);
      }
    }
  } else {
    // ------------------------------------------------------------ phase warps
    const int pt = threadIdx.x - kPhaseThread0;
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int batch = min(meta->batch, kMaxBatch);
    const int T0 = min(meta->t0, NP), T1 = min(meta->t1, NP);
    int si = 0, xit = 0, gseg = 0, eph = 0, nph = 0;
    uint32_t nbarriers = 0;
    // Test hook: when set, grid barrier number *test_stall (1-based) waits
    // for one arrival more than the grid has, so it gives up at the wait
    // bound and the whole grid unwinds through the error word.
    const uint32_t stall = a.test_stall ? *reinterpret_cast<const volatile uint32_t*>(a.test_stall) : 0u;

    auto grid_barrier = [&]() {
      pw_sync();
      if (pt == 0) {
        red_add_release(&a.sync[0], 1u);
        const uint32_t target = (++nbarriers) * (uint32_t)G + (nbarriers == stall ? 1u : 0u);
        if (!ld_err(err)) {
          const uint64_t t0 = dev::globaltimer();
          for (uint32_t i = 0;; ++i) {
            if (ld_acquire(&a.sync[0]) >= target) break;
            if ((i & 15u) == 15u) {
              if (ld_err(err)) break;
              if (dev::globaltimer() - t0 > lim) {
                atomicOr(err, kDevErrGridBarrier);
                break;
              }
            }
          }
        }
        // (the acquire loads above order what follows) X tiles of the next
        // phase are read by TMA (async proxy) after this.
        dev::fence_proxy_async_global();
      }
      pw_sync();
    };

    // Split-K epilogue of a finished gate/up tile: one bulk copy brings all of
    // its partial slots (written by other CTAs, released through the tile
    // counter) into shared memory; they are summed in slot (= K) order.
    auto epilogue = [&](int pi, int tile, int T) {
      const int S = nslots[pi * kFwdMaxTiles + tile], ss = sstride[pi];
      if (pt < 32) {  // issued by lane 0 of the converged first phase warp
        if (dev::elect_one()) {
          dev::fence_proxy_async_global();
          dev::mbar_arrive_expect_tx(ebar, (uint32_t)(T * ss * 512));
          dev::bulk_load(dev::smem_u32(ebuf), a.part + (size_t)tile * NP * ss * 128, (uint32_t)(T * ss * 512), ebar);
        }
        __syncwarp();
      }
      const bool got = wait(ebar, eph & 1, err, lim);
      ++eph;
      // Each thread keeps one accumulator per token (independent chains) and
      // adds the slots in order; f16 gate and up, then SwiGLU (ops.ts:74-89).
      if (got) {
        const int r = pt & 63, tb = (pt >> 6) * (NP / 2);
        float g[NP / 2], u[NP / 2];
#pragma unroll
        for (int j = 0; j < NP / 2; ++j) g[j] = u[j] = 0.f;
        for (int s = 0; s < S; ++s)
#pragma unroll
          for (int j = 0; j < NP / 2; ++j) {
            const float* p = ebuf + ((tb + j) * ss + s) * 128;
            g[j] = __fadd_rn(g[j], p[r]);
            u[j] = __fadd_rn(u[j], p[64 + r]);
          }
#pragma unroll
        for (int j = 0; j < NP / 2; ++j) {
          const int t = tb + j;
          if (t >= T) break;
          const float gh = __half2float(__float2half_rn(g[j])), uh = __half2float(__float2half_rn(u[j]));
          const float silu = __fdiv_rn(gh, __fadd_rn(1.0f, expf(-gh)));
          a.ffn[(size_t)t * kInter + tile * 64 + r] = __float2half_rn(__fmul_rn(silu, uh));
        }
      }
      dev::fence_proxy_async_smem();  // these reads of ebuf precede the next bulk write into it
      pw_sync();
    };

    // TMEM -> partial slot. QKV, O and down partials are summed by the next
    // phase after the grid barrier; gate/up tiles are counted, and the CTA
    // that completes one runs its SwiGLU epilogue (returns true).
    auto drain = [&](const FwdSeg& sg, int T, bool counted) -> bool {
      const int d = gseg & 1;
      const bool got = __all_sync(0xffffffffu, wait(dfull + 8 * d, (gseg >> 1) & 1, err, lim));
      ++gseg;
      const int ss = sstride[sg.proj];
      // O / down: token-major [t][tile][slot] (a norm row reads one block);
      // QKV / gate-up: tile-major [tile][t][slot] (an attention head or a
      // gate/up epilogue reads one block per tile).
      const bool token_major = (sg.proj & 1) != 0;
      const size_t tstride = token_major ? (size_t)(kHidden / 128) * ss * 128 : (size_t)ss * 128;
      float* slot = a.part + (token_major ? (size_t)sg.tile * ss : (size_t)sg.tile * NP * ss) * 128 + (size_t)sg.slot * 128;
      if (got) {
        dev::tc_fence_after();
        const int row = quarter * 32 + lane;
#pragma unroll
        for (int c0 = 0; c0 < NP; c0 += 16) {
          uint32_t v[16];
          dev::tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + d * NP + c0, v);
          dev::tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < T) __stcg(slot + (size_t)(c0 + j) * tstride + row, __uint_as_float(v[j]));
        }
      }
      dev::tc_fence_before();
      dev::mbar_arrive(dempty + 8 * d);
      if (!counted) return false;
      pw_sync();
      if (pt == 0) {
        int last = 0;
        if (!ld_err(err)) {
          const int idx = sg.proj * kFwdMaxTiles + sg.tile;
          const uint32_t old = atom_add_acq_rel(&a.sync[1 + idx], 1u);
          last = old + 1 == (uint32_t)nslots[idx];
        }
        sh->flag = last;
      }
      pw_sync();
      return *reinterpret_cast<volatile int*>(&sh->flag) != 0;
    };

    // A gate/up tile computed whole by this CTA: its accumulator goes from
    // TMEM to shared memory (rows = 64 gate + 64 up columns) and the SwiGLU
    // epilogue runs from there, with the arithmetic of the split-K epilogue
    // above for a single slot.
    auto drain_swiglu = [&](const FwdSeg& sg, int T) {
      const int d = gseg & 1;
      const bool got = __all_sync(0xffffffffu, wait(dfull + 8 * d, (gseg >> 1) & 1, err, lim));
      ++gseg;
      if (got) {
        dev::tc_fence_after();
        const int row = quarter * 32 + lane;
#pragma unroll
        for (int c0 = 0; c0 < NP; c0 += 16) {
          uint32_t v[16];
          dev::tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + d * NP + c0, v);
          dev::tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) ebuf[(c0 + j) * 128 + row] = __uint_as_float(v[j]);
        }
      }
      dev::tc_fence_before();
      dev::mbar_arrive(dempty + 8 * d);
      pw_sync();
      if (got) {
        const int r = pt & 63, tb = (pt >> 6) * (NP / 2);
#pragma unroll
        for (int j = 0; j < NP / 2; ++j) {
          const int t = tb + j;
          if (t >= T) break;
          const float gh = __half2float(__float2half_rn(__fadd_rn(0.f, ebuf[t * 128 + r])));
          const float uh = __half2float(__float2half_rn(__fadd_rn(0.f, ebuf[t * 128 + 64 + r])));
          const float silu = __fdiv_rn(gh, __fadd_rn(1.0f, expf(-gh)));
          a.ffn[(size_t)t * kInter + sg.tile * 64 + r] = __float2half_rn(__fmul_rn(silu, uh));
        }
      }
      dev::fence_proxy_async_smem();  // these accesses of ebuf precede any later bulk write into it
      pw_sync();
    };

    // X slabs by TMA (first phase warp, elected lane 0: the lane that made the
    // barrier's acquire visible to the async proxy), then drains of the
    // finished segments.
    auto projection = [&](int pi, const CUtensorMap* xmap, bool merged) {
      const int T = merged ? T1 : T0;
      const int first = si;
      while (si < nseg && segs[si].proj == pi) ++si;
      const bool counted = (pi & 3) == 2;
      int last_tiles[4], nlast = 0;
      auto publish = [&](int j) {
        if (counted && nslots[pi * kFwdMaxTiles + segs[j].tile] == 1) drain_swiglu(segs[j], T);
        else if (drain(segs[j], T, counted) && nlast < 4) last_tiles[nlast++] = segs[j].tile;
      };
      for (int j = first; j < si; ++j) {
        const FwdSeg sg = segs[j];
        if (pt < 32) {
          for (int sl = sg.s0; sl < sg.s1; ++sl, ++xit) {
            const int xs = xit % kXStages;
            if (__all_sync(0xffffffffu, wait(xempty + 8 * xs, ((xit / kXStages) & 1) ^ 1, err, lim)) && dev::elect_one()) {
              dev::mbar_arrive_expect_tx(xfull + 8 * xs, kXBytes);
              for (int q = 0; q < 4; ++q)
                dev::tma_load_2d(dev::smem_u32(xring + xs * kXBytes + q * NP * 128), xmap, sl * 256 + q * 64, 0,
                                 xfull + 8 * xs);
            }
            __syncwarp();
          }
        }
        if (j > first) publish(j - 1);
      }
      if (si > first) publish(si - 1);
      for (int e = 0; e < nlast; ++e) epilogue(pi, last_tiles[e], T);
    };

    float* stage = reinterpret_cast<float*>(xring);  // X ring + slot buffers, idle outside projections

    // Residual add of projection rpi's output (rpi < 0: none) + RMSNorm of
    // one row (ops.ts:21-72). The row's partial slots of the 16 output tiles
    // are staged first: stage[(tile * ss + slot) * 128 + column].
    auto norm_row = [&](__half* x, int rpi, const float* w, __half* out, int t) {
      const bool res = rpi >= 0;
      const int sst = res ? sstride[rpi] : 0;
      if (res) {
        // Two bulk copies (the row's contiguous slot block, then its residual
        // row) by the elected lane of the first phase warp. The staging area's
        // earlier generic accesses are ordered before the async-proxy writes.
        const uint32_t slot_bytes = (uint32_t)((kHidden / 128) * sst * 512);
        dev::fence_proxy_async_smem();
        pw_sync();
        if (pt < 32) {
          if (dev::elect_one()) {
            dev::mbar_arrive_expect_tx(rowbar, slot_bytes + kHidden * 2);
            dev::bulk_load(dev::smem_u32(stage), a.part + (size_t)t * (kHidden / 128) * sst * 128, slot_bytes, rowbar);
            dev::bulk_load(dev::smem_u32(stage + (kHidden / 128) * sst * 128), x + (size_t)t * kHidden, kHidden * 2,
                           rowbar);
          }
          __syncwarp();
        }
        wait(rowbar, nph & 1, err, lim);
        ++nph;
      }
      float v[2][8];
      float ss[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = h * 1024 + pt * 8;
        if (res)
          unpack8(*reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(stage + (kHidden / 128) * sst * 128) + c),
                  v[h]);
        else
          unpack8(__ldcg(reinterpret_cast<const uint4*>(x + (size_t)t * kHidden + c)), v[h]);
        if (res) {
          const int tile = c >> 7, S = nslots[rpi * kFwdMaxTiles + tile];
          const float* p = stage + tile * sst * 128 + (c & 127);
          float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int sl = 0; sl < S; ++sl) {
            const float4 u0 = *reinterpret_cast<const float4*>(p + sl * 128);
            const float4 u1 = *reinterpret_cast<const float4*>(p + sl * 128 + 4);
            const float uu[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) r8[i] = __fadd_rn(r8[i], uu[i]);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) v[h][i] = __fadd_rn(v[h][i], __half2float(__float2half_rn(r8[i])));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss[h] = __fadd_rn(ss[h], __fmul_rn(v[h][i], v[h][i]));
      }
      const float total = row_sum_256(ss[0], ss[1], sh->red);
      const float inv = rsqrtf(__fadd_rn(__fdiv_rn(total, (float)kHidden), kEpsilon));
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = h * 1024 + pt * 8;
        const uint4 xs = pack8(v[h]);
        if (res) __stcg(reinterpret_cast<uint4*>(x + (size_t)t * kHidden + c), xs);
        float xn[8], o[8];
        unpack8(xs, xn);
        const float4 w0 = *reinterpret_cast<const float4*>(w + c);
        const float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(xn[i], inv), wv[i]);
        __stcg(reinterpret_cast<uint4*>(out + (size_t)t * kHidden + c), pack8(o));
      }
    };

    auto set_quiet = [&](bool on) {
      if (pt == 0) *reinterpret_cast<volatile int*>(&sh->quiet) = on ? 1 : 0;
    };
    // Only CTAs that hold items quiet their decoders: the others keep the
    // weight rings filling through the small phases. Items go to CTAs by
    // rank (the least work in the next projection first).
    auto norm_phase = [&](__half* x, int rpi, const float* w, __half* out, int T, int rank) {
      if (rank < T) set_quiet(true);
      for (int t = rank; t < T; t += G) norm_row(x, rpi, w, out, t);
      set_quiet(false);
    };

    // ---- embedding (ops.ts:680-725) + first RMSNorm, one token per item ----
    for (int t = cta; t < T0; t += G) {
      const int b = find_req(meta->src_off, batch, t);
      const int p = t - meta->src_off[b];
      uint32_t id = a.ids[(size_t)b * meta->seq + p];
      if (id >= (uint32_t)a.vocab) id = 0;  // the host validates ids; keeps reads in bounds
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = h * 1024 + pt * 8;
        const int within = c & 255, hf = within >> 7, position = within & 127;
        const int quad = position >> 5, ln = position & 31;
        const uint8_t* blk = a.embd + ((size_t)id * (kHidden / 256) + (c >> 8)) * 210;
        const float d = half_at(blk + 208);
        const int sc = (int)(int8_t)blk[192 + hf * 8 + ln / 16 + quad * 2];
        const float ds = __fmul_rn(d, (float)sc);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int lb = blk[hf * 64 + ln + i + (quad & 1) * 32];
          const int lo = quad >= 2 ? (lb >> 4) : (lb & 15);
          const int hi = (blk[128 + hf * 32 + ln + i] >> (quad * 2)) & 3;
          v[i] = __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
        }
        __stcg(reinterpret_cast<uint4*>(a.x + (size_t)t * kHidden + c), pack8(v));
      }
      norm_row(a.x, -1, a.attn_norm[0], a.nrm, t);
    }
    grid_barrier();

    for (int l = 0; l < a.n_layers; ++l) {
      const bool merged = !a.exact && l >= kMergeAfterLayer;
      if (l == kMergeAfterLayer && !a.exact) {
        // ---- token merge of x and the normalised state (ops.ts:629-661) ----
        for (int t = cta; t < T1; t += G) {
          const int b = find_req(meta->tgt_off, batch, t);
          const uint32_t p = (uint32_t)(t - meta->tgt_off[b]);
          const uint32_t sl = (uint32_t)meta->src_len[b], tl = (uint32_t)meta->tgt_len[b];
          uint32_t start = 0, end = 1;
          if (p > 0 && tl > 1) {
            const uint32_t st = sl - 1, tt = tl - 1;
            start = 1 + ((p - 1) * st) / tt;
            end = 1 + (p * st) / tt;
            end = max(end, start + 1);
            end = min(end, sl);
          }
          const size_t src = (size_t)meta->src_off[b];
          const float cnt = (float)(end - start);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = h * 1024 + pt * 8;
            float tx[8] = {0, 0, 0, 0, 0, 0, 0, 0}, tn[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (uint32_t s = start; s < end; ++s) {
              float xv[8], nv[8];
              unpack8(__ldcg(reinterpret_cast<const uint4*>(a.x + (src + s) * kHidden + c)), xv);
              unpack8(__ldcg(reinterpret_cast<const uint4*>(a.nrm + (src + s) * kHidden + c)), nv);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                tx[i] = __fadd_rn(tx[i], xv[i]);
                tn[i] = __fadd_rn(tn[i], nv[i]);
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              tx[i] = __fdiv_rn(tx[i], cnt);
              tn[i] = __fdiv_rn(tn[i], cnt);
            }
            __stcg(reinterpret_cast<uint4*>(a.xm + (size_t)t * kHidden + c), pack8(tx));
            __stcg(reinterpret_cast<uint4*>(a.nm + (size_t)t * kHidden + c), pack8(tn));
          }
        }
        grid_barrier();
      }
      __half* X = merged ? a.xm : a.x;
      __half* N = merged ? a.nm : a.nrm;
      const int T = merged ? T1 : T0;

      projection(l * 4 + 0, &a.xmap[merged ? 1 : 0], merged);
      grid_barrier();

      // ---- QKV outputs (ops.ts:168-194): the projection's partial slots summed
      // in K order, f16, RoPE on Q and K (position = row within the request);
      // spread over the grid, item = (128-column tile, token), thread = column.
      // Up to four items per pass keep all their slot loads in flight. ----
      {
        const int qkv_pi = l * 4, ss = sstride[qkv_pi];
        const int* off = merged ? meta->tgt_off : meta->src_off;
        const uint8_t* ns = nslots + qkv_pi * kFwdMaxTiles;
        constexpr int kTiles = kQKVWidth / 128, kItemsPerPass = 4, kSlotRegs = 8;
        const int n_items = kTiles * T;
        for (int i0 = cta; i0 < n_items; i0 += kItemsPerPass * G) {
          float v[kItemsPerPass][kSlotRegs];
#pragma unroll
          for (int k = 0; k < kItemsPerPass; ++k) {
            const int item = i0 + k * G;
            const int tile = item % kTiles, t = item / kTiles;
            const int S = item < n_items ? ns[tile] : 0;
            const float* p = a.part + ((size_t)tile * NP + t) * ss * 128 + pt;
#pragma unroll
            for (int sl = 0; sl < kSlotRegs; ++sl) v[k][sl] = sl < S ? __ldcg(p + sl * 128) : 0.f;
          }
#pragma unroll
          for (int k = 0; k < kItemsPerPass; ++k) {
            const int item = i0 + k * G;
            if (item >= n_items) break;  // uniform over the CTA
            const int tile = item % kTiles, t = item / kTiles;
            const int S = ns[tile];
            const float* p = a.part + ((size_t)tile * NP + t) * ss * 128 + pt;
            float acc = 0.f;
#pragma unroll
            for (int sl = 0; sl < kSlotRegs; ++sl)
              if (sl < S) acc = __fadd_rn(acc, v[k][sl]);
            for (int sl = kSlotRegs; sl < S; ++sl) acc = __fadd_rn(acc, __ldcg(p + sl * 128));
            const float val = __half2float(__float2half_rn(acc));
            const int col = tile * 128 + pt;
            if (col < kQWidth + kKVWidth) {
              const float other = __shfl_xor_sync(0xffffffffu, val, 1);  // the pair partner (adjacent column)
              const bool odd = pt & 1;
              const float even_v = odd ? other : val, odd_v = odd ? val : other;
              const int b = find_req(off, batch, t);
              const float2 cs = *reinterpret_cast<const float2*>(rope + ((t - off[b]) * 64 + ((col & 127) >> 1)) * 2);
              const float r = odd ? __fadd_rn(__fmul_rn(even_v, cs.y), __fmul_rn(odd_v, cs.x))
                                  : __fsub_rn(__fmul_rn(even_v, cs.x), __fmul_rn(odd_v, cs.y));
              if (col < kQWidth) a.q[(size_t)t * kQWidth + col] = __float2half_rn(r);
              else a.k[(size_t)t * kKVWidth + col - kQWidth] = __float2half_rn(r);
            } else {
              a.qkv[(size_t)t * kQKVWidth + col] = __float2half_rn(val);
            }
          }
        }
      }
      grid_barrier();

      // ---- attention (ops.ts:295-362): item = (request, q head, group of up
      // to 8 queries). Thread per (query, key) score with four partial sums,
      // softmax per query row, then thread d accumulates dimension d of each
      // query's output. ----
      {
        float* ks = reinterpret_cast<float*>(xring);  // [NP][128]
        float* vs = ks + NP * kHeadDim;                // [NP][128]
        float* qs = vs + NP * kHeadDim;                // [8][128]
        float* ps = qs + 8 * kHeadDim;                 // [8][NP]
        float* linv = ps + 8 * NP;                     // [8]
        const int* off = merged ? meta->tgt_off : meta->src_off;
        constexpr int kQG = 8, kGroups = (NP + kQG - 1) / kQG;
        const int rank = srank[l * 3];
        if (rank < batch * kQHeads * kGroups) set_quiet(true);
        for (int item = rank; item < batch * kQHeads * kGroups; item += G) {
          const int b = item / (kQHeads * kGroups), rem = item % (kQHeads * kGroups);
          const int h = rem / kGroups, g = rem % kGroups, kvh = h / (kQHeads / kKVHeads);
          const int len = min(merged ? meta->tgt_len[b] : meta->src_len[b], NP);
          const int q0 = g * kQG, nq = min(kQG, len - q0);
          if (nq <= 0) continue;  // uniform over the CTA
          const int base = off[b];
          // K and V rows of the request, Q rows of the group: every load is
          // issued before the first shared-memory store
          constexpr int kLoads = ((2 * NP + kQG) * 16 + 127) / 128;
          uint4 buf[kLoads];
          float* dsts[kLoads];
#pragma unroll
          for (int k = 0; k < kLoads; ++k) {
            const int u = pt + k * 128, row = u >> 4, c = (u & 15) * 8;
            dsts[k] = nullptr;
            if (row < len) {
              buf[k] = __ldcg(reinterpret_cast<const uint4*>(a.k + ((size_t)(base + row) * kKVHeads + kvh) * kHeadDim + c));
              dsts[k] = ks + row * kHeadDim + c;
            } else if (row < 2 * len) {
              buf[k] = __ldcg(reinterpret_cast<const uint4*>(a.qkv + (size_t)(base + row - len) * kQKVWidth + kQWidth +
                                                             kKVWidth + kvh * kHeadDim + c));
              dsts[k] = vs + (row - len) * kHeadDim + c;
            } else if (row < 2 * len + nq) {
              buf[k] = __ldcg(reinterpret_cast<const uint4*>(a.q + ((size_t)(base + q0 + row - 2 * len) * kQHeads + h) * kHeadDim + c));
              dsts[k] = qs + (row - 2 * len) * kHeadDim + c;
            }
          }
#pragma unroll
          for (int k = 0; k < kLoads; ++k)
            if (dsts[k]) {
              float f[8];
              unpack8(buf[k], f);
#pragma unroll
              for (int e = 0; e < 8; ++e) dsts[k][e] = f[e];
            }
          pw_sync();
          {
            // thread = (query i, key j): kQG x NP = 128 scores; each query
            // row's softmax runs across its 16 lanes by shuffles
            static_assert(kQG * NP == 128, "one score per phase thread");
            const float scale = 0.08838834764831845f;
            const int i = pt >> 4, j = pt & 15;
            const bool valid = i < nq && j < len;
            float sc = -INFINITY;
            if (valid) {
              float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
              for (int dd = 0; dd < kHeadDim; dd += 4) {
                const int d = (dd + 4 * j) & (kHeadDim - 1);
                const float4 q4 = *reinterpret_cast<const float4*>(qs + i * kHeadDim + d);
                const float4 k4 = *reinterpret_cast<const float4*>(ks + j * kHeadDim + d);
                s4[0] = fmaf(q4.x, k4.x, s4[0]);
                s4[1] = fmaf(q4.y, k4.y, s4[1]);
                s4[2] = fmaf(q4.z, k4.z, s4[2]);
                s4[3] = fmaf(q4.w, k4.w, s4[3]);
              }
              const int pos = q0 + i;
              const float temp = pos >= 16384 ? logf(floorf((float)pos / 16384.0f) + 1.0f) * 0.1f + 1.0f : 1.0f;
              sc = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * scale * temp;
            }
            float m = sc;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float p = valid ? expf(sc - m) : 0.f;
            float lsum = p;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
            ps[i * NP + j] = p;
            if (j == 0) linv[i] = 1.0f / lsum;
          }
          pw_sync();
          float acc[kQG];
#pragma unroll
          for (int i = 0; i < kQG; ++i) acc[i] = 0.f;
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            if (j < len) {
              const float v = vs[j * kHeadDim + pt];
#pragma unroll
              for (int i = 0; i < kQG; ++i) acc[i] = fmaf(ps[i * NP + j], v, acc[i]);
            }
          }
#pragma unroll
          for (int i = 0; i < kQG; ++i)
            if (i < nq)
              a.attn[(size_t)(base + q0 + i) * kQWidth + h * kHeadDim + pt] = __float2half_rn(acc[i] * linv[i]);
          pw_sync();
        }
        set_quiet(false);
      }
      grid_barrier();

      projection(l * 4 + 1, &a.xmap[2], merged);
      grid_barrier();
      norm_phase(X, l * 4 + 1, a.ffn_norm[l], N, T, srank[l * 3 + 1]);
      grid_barrier();
      projection(l * 4 + 2, &a.xmap[merged ? 1 : 0], merged);
      grid_barrier();
      projection(l * 4 + 3, &a.xmap[3], merged);
      grid_barrier();
      norm_phase(X, l * 4 + 3, l + 1 < a.n_layers ? a.attn_norm[l + 1] : a.output_norm, N, T, srank[l * 3 + 2]);
      grid_barrier();
    }

    // ---- mean pool over the valid merged rows + L2 (ops.ts:596-627) ----
    for (int b = cta; b < batch; b += G) {
      const int len = meta->tgt_len[b];
      const size_t base = (size_t)meta->tgt_off[b];
      float t[2][8];
      float ss[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = h * 1024 + pt * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) t[h][i] = 0.f;
        for (int p = 0; p < len; ++p) {
          float v[8];
          unpack8(__ldcg(reinterpret_cast<const uint4*>((a.exact ? a.nrm : a.nm) + (base + p) * kHidden + c)), v);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[h][i] = __fadd_rn(t[h][i], v[i]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          t[h][i] = __fdiv_rn(t[h][i], (float)len);
          ss[h] = __fadd_rn(ss[h], __fmul_rn(t[h][i], t[h][i]));
        }
      }
      const float inv = rsqrtf(row_sum_256(ss[0], ss[1], sh->red));
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float4* o = reinterpret_cast<float4*>(a.out + (size_t)b * kHidden + h * 1024 + pt * 8);
        o[0] = make_float4(t[h][0] * inv, t[h][1] * inv, t[h][2] * inv, t[h][3] * inv);
        o[1] = make_float4(t[h][4] * inv, t[h][5] * inv, t[h][6] * inv, t[h][7] * inv);
      }
    }
    // The last epilogue and norm copies have landed before the CTA may exit.
    if (pt == 0 && eph > 0) dev::mbar_wait(ebar, (eph - 1) & 1, err, 100000000ull);
    if (pt == 0 && nph > 0) dev::mbar_wait(rowbar, (nph - 1) & 1, err, 100000000ull);
    // TMA loads of X issued without a matching MMA (after an error) land too.
    if (pt == 0)
      for (int j = xit > kXStages ? xit - kXStages : 0; j < xit; ++j)
        dev::mbar_wait(xfull + 8 * (j % kXStages), (j / kXStages) & 1, err, 100000000ull);
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int forward_scratch_slots(int gate_up_slots, int residual_slots) {
  constexpr int kSlot = kFwdNP * 128 * 4, kXRing = kXStages * 4 * kFwdNP * 128;
  // norm_row stages [16 tiles][slots][128] f32 of the residual projection and
  // the f16 residual row from the start of the X ring onwards.
  const int stage = (kHidden / 128) * residual_slots * 128 * 4 + kHidden * 2;
  const int over = stage > kXRing ? (stage - kXRing + kSlot - 1) / kSlot : 0;
  return gate_up_slots > over ? gate_up_slots : over;
}

size_t forward_smem_bytes(int chunk_max, int scratch_slots, int max_segs, int n_layers) {
  constexpr int kXBytes = 4 * kFwdNP * 128;
  return 1024 + (size_t)kXStages * kXBytes + (size_t)scratch_slots * kFwdNP * 128 * 4 +
         (((size_t)kRawStages * chunk_max + 15) & ~15) + 8 * (2 * kRawStages + 2 * kASlabs + 2 * kXStages + 7) +
         ((sizeof(Shared) + 15) & ~15) + (size_t)max_segs * sizeof(FwdSeg) + sizeof(Meta) + 16 + kFwdNP * 128 * 4 +
         (size_t)n_layers * 4 * (4 + kFwdMaxTiles) + (size_t)n_layers * 3;
}

cudaError_t launch_forward(const FwdArgs& a, int grid, cudaStream_t s) {
  if (grid < 1 || a.max_slots < 1 || a.scratch_slots < 1) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64) return cudaErrorInvalidValue;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(forward_kernel<kFwdNP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = forward_smem_bytes(a.chunk_max, a.scratch_slots, a.max_segs, a.n_layers);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, forward_kernel<kFwdNP>, a);
}

cudaError_t forward_max_grid(size_t smem_bytes, int* grid) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(forward_kernel<kFwdNP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, forward_kernel<kFwdNP>, kThreads, smem_bytes);
  if (e != cudaSuccess) return e;
  // One CTA per SM: a second resident CTA could not allocate the full TMEM.
  *grid = per_sm >= 1 ? sms : 0;
  return cudaSuccess;
}

}  // namespace nemo
