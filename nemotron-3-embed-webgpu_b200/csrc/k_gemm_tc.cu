// Projection GEMM on the 5th-generation tensor cores (tcgen05) for the
// batched regime: Y[M x N] = X[M x K] . W[N x K]^T with f16 operands and f32
// accumulation in tensor memory. It replaces the reference's quantised matmul
// pipelines (src/webgpu/quant-matmul.ts:438-563) for the projections of
// src/webgpu/model.ts:126-134; the weights are the effective f16 values of the
// quantised blocks, decoded once at load.
//
// Persistent: one CTA per SM walks its 128 x BN output tiles; two TMEM
// accumulators let the epilogue of one tile overlap the MMAs of the next.
// Warp roles (320 threads):
//   warp 0      TMA producer: 64-wide K slabs of A (128 x 64) and B (BN x 64)
//               into a STAGES-deep ring that runs on across tiles, 128-byte
//               swizzled, mbarrier complete_tx
//   warp 1      TMEM allocator + tcgen05.mma issuer (M=128, N=BN, K=16 per
//               instruction; converged warp, elected lane), tcgen05.commit
//               frees each stage
//   warps 2..9  epilogue: tcgen05.ld 32x32b (one row per thread), then an f16
//               store, RoPE (QKV: Q/K pairs rotated into the attention
//               inputs, ops.ts:168-194) or SwiGLU (gate/up: the B tile holds
//               BN/2 gate rows then the matching BN/2 up rows, ops.ts:74-89).
//               Warps 2-5 take the first half of the tile's columns, warps
//               6-9 (same TMEM lane quarters) the second: with one tile per
//               CTA (few tokens) nothing overlaps the epilogue, so its length
//               is on the critical path.
// Every mbarrier wait is bounded (2 s); a timeout sets the device error word,
// drains what this CTA has in flight and frees its TMEM before returning.
#include <cudaTypedefs.h>

#include <algorithm>

#include "kernels.cuh"

namespace nemo {
namespace {

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int STAGES = BN >= 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators: epilogue of tile i || MMAs of tile i + 1
  static constexpr int STAGE_OUT = 4 * 32 * 128;  // per epilogue warp: 32 rows x 64 f16 (head-parallel stores)
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + STAGE_OUT;
};

// (even, odd) column pairs of a 32-column accumulator chunk rounded to f16,
// rotated by the 16 (cos, sin) table pairs cs, rounded again (as the
// f16-stored QKV would be, k_misc.cu rope_kernel), packed as 16 half2.
__device__ __forceinline__ void rope_pack(const uint32_t (&r)[32], const float4 (&cs)[8], uint32_t (&o)[16]) {
  const float* tcs = reinterpret_cast<const float*>(cs);
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    const float even = __half2float(__float2half_rn(__uint_as_float(r[2 * p])));
    const float odd = __half2float(__float2half_rn(__uint_as_float(r[2 * p + 1])));
    const float2 tc = make_float2(tcs[2 * p], tcs[2 * p + 1]);
    const float first = __fsub_rn(__fmul_rn(even, tc.x), __fmul_rn(odd, tc.y));
    const float second = __fadd_rn(__fmul_rn(even, tc.y), __fmul_rn(odd, tc.x));
    __half2 h = __halves2half2(__float2half_rn(first), __float2half_rn(second));
    o[p] = *reinterpret_cast<uint32_t*>(&h);
  }
}

__device__ __forceinline__ void plain_pack(const uint32_t (&r)[32], uint32_t (&o)[16]) {
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    __half2 h = __floats2half2_rn(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
    o[p] = *reinterpret_cast<uint32_t*>(&h);
  }
}

// Persistent: CTA c takes tiles c, c + grid, ... of the (m tile, n tile)
// grid in n-fastest order; M (valid token rows) is read on the device.
template <int BN>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, __half* y,
                   int ldy, const int* __restrict__ d_rows, int k, int n_tiles, uint32_t* err, GemmEpi e) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const int M = *d_rows;
  const int KT = k / C::BK;
  // Work units: (K split, m tile, n tile), n fastest; one split unless
  // e.part asks for K-split partial sums (plain mode).
  const int tiles = (M + C::BM - 1) / C::BM * n_tiles;
  const int splits = e.part ? gemm_ksplit((M + C::BM - 1) / C::BM, n_tiles, KT, (int)gridDim.x) : 1;
  const int total = tiles * splits;
  if (e.splits_out && blockIdx.x == 0 && threadIdx.x == 0) *e.splits_out = splits;
  // 1024-byte alignment of the shared-window address (the 128-byte swizzle
  // pattern repeats every 1024 bytes and the descriptors assume base offset 0).
  const uint32_t raw_s = dev::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  const uint32_t full0 = dev::smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * C::STAGES;
  const uint32_t tfull = empty0 + 8 * C::STAGES, tempty = tfull + 16, fin = tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::STAGES + 5);
  const uint32_t sbase = dev::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    dev::prefetch_tmap(&map_a);
    dev::prefetch_tmap(&map_b);
    for (int s = 0; s < C::STAGES; ++s) {
      dev::mbar_init(full0 + 8 * s, 1);
      dev::mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      dev::mbar_init(tfull + 8 * b, 1);
      dev::mbar_init(tempty + 8 * b, 256);
    }
    dev::mbar_init(fin, 1);
    dev::fence_mbar_init();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), C::TMEM_COLS);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // Converged warp; the elected lane issues the copies. The stage ring runs
    // on across tiles.
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int sp = t / tiles, tt = t % tiles;
      const int m0 = (tt / n_tiles) * C::BM, nt = tt % n_tiles, n0 = nt * BN;
      const int kt1 = (sp + 1) * KT / splits;
      for (int kt = sp * KT / splits; kt < kt1; ++kt, ++it) {
        const int s = it % C::STAGES;
        if (!__all_sync(0xffffffffu, dev::mbar_wait(empty0 + 8 * s, ((it / C::STAGES) & 1) ^ 1, err))) {
          ok = false;
          break;
        }
        const uint32_t sa = sbase + s * C::STAGE_BYTES;
        if (dev::elect_one()) {
          dev::mbar_arrive_expect_tx(full0 + 8 * s, C::STAGE_BYTES);
          dev::tma_load_2d(sa, &map_a, kt * C::BK, m0, full0 + 8 * s);
          if (e.mode == kSkinnySwiglu) {
            // map_b box is BN/2 rows: gate rows, then the matching up rows
            dev::tma_load_2d(sa + C::A_BYTES, &map_b, kt * C::BK, nt * (BN / 2), full0 + 8 * s);
            dev::tma_load_2d(sa + C::A_BYTES + (BN / 2) * 128, &map_b, kt * C::BK, kInter + nt * (BN / 2),
                             full0 + 8 * s);
          } else {
            dev::tma_load_2d(sa + C::A_BYTES, &map_b, kt * C::BK, n0, full0 + 8 * s);
          }
        }
        __syncwarp();
      }
    }
    // Drain: every issued copy has landed before shared memory is released.
    for (int i = it > C::STAGES ? it - C::STAGES : 0; i < it; ++i)
      dev::mbar_wait(full0 + 8 * (i % C::STAGES), (i / C::STAGES) & 1, err, 100000000ull);
  } else if (warp == 1) {
    // Converged warp; the elected lane (lane 0) issues every MMA and commit.
    constexpr uint32_t idesc = dev::make_idesc_f16(C::BM, BN);
    int it = 0, i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
      const int buf = i & 1;
      const int sp = t / tiles, kt0 = sp * KT / splits, kt1 = (sp + 1) * KT / splits;
      // the epilogue has drained this accumulator (tile i - 2)
      if (!__all_sync(0xffffffffu, dev::mbar_wait(tempty + 8 * buf, ((i >> 1) & 1) ^ 1, err))) break;
      dev::tc_fence_after();
      for (int kt = kt0; kt < kt1; ++kt, ++it) {
        const int s = it % C::STAGES;
        if (!__all_sync(0xffffffffu, dev::mbar_wait(full0 + 8 * s, (it / C::STAGES) & 1, err))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t sa = sbase + s * C::STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk) {
          if (dev::elect_one()) {
            const uint64_t ad = dev::make_sw128_desc(sa + kk * 32);
            const uint64_t bd = dev::make_sw128_desc(sa + C::A_BYTES + kk * 32);
            dev::tc_mma_f16(tmem + buf * BN, ad, bd, idesc, (kt != kt0 || kk != 0) ? 1u : 0u);
          }
          __syncwarp();
        }
        if (dev::elect_one()) dev::tc_commit(empty0 + 8 * s);
        __syncwarp();
      }
      if (!ok) break;
      if (dev::elect_one()) dev::tc_commit(tfull + 8 * buf);
      __syncwarp();
    }
    if (dev::elect_one()) dev::tc_commit(fin);
    __syncwarp();
    // All MMAs of this CTA have retired before TMEM is released below.
    dev::mbar_wait(fin, 0, err, 100000000ull);
  } else {
    const int quarter = warp & 3, group = (warp - 2) >> 2;
    uint8_t* stage = smem + C::STAGES * C::STAGE_BYTES + 256 + quarter * (32 * 128);  // group 0 only
    int i = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      const int buf = i & 1;
      const int sp = t / tiles, tt = t % tiles;
      const int m0 = (tt / n_tiles) * C::BM, nt = tt % n_tiles, n0 = nt * BN;
      const int row = m0 + quarter * 32 + lane;
      // warp-uniform: tcgen05.ld is collective
      if (!__all_sync(0xffffffffu, dev::mbar_wait(tfull + 8 * buf, (i >> 1) & 1, err))) break;
      dev::tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      if (e.mode == kSkinnySwiglu) {
        // out[row][g] = f16(silu(f16 gate) * f16 up) for the tile's BN/2 outputs
#pragma unroll 1
        for (int c = group * (BN / 4); c < (group + 1) * (BN / 4); c += 32) {
          uint32_t g[32], u[32];
          dev::tmem_ld_32x32b_x32(tbase + c, g);
          dev::tmem_ld_32x32b_x32(tbase + BN / 2 + c, u);
          dev::tc_wait_ld();
          if (row < M) {
            uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * ldy + nt * (BN / 2) + c);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float o[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float gh = __half2float(__float2half_rn(__uint_as_float(g[v * 8 + j])));
                const float uh = __half2float(__float2half_rn(__uint_as_float(u[v * 8 + j])));
                o[j] = __fmul_rn(__fdiv_rn(gh, __fadd_rn(1.0f, expf(-gh))), uh);
              }
              uint4 w;
              __half2* h = reinterpret_cast<__half2*>(&w);
#pragma unroll
              for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
              dst[v] = w;
            }
          }
        }
      } else {
        // RoPE: position of this token row within its request (ops.ts:188)
        int pos = 0;
        if (e.mode == kSkinnyRope && row < M) {
          const int* off = e.merged ? e.meta->tgt_off : e.meta->src_off;
          int b = 0;
          while (b + 1 < e.meta->batch && row >= off[b + 1]) ++b;
          pos = row - off[b] + e.hp.row0;  // row0: shard offset of a head-parallel run, else 0
        }
        // The 32 table floats (16 cos/sin pairs, 128 contiguous bytes) of a
        // chunk's rotated columns are loaded one chunk ahead, so their latency
        // overlaps the previous chunk instead of following the TMEM load.
        const bool rot_tile = e.mode == kSkinnyRope && row < M;
        auto load_cs = [&](int c, float4 (&cs)[8]) {
          const int col0 = n0 + c * 32;
          if (rot_tile && c < BN / 32 && col0 < kQWidth + kKVWidth) {
            const float4* src = reinterpret_cast<const float4*>(e.rope + ((size_t)pos * 64 + ((col0 & 127) >> 1)) * 2);
#pragma unroll
            for (int v = 0; v < 8; ++v) cs[v] = __ldg(src + v);
          }
        };
        // 32-column chunks of this warp's group; a head-parallel run's staged
        // peer stores pair chunks, so group 0 takes the whole tile there.
        const int c0 = e.hp.n_dev ? (group ? BN / 32 : 0) : group * (BN / 64);
        const int c1 = e.hp.n_dev ? BN / 32 : (group + 1) * (BN / 64);
        float4 cs_cur[8], cs_nxt[8];
        load_cs(c0, cs_cur);
#pragma unroll 1
        for (int c = c0; c < c1; ++c) {
          const int col0 = n0 + c * 32;
          uint32_t r[32];
          dev::tmem_ld_32x32b_x32(tbase + c * 32, r);
          load_cs(c + 1, cs_nxt);
          dev::tc_wait_ld();
          // no early exit: every lane reaches the next (warp-collective) tcgen05.ld
          if (e.hp.n_dev) {
            // Head-parallel QKV (warp-uniform branch): the 32 x 32 chunk goes
            // through this warp's shared-memory stage; every second chunk the
            // warp writes the staged 32 rows x 64 columns out as 128-byte row
            // segments (8 lanes per row), so each peer store is a whole line.
            uint32_t o[16];
            if (row < M) {
              if (col0 < kQWidth + kKVWidth)
                rope_pack(r, cs_cur, o);
              else
                plain_pack(r, o);
            } else {
#pragma unroll
              for (int p = 0; p < 16; ++p) o[p] = 0u;
            }
            // 16-byte unit u of row `lane` at unit u ^ (lane & 7): conflict-free both ways
#pragma unroll
            for (int v = 0; v < 4; ++v)
              *reinterpret_cast<uint4*>(stage + lane * 128 + ((((c & 1) * 4 + v) ^ (lane & 7)) * 16)) =
                  make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            if (c & 1) {
              __syncwarp();
              int j, b, dc;
              hp_qkv_route(col0 - 32, e.hp.n_dev, &j, &b, &dc);  // 64 columns within one head
              const int w = b == 0 ? kQWidth / e.hp.n_dev : kKVWidth / e.hp.n_dev;
              __half *dst = nullptr, *cdst = nullptr;
#pragma unroll
              for (int i = 0; i < 8; ++i)  // selects, no local copy of the pointer arrays
                if (i == j) {
                  dst = b == 0 ? e.hp.q[i] : b == 1 ? e.hp.k[i] : e.hp.v[i];
                  cdst = b == 1 ? e.hp.kc[i] : e.hp.vc[i];
                }
              const int u = lane & 7;
#pragma unroll
              for (int it = 0; it < 8; ++it) {
                const int rr = it * 4 + (lane >> 3);
                const int lrow = m0 + quarter * 32 + rr;
                if (lrow < M) {
                  // one request starting at local row 0: position = row0 + local row
                  const int p = e.hp.row0 + lrow;
                  const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((u ^ (rr & 7)) * 16));
                  *reinterpret_cast<uint4*>(dst + (size_t)p * w + dc + u * 8) = val;
                  if (e.hp.sample && b > 0 && p % kSampleStride == 0)
                    *reinterpret_cast<uint4*>(cdst + (size_t)(p / kSampleStride) * w + dc + u * 8) = val;
                }
              }
              __syncwarp();
            }
          } else if (row < M && e.mode == kSkinnyRope && col0 < kQWidth + kKVWidth) {
            uint32_t o[16];
            rope_pack(r, cs_cur, o);
            __half* dst = col0 < kQWidth ? e.q + (size_t)row * kQWidth + col0
                                         : e.k + (size_t)row * kKVWidth + (col0 - kQWidth);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              reinterpret_cast<uint4*>(dst)[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
          } else if (row < M && splits > 1) {
            // f32 partial sums of split sp (summed by the consumer in split order)
            float4* dst = reinterpret_cast<float4*>(e.part + ((size_t)sp * M + row) * (n_tiles * BN) + col0);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          } else if (row < M) {
          uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * ldy + col0);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 u;
            __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              h[j] = __floats2half2_rn(__uint_as_float(r[v * 8 + 2 * j]), __uint_as_float(r[v * 8 + 2 * j + 1]));
            dst[v] = u;
          }
          }
#pragma unroll
          for (int v = 0; v < 8; ++v) cs_cur[v] = cs_nxt[v];
        }
      }
      dev::tc_fence_before();
      dev::mbar_arrive(tempty + 8 * buf);
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap* ma, const CUtensorMap* mb, __half* y, int ldy, const int* d_rows,
                      int max_rows, int n, int k, uint32_t* err, const GemmEpi& ep, cudaStream_t s) {
  using C = GemmCfg<BN>;
  static bool configured[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  // One CTA per SM (shared memory and TMEM allow one), never more than tiles.
  const int n_tiles = n / BN;
  const long long tiles = (long long)((max_rows + C::BM - 1) / C::BM) * n_tiles;
  // With K-split partial sums every SM takes units (gemm_ksplit sees the grid).
  const int grid = ep.part ? sms[dev] : (int)std::min<long long>(sms[dev], std::max<long long>(tiles, 1));
  gemm_tc_kernel<BN><<<grid, 320, C::SMEM, s>>>(*ma, *mb, y, ldy, d_rows, k, n_tiles, err, ep);
  return cudaGetLastError();
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

cudaError_t launch_gemm_tc_epi(const CUtensorMap* ma, const CUtensorMap* mb, __half* y, int ldy, const int* d_rows,
                               int max_rows, int n, int k, int bn, const GemmEpi& ep, uint32_t* err, cudaStream_t s) {
  if (k % 64 != 0 || n % bn != 0) return cudaErrorInvalidValue;
  if (ep.mode == kSkinnySwiglu && (bn < 128 || n != 2 * kInter)) return cudaErrorInvalidValue;
  if (ep.mode == kSkinnyRope && (n != kQKVWidth || !ep.meta || !ep.rope || (!ep.hp.n_dev && (!ep.q || !ep.k))))
    return cudaErrorInvalidValue;
  if (ep.hp.n_dev) {
    const int nd = ep.hp.n_dev;
    if (ep.mode != kSkinnyRope || (nd != 2 && nd != 4 && nd != 8) || ep.hp.row0 < 0) return cudaErrorInvalidValue;
    for (int i = 0; i < nd; ++i)
      if (!ep.hp.q[i] || !ep.hp.k[i] || !ep.hp.v[i] || (ep.hp.sample && (!ep.hp.kc[i] || !ep.hp.vc[i])))
        return cudaErrorInvalidValue;
  }
  if ((ep.part != nullptr) != (ep.splits_out != nullptr) || (ep.part && ep.mode != kSkinnyPlain))
    return cudaErrorInvalidValue;
  switch (bn) {
    case 64: return launch_bn<64>(ma, mb, y, ldy, d_rows, max_rows, n, k, err, ep, s);
    case 128: return launch_bn<128>(ma, mb, y, ldy, d_rows, max_rows, n, k, err, ep, s);
    case 256: return launch_bn<256>(ma, mb, y, ldy, d_rows, max_rows, n, k, err, ep, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm_tc(const CUtensorMap* ma, const CUtensorMap* mb, __half* y, int ldy, const int* d_rows,
                           int max_rows, int n, int k, int bn, uint32_t* err, cudaStream_t s) {
  return launch_gemm_tc_epi(ma, mb, y, ldy, d_rows, max_rows, n, k, bn, GemmEpi{}, err, s);
}

int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                  uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return kErrCuda;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return kErrCuda;
  }
  return kOk;
}

}  // namespace nemo
