// Dequant-fused projection GEMM on the tensor cores (tcgen05) for the
// batched regime (more than 64 tokens): Y[M x N] = X[M x K] . W[N x K]^T where
// W stays in its quantised blocks in HBM and is decoded to f16 in shared
// memory inside the GEMM. It replaces the reference's quantised matmul
// pipelines for batched work (src/webgpu/quant-matmul.ts:225-353,438-563,
// dispatched per src/webgpu/model.ts:313-320 for the projections of
// src/webgpu/model.ts:126-134); the decode is the reference's arithmetic
// (quantization.ts:19-74), so the MMA operands are exactly the effective f16
// weights every reference pipeline multiplies with.
//
// One CTA computes 128 * MB tokens x one 128-row weight tile of the tile-slab
// image (k_skinny.cu layout: chunk (tile, slab) = 128 rows x 256 columns, two
// 64-row format regions), over the whole K; each decoded W stage feeds MB
// accumulators (MB = 2 or 4 divide the decode work per FLOP):
//
//   D_b[128 tokens x 128 rows] += X_b[128 x 16] . W^T[16 x 128]   (f16 in, f32 in TMEM)
//
// Warp roles (480 threads):
//   warp 0      activation producer: K stages of X (MB x 128 x 64, 128B
//               swizzle) by TMA into an X ring
//   warp 14     weight producer: packed chunks by cp.async.bulk into a 2-deep
//               raw ring
//   warp 1      TMEM allocation + tcgen05.mma issue (converged warp, elected lane)
//   warps 2-9   decoders: thread = (weight row, quarter parity); each 64-column
//               quarter of a chunk is decoded straight into one stage of the
//               W ring in the canonical 128B-swizzled K-major layout
//   warps 10-13 epilogue: TMEM -> f16 rows, or SwiGLU of the tile's interleaved
//               64 gate + 64 up rows (ops.ts:74-89) into the 6144-wide output
// Every wait is bounded; a timeout sets the device error word and the CTA
// unwinds (drains its copies and MMAs, frees its TMEM) instead of hanging.
#include "tile_decode.cuh"

namespace nemo {
namespace {

using namespace tsd;

constexpr int kQThreads = 480;
constexpr int kQRaw = 2;              // packed chunks in flight
constexpr int kQOp = 128 * 64 * 2;    // one 128 x 64 f16 operand (16 KB)

template <int MB>
struct QCfg {
  static constexpr int kXStages = MB == 1 ? 6 : MB == 2 ? 3 : 2;  // X ring (MB operands per stage)
  static constexpr int kWStages = MB == 1 ? 4 : MB == 2 ? 3 : 2;  // decoded W quarters
  static constexpr uint32_t kTmemCols = 128 * MB;
};

template <int MB>
size_t gemm_q_smem_bytes(int chunk_max) {
  using C = QCfg<MB>;
  return 1024 + (size_t)(C::kXStages * MB + C::kWStages) * kQOp + (((size_t)kQRaw * chunk_max + 15) & ~(size_t)15) +
         8 * (2 * C::kXStages + 2 * C::kWStages + 2 * kQRaw + 1) + 16;
}

template <int MB>
__global__ void __launch_bounds__(kQThreads, 1)
    gemm_q_kernel(const __grid_constant__ CUtensorMap map_x, const uint8_t* __restrict__ packed,
                  const SkinnyTile* __restrict__ tiles, int slabs, int chunk_max, int mode, __half* y, int ldy,
                  const int* __restrict__ d_rows, int rows_value, uint32_t* err) {
  using C = QCfg<MB>;
  constexpr int kQXStages = C::kXStages, kQWStages = C::kWStages;
  constexpr uint32_t kQTmemCols = C::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  const int M = d_rows ? *d_rows : rows_value;
  const int m0 = blockIdx.y * 128 * MB;
  if (m0 >= M) return;  // uniform over the CTA
  const int tile = blockIdx.x;
  const uint32_t raw_s = dev::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_s + 1023u) & ~1023u) - raw_s);
  uint8_t* xst = smem;                     // 1024-aligned (SW128 operands)
  uint8_t* wst = xst + kQXStages * MB * kQOp;
  uint8_t* raw = wst + kQWStages * kQOp;
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + ((kQRaw * chunk_max + 15) & ~15));
  const uint32_t xfull = dev::smem_u32(bars), xempty = xfull + 8 * kQXStages;
  const uint32_t wfull = xempty + 8 * kQXStages, wempty = wfull + 8 * kQWStages;
  const uint32_t rfull = wempty + 8 * kQWStages, rempty = rfull + 8 * kQRaw, accum = rempty + 8 * kQRaw;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kQXStages + 2 * kQWStages + 2 * kQRaw + 1);
  const uint32_t xbase = dev::smem_u32(xst), wbase = dev::smem_u32(wst);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const SkinnyTile ti = tiles[tile];
  const int KT = slabs * 4;

  if (threadIdx.x == 0) {
    dev::prefetch_tmap(&map_x);
    for (int s = 0; s < kQXStages; ++s) {
      dev::mbar_init(xfull + 8 * s, 1);
      dev::mbar_init(xempty + 8 * s, 1);
    }
    for (int s = 0; s < kQWStages; ++s) {
      dev::mbar_init(wfull + 8 * s, 128);  // one quarter's decoder threads
      dev::mbar_init(wempty + 8 * s, 1);
    }
    for (int s = 0; s < kQRaw; ++s) {
      dev::mbar_init(rfull + 8 * s, 1);
      dev::mbar_init(rempty + 8 * s, 256);
    }
    dev::mbar_init(accum, 1);
    dev::fence_mbar_init();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), kQTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint8_t* chunk0 = packed + ti.offset;

  if (warp == 0) {
    // ------------------------------------------------------------ X producer
    int issued = 0;
    for (int kt = 0; kt < KT; ++kt) {
      const int st = kt % kQXStages;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(xempty + 8 * st, ((kt / kQXStages) & 1) ^ 1, err))) break;
      if (dev::elect_one()) {
        dev::mbar_arrive_expect_tx(xfull + 8 * st, MB * kQOp);
#pragma unroll
        for (int b = 0; b < MB; ++b)  // rows past the map read the zero fill
          dev::tma_load_2d(xbase + (st * MB + b) * kQOp, &map_x, kt * 64, m0 + 128 * b, xfull + 8 * st);
      }
      __syncwarp();
      ++issued;
    }
    // Every issued copy lands before shared memory is released.
    for (int i = issued > kQXStages ? issued - kQXStages : 0; i < issued; ++i)
      dev::mbar_wait(xfull + 8 * (i % kQXStages), (i / kQXStages) & 1, err, 100000000ull);
  } else if (warp == 14) {
    // ------------------------------------------------------------ W producer
    int issued = 0;
    for (int s = 0; s < slabs; ++s) {
      const int rs = s % kQRaw;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(rempty + 8 * rs, ((s / kQRaw) & 1) ^ 1, err))) break;
      if (dev::elect_one()) {
        dev::mbar_arrive_expect_tx(rfull + 8 * rs, ti.chunk_bytes);
        dev::bulk_load(dev::smem_u32(raw + rs * chunk_max), chunk0 + (size_t)s * ti.chunk_bytes, ti.chunk_bytes,
                       rfull + 8 * rs);
      }
      __syncwarp();
      ++issued;
    }
    for (int i = issued > kQRaw ? issued - kQRaw : 0; i < issued; ++i)
      dev::mbar_wait(rfull + 8 * (i % kQRaw), (i / kQRaw) & 1, err, 100000000ull);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = dev::make_idesc_f16(128, 128);  // per accumulator
    for (int kt = 0; kt < KT; ++kt) {
      const int xs = kt % kQXStages, ws = kt % kQWStages;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(xfull + 8 * xs, (kt / kQXStages) & 1, err) &&
                                       dev::mbar_wait(wfull + 8 * ws, (kt / kQWStages) & 1, err)))
        break;
      dev::tc_fence_after();
      const uint32_t xa = xbase + xs * MB * kQOp, wa = wbase + ws * kQOp;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (dev::elect_one()) {
          const uint64_t bd = dev::make_sw128_desc(wa + kk * 32);
#pragma unroll
          for (int b = 0; b < MB; ++b) {
            const uint64_t ad = dev::make_sw128_desc(xa + b * kQOp + kk * 32);
            dev::tc_mma_f16(tmem + 128 * b, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
        }
        __syncwarp();
      }
      if (dev::elect_one()) {
        dev::tc_commit(xempty + 8 * xs);
        dev::tc_commit(wempty + 8 * ws);
      }
      __syncwarp();
    }
    if (dev::elect_one()) dev::tc_commit(accum);
    __syncwarp();
    dev::mbar_wait(accum, 0, err, 100000000ull);  // all MMAs retired before TMEM is released
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------ decoders
    const int dt = threadIdx.x - 64;
    const int r = dt & 127, par = dt >> 7;  // weight row; quarters par and par + 2
    const int half = r >> 6, rr = r & 63;   // half is uniform within a warp
    const int fmt = ti.fmt[half];
    const int roff = half ? region_bytes(ti.fmt[0]) : 0;
    for (int s = 0; s < slabs; ++s) {
      const int rs = s % kQRaw;
      if (!__all_sync(0xffffffffu, dev::mbar_wait(rfull + 8 * rs, (s / kQRaw) & 1, err))) break;
      const uint8_t* region = raw + rs * chunk_max + roff;
      const uint8_t* blk = region + rr * (fmt == kSegQ6K ? 208 : 144);
      const uint16_t d6 = fmt == kSegQ6K ? *reinterpret_cast<const uint16_t*>(region + 64 * 208 + rr * 2) : 0;
      bool ok = true;
#pragma unroll 1
      for (int qq = 0; qq < 2; ++qq) {
        const int q = par + 2 * qq, kt = 4 * s + q, ws = kt % kQWStages;
        if (!__all_sync(0xffffffffu, dev::mbar_wait(wempty + 8 * ws, ((kt / kQWStages) & 1) ^ 1, err))) {
          ok = false;
          break;
        }
        const SmemTileSink sink{wst + ws * kQOp, r};
        if (fmt == kSegQ4K) decode_q4k(blk, q, sink);
        else if (fmt == kSegQ6K) decode_q6k(blk, d6, q, sink);
        else decode_q40(blk, q, sink);
        dev::fence_proxy_async_smem();  // generic stores -> tensor core operand reads
        dev::mbar_arrive(wfull + 8 * ws);
      }
      if (!ok) break;
      dev::mbar_arrive(rempty + 8 * rs);
    }
  } else if (warp < 14) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const bool got = __all_sync(0xffffffffu, dev::mbar_wait(accum, 0, err));  // warp-uniform: tcgen05.ld is collective
    if (got) dev::tc_fence_after();
#pragma unroll 1
    for (int b = 0; b < MB && got; ++b) {
      const int row = m0 + 128 * b + quarter * 32 + lane;
      const uint32_t base = tmem + ((uint32_t)(quarter * 32) << 16) + 128 * b;
      if (mode == kSkinnySwiglu) {
        // columns 0-63: gate rows 64 * tile + c; 64-127: the matching up rows
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t g[32], u[32];
          dev::tmem_ld_32x32b_x32(base + c, g);
          dev::tmem_ld_32x32b_x32(base + 64 + c, u);
          dev::tc_wait_ld();
          if (row < M) {
            uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * ldy + tile * 64 + c);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float o[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float gh = __half2float(__float2half_rn(__uint_as_float(g[v * 8 + j])));
                const float uh = __half2float(__float2half_rn(__uint_as_float(u[v * 8 + j])));
                const float silu = __fdiv_rn(gh, __fadd_rn(1.0f, expf(-gh)));
                o[j] = __fmul_rn(silu, uh);
              }
              uint4 w;
              __half2* h = reinterpret_cast<__half2*>(&w);
#pragma unroll
              for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
              dst[v] = w;
            }
          }
        }
      } else if (mode == kSkinnyF32) {
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t v32[32];
          dev::tmem_ld_32x32b_x32(base + c, v32);
          dev::tc_wait_ld();
          if (row < M) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<float*>(y) + (size_t)row * ldy + tile * 128 + c);
#pragma unroll
            for (int v = 0; v < 8; ++v) dst[v] = make_uint4(v32[4 * v], v32[4 * v + 1], v32[4 * v + 2], v32[4 * v + 3]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t v32[32];
          dev::tmem_ld_32x32b_x32(base + c, v32);
          dev::tc_wait_ld();
          if (row < M) {
            uint4* dst = reinterpret_cast<uint4*>(y + (size_t)row * ldy + tile * 128 + c);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              __half2* h = reinterpret_cast<__half2*>(&w);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                h[j] = __floats2half2_rn(__uint_as_float(v32[v * 8 + 2 * j]), __uint_as_float(v32[v * 8 + 2 * j + 1]));
              dst[v] = w;
            }
          }
        }
      }
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, kQTmemCols);
  }
}

}  // namespace

namespace {
template <int MB>
cudaError_t launch_mb(const CUtensorMap* map_x, const uint8_t* packed, const SkinnyTile* tiles, int n_tiles,
                      int slabs, int chunk_max, int mode, __half* y, int ldy, const int* d_rows, int max_rows,
                      uint32_t* err, cudaStream_t s) {
  const size_t smem = gemm_q_smem_bytes<MB>(chunk_max);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_q_kernel<MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(n_tiles, (max_rows + 128 * MB - 1) / (128 * MB));
  gemm_q_kernel<MB><<<grid, kQThreads, smem, s>>>(*map_x, packed, tiles, slabs, chunk_max, mode, y, ldy, d_rows,
                                                   max_rows, err);
  return cudaGetLastError();
}
}  // namespace

// The most tokens per CTA (512, 256 or 128) that still leaves at least two
// CTAs per SM (148 SMs): fewer decodes of each weight tile per token.
cudaError_t launch_gemm_q(const CUtensorMap* map_x, const uint8_t* packed, const SkinnyTile* tiles, int n_tiles,
                          int slabs, int chunk_max, int mode, __half* y, int ldy, const int* d_rows, int max_rows,
                          uint32_t* err, cudaStream_t s) {
  if (n_tiles < 1 || slabs < 1 || chunk_max < 1 || max_rows < 1 ||
      (mode != kSkinnyPlain && mode != kSkinnySwiglu && mode != kSkinnyF32))
    return cudaErrorInvalidValue;
  if ((long long)n_tiles * ((max_rows + 511) / 512) >= 2 * 148)
    return launch_mb<4>(map_x, packed, tiles, n_tiles, slabs, chunk_max, mode, y, ldy, d_rows, max_rows, err, s);
  if ((long long)n_tiles * ((max_rows + 255) / 256) >= 2 * 148)
    return launch_mb<2>(map_x, packed, tiles, n_tiles, slabs, chunk_max, mode, y, ldy, d_rows, max_rows, err, s);
  return launch_mb<1>(map_x, packed, tiles, n_tiles, slabs, chunk_max, mode, y, ldy, d_rows, max_rows, err, s);
}

}  // namespace nemo
