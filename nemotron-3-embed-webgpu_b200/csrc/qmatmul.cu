// Standalone quantised matmul: Y[m x n] (f32) = X[m x k] (f16) . W[n x k]^T,
// W in GGUF Q4_K / Q6_K / Q4_0 row-major blocks or the q4_0-tile32-compact
// layout. The reference's QuantMatmulKernel (src/webgpu/quant-matmul.ts:438-563)
// takes the same operands: one weight buffer in GGUF or tile32 layout, an
// [m x k] activation buffer, K divisible by 256 (quant-matmul.ts:513).
//
// Like the model load (model.cu build_tile_slab), the weights are first
// re-tiled into the tile-slab image the projection kernels stream: 128-row
// tiles x 256-column slabs, chunk (tile, slab) contiguous, holding two 64-row
// regions (Q4_K 144 B per row; Q6_K 208 B per row then 64 f16 scales; Q4_0 and
// tile32 as 8 f16 scales + 128 quant bytes per row). Here the re-tile runs on
// the device. The matmul then runs the same dequant-fused tcgen05 kernels as
// the forward: the split-K small-token kernel (k_skinny.cu) for m <= 64, the
// batched dequant-fused GEMM (k_gemm_q.cu) above, both with f32 stores.
//
// Image: [SkinnyTile table of n/128 entries, padded to 256 B][chunks].
#include <algorithm>

#include "runtime.h"
#include "tile_decode.cuh"

namespace nemo {
namespace {

constexpr size_t kTableAlign = 256;

__host__ __device__ inline int q_chunk_bytes(int fmt) { return fmt == kSegQ6K ? 2 * 64 * 210 : 2 * 64 * 144; }

__host__ __device__ inline size_t q_table_bytes(int n) {
  return ((size_t)(n / 128) * sizeof(SkinnyTile) + kTableAlign - 1) / kTableAlign * kTableAlign;
}

// Thread per (row, slab): copies that row's block(s) of the slab into its
// region row (layout of model.cu build_tile_slab, non-interleaved tiles).
__global__ void retile_kernel(int fmt, const uint8_t* __restrict__ src, int n, int k, uint8_t* __restrict__ image) {
  const int slabs = k / 256, kb32 = k / 32;
  const int chunk = q_chunk_bytes(fmt), region = chunk / 2;
  SkinnyTile* table = reinterpret_cast<SkinnyTile*>(image);
  uint8_t* chunks = image + q_table_bytes(n);
  const int total = n * slabs;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int row = i / slabs, s = i % slabs;
    const int tile = row >> 7, half = (row >> 6) & 1, rr = row & 63;
    if (s == 0 && (row & 127) == 0) {
      SkinnyTile t = {};
      t.offset = (uint32_t)((size_t)tile * slabs * chunk);
      t.chunk_bytes = (uint32_t)chunk;
      t.fmt[0] = t.fmt[1] = (uint8_t)(fmt == kSegQ40Tile32 ? kSegQ40 : fmt);
      table[tile] = t;
    }
    uint8_t* reg = chunks + ((size_t)tile * slabs + s) * chunk + (size_t)half * region;
    if (fmt == kSegQ4K) {
      const uint4* a = reinterpret_cast<const uint4*>(src + ((size_t)row * slabs + s) * 144);
      uint4* b = reinterpret_cast<uint4*>(reg + rr * 144);
#pragma unroll
      for (int j = 0; j < 9; ++j) b[j] = a[j];
    } else if (fmt == kSegQ6K) {
      const uint8_t* a = src + ((size_t)row * slabs + s) * 210;
      uint8_t* b = reg + rr * 208;
      for (int j = 0; j < 208; ++j) b[j] = a[j];
      reg[64 * 208 + rr * 2] = a[208];
      reg[64 * 208 + rr * 2 + 1] = a[209];
    } else {
      uint8_t* dst = reg + rr * 144;
      for (int b = 0; b < 8; ++b) {
        const uint8_t* blk;
        const uint8_t* qs;
        if (fmt == kSegQ40) {  // GGUF 18-byte blocks: f16 d, 16 quant bytes
          blk = src + ((size_t)row * kb32 + s * 8 + b) * 18;
          qs = blk + 2;
        } else {  // tile32: [n/32][k/32][32 rows][20 B] (format.ts:84-97)
          blk = src + ((((size_t)(row / 32)) * kb32 + s * 8 + b) * 32 + (row % 32)) * 20;
          qs = blk + 4;
        }
        dst[2 * b] = blk[0];
        dst[2 * b + 1] = blk[1];
        for (int j = 0; j < 16; ++j) dst[16 + b * 16 + j] = qs[j];
      }
    }
  }
}

// Writes each finished 16-byte chunk c of a decoded quarter (values 8c..8c+7)
// to a row-major f16 matrix row.
struct GlobalRowSink {
  __half* row;  // first column of the quarter
  __device__ __forceinline__ void operator()(int c, uint4 v) const { *reinterpret_cast<uint4*>(row + 8 * c) = v; }
};

// Thread per (tile, slab, row, quarter): the exact decode of one 64-value
// quarter of one row of a tile-slab image into the row-major f16 matrix
// (gate/up tiles: rows 0-63 are gate rows 64t.., rows 64-127 up rows n/2 + 64t..).
__global__ void decode_image_kernel(const uint8_t* __restrict__ chunks, const SkinnyTile* __restrict__ tiles,
                                    int ntiles, int slabs, int interleave, int n, int k, __half* __restrict__ w16) {
  using namespace tsd;
  const long long total = (long long)ntiles * slabs * 512;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i & 3), row = (int)((i >> 2) & 127);
    const long long ts = i >> 9;
    const int slab = (int)(ts % slabs), tile = (int)(ts / slabs);
    const SkinnyTile ti = tiles[tile];
    const int half = row >> 6, rr = row & 63, fmt = ti.fmt[half];
    const uint8_t* region = chunks + ti.offset + (size_t)slab * ti.chunk_bytes + (half ? region_bytes(ti.fmt[0]) : 0);
    const uint8_t* blk = region + rr * (fmt == kSegQ6K ? 208 : 144);
    const int mrow = interleave ? (half ? n / 2 + tile * 64 + rr : tile * 64 + rr) : tile * 128 + row;
    const GlobalRowSink sink{w16 + (size_t)mrow * k + slab * 256 + q * 64};
    if (fmt == kSegQ4K) decode_q4k(blk, q, sink);
    else if (fmt == kSegQ6K) decode_q6k(blk, *reinterpret_cast<const uint16_t*>(region + 64 * 208 + rr * 2), q, sink);
    else decode_q40(blk, q, sink);
  }
}

}  // namespace

cudaError_t launch_decode_image(const uint8_t* chunks, const SkinnyTile* tiles, int ntiles, int slabs, bool interleave,
                                int n, int k, __half* w16, cudaStream_t s) {
  if (ntiles < 1 || slabs < 1 || n != ntiles * 128 || k != slabs * 256) return cudaErrorInvalidValue;
  const long long total = (long long)ntiles * slabs * 512;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 148 * 16);
  decode_image_kernel<<<blocks, 256, 0, s>>>(chunks, tiles, ntiles, slabs, interleave ? 1 : 0, n, k, w16);
  return cudaGetLastError();
}

size_t qmatmul_image_bytes(int fmt, int n, int k) {
  if (fmt < kSegQ4K || fmt > kSegQ40Tile32 || n < 128 || n % 128 || k < 256 || k % 256) return 0;
  return q_table_bytes(n) + (size_t)(n / 128) * (k / 256) * q_chunk_bytes(fmt);
}

cudaError_t launch_qmatmul_retile(int fmt, const uint8_t* src, int n, int k, uint8_t* image, cudaStream_t s) {
  if (!qmatmul_image_bytes(fmt, n, k)) return cudaErrorInvalidValue;
  const int total = n * (k / 256);
  retile_kernel<<<(total + 255) / 256, 256, 0, s>>>(fmt, src, n, k, image);
  return cudaGetLastError();
}

cudaError_t launch_qmatmul_image_decode(int fmt, const uint8_t* image, int n, int k, __half* w16, cudaStream_t s) {
  if (!qmatmul_image_bytes(fmt, n, k)) return cudaErrorInvalidValue;
  return launch_decode_image(image + q_table_bytes(n), reinterpret_cast<const SkinnyTile*>(image), n / 128, k / 256,
                             false, n, k, w16, s);
}

int qmatmul_enqueue(int fmt, const uint8_t* image, const __half* x, int m, int n, int k, float* y, uint32_t* err,
                    cudaStream_t s) {
  if (!qmatmul_image_bytes(fmt, n, k) || m < 1) {
    set_error("quantized matmul: n must be a multiple of 128 and K divisible by 256");
    return kErrArgs;
  }
  const int tiles = n / 128, slabs = k / 256, chunk = q_chunk_bytes(fmt);
  const SkinnyTile* table = reinterpret_cast<const SkinnyTile*>(image);
  const uint8_t* packed = image + q_table_bytes(n);
  CUtensorMap map;
  if (m <= 64) {
    const int np = m <= 16 ? 16 : m <= 32 ? 32 : 64;
    if (int rc = make_tmap_f16(&map, x, (uint64_t)k, (uint64_t)m, 64, np)) return rc;
    SkinnyArgs a = {};
    a.packed = packed;
    a.tiles = table;
    a.err = err;
    a.d_tokens = nullptr;
    a.tokens = m;
    a.n = n;
    a.slabs = slabs;
    pick_splits(tiles, slabs, np, chunk, &a.splits, &a.rstages);
    a.slabs_max = (slabs + a.splits - 1) / a.splits;
    a.chunk_max = chunk;
    a.mode = kSkinnyF32;
    a.out = reinterpret_cast<__half*>(y);
    a.ldo = n;
    // on a created stream the weights stream before the previous kernel ends
    a.pdl = s ? 1 : 0;
    if (skinny_smem_bytes(np, a.slabs_max, chunk, a.rstages) > 227 * 1024) {
      set_error("quantized matmul: K range does not fit shared memory");
      return kErrArgs;
    }
    const cudaError_t e = launch_skinny(&map, a, np, tiles, s);
    if (e != cudaSuccess) {
      set_error(std::string("quantized matmul launch failed: ") + cudaGetErrorString(e));
      return kErrCuda;
    }
    return kOk;
  }
  if (int rc = make_tmap_f16(&map, x, (uint64_t)k, (uint64_t)m, 64, 128)) return rc;
  const cudaError_t e = launch_gemm_q(&map, packed, table, tiles, slabs, chunk, kSkinnyF32, reinterpret_cast<__half*>(y),
                                      n, nullptr, m, err, s);
  if (e != cudaSuccess) {
    set_error(std::string("quantized matmul launch failed: ") + cudaGetErrorString(e));
    return kErrCuda;
  }
  return kOk;
}

}  // namespace nemo
