// Tile-slab weight decoders shared by the fused-dequant projection kernels
// (k_forward.cu, k_skinny.cu, k_gemm_q.cu) and by the image decode of model
// load and nemo_op_qmatmul_image_decode (qmatmul.cu). A decoder thread owns
// one weight row of a 128-row tile and turns one 64-value quarter of a
// 256-column slab into eight 16-byte chunks of the canonical 128B-swizzled
// K-major f16 A tile that tcgen05.mma reads. Values follow the reference's
// decode arithmetic exactly (quantization.ts:19-74); each intermediate is
// exact or rounded once, as there, and the f16 store rounds to nearest even.
#pragma once

#include "kernels.cuh"

namespace nemo {
namespace tsd {

__device__ __forceinline__ float half_at(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void st_chunk(uint8_t* a_tile, int r, int c, uint4 v) {
  *reinterpret_cast<uint4*>(a_tile + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

// Decoders hand each finished 16-byte chunk c (values 8c..8c+7 of the
// quarter) to a sink: a 128B-swizzled shared-memory A tile, or registers that
// are then stored to tensor memory (column 4c + i holds word i of chunk c).
struct SmemTileSink {
  uint8_t* a_tile;
  int r;
  __device__ __forceinline__ void operator()(int c, uint4 v) const { st_chunk(a_tile, r, c, v); }
};
struct RegSink {
  uint32_t* h;  // [32], indexed with compile-time constants after unrolling
  __device__ __forceinline__ void operator()(int c, uint4 v) const {
    h[4 * c] = v.x;
    h[4 * c + 1] = v.y;
    h[4 * c + 2] = v.z;
    h[4 * c + 3] = v.w;
  }
};

__device__ __forceinline__ int region_bytes(int fmt) { return fmt == kSegQ6K ? 64 * 210 : 64 * 144; }

// --- bit-level helpers -------------------------------------------------------
// (a & b) | c in one logic op (the compiler otherwise splits a mask-and-or with
// two constants into two).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hadd2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// f32 result of f16 a times the low / high f16 half of b plus f32 c, rounded
// once (the mixed-precision fma of sm_100: both f16 operands widen exactly).
__device__ __forceinline__ float mixed_fma_lo(uint16_t a, uint32_t b, float c) {
  float r;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %2; fma.rn.f32.f16 %0, %1, l, %3;}" : "=f"(r) : "h"(a), "r"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float mixed_fma_hi(uint16_t a, uint32_t b, float c) {
  float r;
  asm("{.reg .b16 l, h; mov.b32 {l, h}, %2; fma.rn.f32.f16 %0, %1, h, %3;}" : "=f"(r) : "h"(a), "r"(b), "f"(c));
  return r;
}
// f16 bits of v (exactly representable) in both halves.
__device__ __forceinline__ uint32_t f16x2_bits(float v) {
  const uint32_t b = __half_as_ushort(__float2half_rn(v));
  return b | (b << 16);
}

// Q4_K row block (GGUF 144 B). Quarter q = elements 64q..64q+63 of the slab:
// sub-block 2q in the low nibbles of quant bytes 32q..32q+31, sub-block 2q+1 in
// their high nibbles. value = f32(d*sc*q - dmin*m) (quantization.ts:33-34):
// d*sc*q is exact and the subtraction of dmin*m rounds once.
// Here t = sc*q, an integer <= 945, is formed exactly in f16x2 arithmetic from
// nibbles masked under the f16 exponent of 1024 ((w & 0x000F000F) | 0x64006400
// = {1024 + q, 1024 + q'}; high nibbles give 1024 + 16q): t = fma(sc, 1024 + q,
// -1024 sc), or fma(sc / 16, 1024 + 16 q, -64 sc). Then one mixed fma
// d (f16) * t - dmin*m computes d*sc*q exactly and rounds the difference once:
// the same f32 value, zero signs included.
template <typename Sink>
__device__ __forceinline__ void decode_q4k(const uint8_t* blk, int q, Sink&& sink) {
  const uint16_t dh = *reinterpret_cast<const uint16_t*>(blk);
  const float dmin = half_at(blk + 2);
  const uint8_t* s = blk + 4;
  const int lo = 2 * q, hi = 2 * q + 1;
  int sc_lo, m_lo, sc_hi, m_hi;
  if (lo < 4) {
    sc_lo = s[lo] & 63;
    m_lo = s[lo + 4] & 63;
    sc_hi = s[hi] & 63;
    m_hi = s[hi + 4] & 63;
  } else {
    sc_lo = (s[lo + 4] & 15) | ((s[lo - 4] >> 6) << 4);
    m_lo = (s[lo + 4] >> 4) | ((s[lo] >> 6) << 4);
    sc_hi = (s[hi + 4] & 15) | ((s[hi - 4] >> 6) << 4);
    m_hi = (s[hi + 4] >> 4) | ((s[hi] >> 6) << 4);
  }
  const float o_lo = -__fmul_rn(dmin, (float)m_lo), o_hi = -__fmul_rn(dmin, (float)m_hi);
  const uint32_t SL = f16x2_bits((float)sc_lo), CL = f16x2_bits(-1024.f * sc_lo);
  const uint32_t SH = f16x2_bits(0.0625f * sc_hi), CH = f16x2_bits(-64.f * sc_hi);
  const uint4* qv = reinterpret_cast<const uint4*>(blk + 16 + q * 32);
  const uint4 w0 = qv[0], w1 = qv[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // words 2c, 2c+1: low chunk c and high chunk 4 + c
    uint32_t lv[4], hv[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // word = bytes 4j..4j+3 of the chunk's 8
      const uint32_t x = w[2 * c + j], y = x >> 8;
      const uint32_t l02 = hfma2_bits(and_or(x, 0x000F000Fu, 0x64006400u), SL, CL);  // bytes 0, 2
      const uint32_t l13 = hfma2_bits(and_or(y, 0x000F000Fu, 0x64006400u), SL, CL);  // bytes 1, 3
      const uint32_t h02 = hfma2_bits(and_or(x, 0x00F000F0u, 0x64006400u), SH, CH);
      const uint32_t h13 = hfma2_bits(and_or(y, 0x00F000F0u, 0x64006400u), SH, CH);
      lv[2 * j] = pack_h2(mixed_fma_lo(dh, l02, o_lo), mixed_fma_lo(dh, l13, o_lo));
      lv[2 * j + 1] = pack_h2(mixed_fma_hi(dh, l02, o_lo), mixed_fma_hi(dh, l13, o_lo));
      hv[2 * j] = pack_h2(mixed_fma_lo(dh, h02, o_hi), mixed_fma_lo(dh, h13, o_hi));
      hv[2 * j + 1] = pack_h2(mixed_fma_hi(dh, h02, o_hi), mixed_fma_hi(dh, h13, o_hi));
    }
    sink(c, make_uint4(lv[0], lv[1], lv[2], lv[3]));
    sink(4 + c, make_uint4(hv[0], hv[1], hv[2], hv[3]));
  }
}

// Q6_K row block: ql[128] qh[64] scales[16] (208 B); dh = the row's f16 d bits.
// value = f32((d*sc) * (q - 32)) (quantization.ts:67-70): d*sc exact, one
// rounding in the product. The 6-bit q of four consecutive elements are put
// together in the bytes of one word (low 4 bits from ql, high 2 from qh); a
// byte permute with 0x64 bytes makes f16 pairs 1024 + q, and adding -1056 gives
// q - 32 exactly. d * (q - 32) is exact in f32 (mixed fma with a -0 addend,
// which keeps the sign of a zero product), and the product with sc rounds once.
template <typename Sink>
__device__ __forceinline__ void decode_q6k(const uint8_t* blk, uint16_t dh, int q, Sink&& sink) {
  const int h = q >> 1, odd = q & 1;
  const uint8_t* ql = blk + h * 64;
  const uint8_t* qh = blk + 128 + h * 32;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + h * 8);
  const uint4 l0 = reinterpret_cast<const uint4*>(ql)[0], l1 = reinterpret_cast<const uint4*>(ql)[1];
  const uint4 l2 = reinterpret_cast<const uint4*>(ql)[2], l3 = reinterpret_cast<const uint4*>(ql)[3];
  const uint4 h0 = reinterpret_cast<const uint4*>(qh)[0], h1 = reinterpret_cast<const uint4*>(qh)[1];
  const uint32_t lw[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w, l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t kM1056 = 0xE420E420u;  // f16 -1056 in both halves
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int qi = c >> 2;
    const int lane0 = (c & 3) * 8;
    const int hsh = 4 * odd + 2 * qi;  // bit of the element's 2 high bits in its qh byte
    const float s = (float)sc[(2 * odd + qi) * 2 + lane0 / 16];
    uint32_t hv[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // elements 4j..4j+3 of the chunk
      const uint32_t L = odd ? lw[qi * 8 + lane0 / 4 + j] >> 4 : lw[qi * 8 + lane0 / 4 + j];
      const uint32_t Hs = hw[lane0 / 4 + j];
      const uint32_t H = hsh >= 4 ? Hs >> (hsh - 4) : Hs << (4 - hsh);
      const uint32_t qb = and_or(L, 0x0F0F0F0Fu, H & 0x30303030u);
      const uint32_t t01 = hadd2_bits(__byte_perm(qb, 0x64646464u, 0x5140u), kM1056);
      const uint32_t t23 = hadd2_bits(__byte_perm(qb, 0x64646464u, 0x5342u), kM1056);
      hv[2 * j] = pack_h2(__fmul_rn(mixed_fma_lo(dh, t01, -0.f), s), __fmul_rn(mixed_fma_hi(dh, t01, -0.f), s));
      hv[2 * j + 1] = pack_h2(__fmul_rn(mixed_fma_lo(dh, t23, -0.f), s), __fmul_rn(mixed_fma_hi(dh, t23, -0.f), s));
    }
    sink(c, make_uint4(hv[0], hv[1], hv[2], hv[3]));
  }
}

// Q4_0 row block for one 256 slab: d[8] (16 B) then 8 x 16 quant bytes.
// value = f16(d * (q - 8)) (quantization.ts:42, quant-matmul.ts:106): computed
// in f16x2: (1024 + q) - 1032 is exact and the f16 product rounds once to
// nearest even, the same value as the exact f32 product rounded to f16.
template <typename Sink>
__device__ __forceinline__ void decode_q40(const uint8_t* blk, int q, Sink&& sink) {
  const __half2 k1032 = __float2half2_rn(1032.0f);
  const __half2 k16th = __float2half2_rn(0.0625f);
  const __half2 k72 = __float2half2_rn(-72.0f);
#pragma unroll
  for (int bi = 0; bi < 2; ++bi) {
    const int b = 2 * q + bi;
    const __half dh = __ushort_as_half(*reinterpret_cast<const unsigned short*>(blk + 2 * b));
    const __half2 d2 = __halves2half2(dh, dh);
    const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + b * 16);
    const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const bool high = cc >= 2;  // elements 16..31 are the high nibbles of bytes 0..15
      const uint32_t wa = w[(cc & 1) * 2], wb = w[(cc & 1) * 2 + 1];
      uint32_t hv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t src = i < 2 ? wa : wb;
        const uint32_t pair = __byte_perm(src, 0, (i & 1) ? 0x4342u : 0x4140u);  // bytes -> low bytes of halves
        __half2 qh;
        if (!high) {
          const uint32_t m = and_or(pair, 0x000F000Fu, 0x64006400u);  // 1024 + q
          qh = __hsub2(*reinterpret_cast<const __half2*>(&m), k1032);
        } else {
          const uint32_t m = and_or(pair, 0x00F000F0u, 0x64006400u);  // 1024 + 16q
          qh = __hfma2(*reinterpret_cast<const __half2*>(&m), k16th, k72);
        }
        const __half2 v = __hmul2(d2, qh);
        hv[i] = *reinterpret_cast<const uint32_t*>(&v);
      }
      sink(bi * 4 + cc, make_uint4(hv[0], hv[1], hv[2], hv[3]));
    }
  }
}

__device__ __forceinline__ int find_req(const int* off, int batch, int tok) {
  int b = 0;
  while (b + 1 < batch && tok >= off[b + 1]) ++b;
  return b;
}

}  // namespace tsd
}  // namespace nemo
