// Tile-slab weight decoders shared by the fused-dequant projection kernels
// (k_skinny.cu, k_forward.cu). A decoder thread owns one weight row of a
// 128-row tile and turns one 64-value quarter of a 256-column slab into eight
// 16-byte chunks of the canonical 128B-swizzled K-major f16 A tile that
// tcgen05.mma reads. Values follow the reference's decode arithmetic exactly
// (quantization.ts:19-74); each intermediate is exact or rounded once, as
// there, and the f16 store rounds to nearest even.
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

// --- packed f32x2 arithmetic (sm_100) ---------------------------------------
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint32_t f2_to_h2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return pack_h2(a, b);
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 2^23 + n as f32 bits, for a small unsigned n.
__device__ __forceinline__ float magic(uint32_t n) { return __uint_as_float(0x4B000000u | n); }

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

// Q4_K row block (GGUF 144 B). Quarter q = elements 64q..64q+63 of the slab.
// value = f32(d*sc*q - dmin*m) (quantization.ts:33-34): s = d*sc and
// o = dmin*m are exact; one rounding in the subtraction of o, as in the
// reference. A nibble at bit p of a word is masked in place under the f32
// exponent of 2^23: (w & (15 << p)) | 0x4B000000 = 2^23 + q * 2^p (p <= 12
// here), and fma(s * 2^-p, 2^23 + q * 2^p, -s * 2^(23-p)) = s * q exactly
// (s * 2^-p is exact: s >= 2^-24 stays far above the f32 subnormal range).
template <typename Sink>
__device__ __forceinline__ void decode_q4k(const uint8_t* blk, int q, Sink&& sink) {
  const float d = half_at(blk), dmin = half_at(blk + 2);
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
  const float s_lo = __fmul_rn(d, (float)sc_lo), s_hi = __fmul_rn(d, (float)sc_hi);
  const float o_lo = __fmul_rn(dmin, (float)m_lo), o_hi = __fmul_rn(dmin, (float)m_hi);
  // low nibbles at bits 0 and 8, high nibbles at bits 4 and 12 (of w or w >> 16)
  const uint64_t S_lo = f2(s_lo, __fmul_rn(s_lo, 0x1p-8f)), S_hi = f2(__fmul_rn(s_hi, 0x1p-4f), __fmul_rn(s_hi, 0x1p-12f));
  const uint64_t C_lo = f2(-__fmul_rn(s_lo, 0x1p23f), -__fmul_rn(s_lo, 0x1p15f));
  const uint64_t C_hi = f2(-__fmul_rn(s_hi, 0x1p19f), -__fmul_rn(s_hi, 0x1p11f));
  const uint64_t O_lo = f2(-o_lo, -o_lo), O_hi = f2(-o_hi, -o_hi);
  const uint4* qv = reinterpret_cast<const uint4*>(blk + 16 + q * 32);
  const uint4 w0 = qv[0], w1 = qv[1];
  const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint32_t m0 = c < 4 ? 0x0Fu : 0xF0u, m1 = m0 << 8;
    const uint64_t S = c < 4 ? S_lo : S_hi, C = c < 4 ? C_lo : C_hi, O = c < 4 ? O_lo : O_hi;
    const uint32_t wa = w[(c & 3) * 2], wb = w[(c & 3) * 2 + 1];
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t src = i < 2 ? wa : wb;
      const uint32_t x = (i & 1) ? src >> 16 : src;
      const uint64_t qf = f2(__uint_as_float((x & m0) | 0x4B000000u), __uint_as_float((x & m1) | 0x4B000000u));
      h[i] = f2_to_h2(fadd2(ffma2(S, qf, C), O));
    }
    sink(c, make_uint4(h[0], h[1], h[2], h[3]));
  }
}

// Q6_K row block: ql[128] qh[64] scales[16] (208 B), d separate.
// value = f32((d*sc) * (q - 32)) (quantization.ts:67-70): d*sc exact, q - 32
// exact ((2^23+q) - (2^23+32)), one rounding in the product.
template <typename Sink>
__device__ __forceinline__ void decode_q6k(const uint8_t* blk, float d, int q, Sink&& sink) {
  const int h = q >> 1, odd = q & 1;
  const uint8_t* ql = blk + h * 64;
  const uint8_t* qh = blk + 128 + h * 32;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + h * 8);
  const uint4 l0 = reinterpret_cast<const uint4*>(ql)[0], l1 = reinterpret_cast<const uint4*>(ql)[1];
  const uint4 l2 = reinterpret_cast<const uint4*>(ql)[2], l3 = reinterpret_cast<const uint4*>(ql)[3];
  const uint4 h0 = reinterpret_cast<const uint4*>(qh)[0], h1 = reinterpret_cast<const uint4*>(qh)[1];
  const uint32_t lw[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w, l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
  const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const int nsh = odd ? 4 : 0;
  const uint64_t M32 = f2(-8388640.0f, -8388640.0f);  // -(2^23 + 32)
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int qi = c >> 2;
    const int lane0 = (c & 3) * 8;
    const int hsh = 4 * odd + 2 * qi;
    const float ds = __fmul_rn(d, (float)sc[(2 * odd + qi) * 2 + lane0 / 16]);
    const uint64_t DS = f2(ds, ds);
    const uint32_t la = lw[qi * 8 + lane0 / 4], lb = lw[qi * 8 + lane0 / 4 + 1];
    const uint32_t ha = hw[lane0 / 4], hb = hw[lane0 / 4 + 1];
    uint32_t hv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t L = i < 2 ? la : lb, H = i < 2 ? ha : hb;
      const int b0 = (i & 1) * 2;
      const uint32_t qa = ((L >> (8 * b0 + nsh)) & 15u) | (((H >> (8 * b0 + hsh)) & 3u) << 4);
      const uint32_t qb = ((L >> (8 * b0 + 8 + nsh)) & 15u) | (((H >> (8 * b0 + 8 + hsh)) & 3u) << 4);
      hv[i] = f2_to_h2(fmul2(DS, fadd2(f2(magic(qa), magic(qb)), M32)));
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
          const uint32_t m = (pair & 0x000F000Fu) | 0x64006400u;  // 1024 + q
          qh = __hsub2(*reinterpret_cast<const __half2*>(&m), k1032);
        } else {
          const uint32_t m = (pair & 0x00F000F0u) | 0x64006400u;  // 1024 + 16q
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
