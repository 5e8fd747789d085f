// Decode, embedding, residual+RMSNorm, RoPE, SwiGLU, token merge, mean pool
// and run-metadata kernels. Each kernel restates one WGSL shader of the
// reference (cited per kernel); all are memory-bound row kernels that move
// 16-byte vectors per thread and size grids to the plan's worst-case token
// count, with rows beyond the run's valid-token count exiting at once.
#include <math.h>

#include "kernels.cuh"

namespace nemo {
namespace {

__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
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

// Request index of a packed token (offsets has batch + 1 entries).
__device__ __forceinline__ int find_request(const int* offsets, int batch, int tok) {
  int b = 0;
  while (b + 1 < batch && tok >= offsets[b + 1]) ++b;
  return b;
}

// Sum over the block (any multiple of 32 threads up to 1024), in a fixed order.
__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// ---------------------------------------------------------------------------
// Decoders. One thread per (row, 32-value group). Values are exact in f32
// (see quantization.ts:19-74 and quant-matmul.ts:37-154: every product fits
// the f32 significand), f16 output rounds to nearest even as the shaders'
// f16() casts do.

__device__ void decode_group(int fmt, const uint8_t* __restrict__ src, int r, int g, int k, float (&v)[32]) {
  if (fmt == kSegQ4K) {
    const uint8_t* blk = src + ((size_t)r * (k / 256) + g / 8) * 144;
    const int sub = g & 7;
    const float d = ld_half(blk), dmin = ld_half(blk + 2);
    const uint8_t* s = blk + 4;
    int sc, mn;
    if (sub < 4) {
      sc = s[sub] & 63;
      mn = s[sub + 4] & 63;
    } else {
      sc = (s[sub + 4] & 15) | ((s[sub - 4] >> 6) << 4);
      mn = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4);
    }
    const uint8_t* q = blk + 16 + (sub >> 1) * 32;
    const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int qq = (sub & 1) ? (q[j] >> 4) : (q[j] & 15);
      v[j] = __fsub_rn(__fmul_rn(ds, (float)qq), dm);
    }
  } else if (fmt == kSegQ6K) {
    const uint8_t* blk = src + ((size_t)r * (k / 256) + g / 8) * 210;
    const int sub = g & 7, half = sub >> 2, quad = sub & 3;
    const float d = ld_half(blk + 208);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int lb = blk[half * 64 + j + (quad & 1) * 32];
      const int lo = quad >= 2 ? (lb >> 4) : (lb & 15);
      const int hi = (blk[128 + half * 32 + j] >> (quad * 2)) & 3;
      const int qq = (lo | (hi << 4)) - 32;
      const int sc = (int)(int8_t)blk[192 + half * 8 + j / 16 + quad * 2];
      // (d * scale) * q as the CPU decoder orders it: exact, and a zero keeps
      // the sign of d * scale (quantization.ts:67-70).
      v[j] = __fmul_rn(__fmul_rn(d, (float)sc), (float)qq);
    }
  } else {
    const uint8_t* blk;
    const uint8_t* qs;
    if (fmt == kSegQ40) {
      blk = src + ((size_t)r * (k / 32) + g) * 18;
      qs = blk + 2;
    } else {  // q4_0-tile32-compact, format.ts:84-97
      blk = src + ((((size_t)(r / 32) * (k / 32) + g) * 32) + (r & 31)) * 20;
      qs = blk + 4;
    }
    const float d = ld_half(blk);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = __fmul_rn(d, (float)((qs[j] & 15) - 8));
      v[j + 16] = __fmul_rn(d, (float)((qs[j] >> 4) - 8));
    }
  }
}

__global__ void decode_kernel(int fmt, const uint8_t* __restrict__ src, int rows, int k, __half* out16,
                              float* out32) {
  const int groups = k / 32;
  const long long total = (long long)rows * groups;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / groups), g = (int)(idx % groups);
    float v[32];
    decode_group(fmt, src, r, g, k, v);
    uint4* o16 = reinterpret_cast<uint4*>(out16 + (size_t)r * k + g * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = v[c * 8 + i];
      o16[c] = pack8(t);
    }
    if (out32) {
      float4* o = reinterpret_cast<float4*>(out32 + (size_t)r * k + g * 32);
#pragma unroll
      for (int c = 0; c < 8; ++c) o[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
  }
}

// ---------------------------------------------------------------------------

// model.ts:226-233 with contextualMergedLength (model.ts:30-32). Lengths are
// clamped to [1, seq] so a bad device-side input cannot index out of bounds
// (the host API rejects such inputs before they get here).
__global__ void meta_kernel(const uint32_t* lengths, int batch, int seq, const uint32_t* run_batch, Meta* meta,
                            int exact) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (run_batch) {
    const int rb = (int)*run_batch;
    batch = rb < 1 ? 1 : (rb > batch ? batch : rb);
  }
  const int mseq = exact ? seq : max(1, (int)ceil((double)seq * 0.64));
  meta->batch = batch;
  meta->seq = seq;
  meta->merged_seq = mseq;
  int o0 = 0, o1 = 0, s0 = 0, s1 = 0;
  for (int b = 0; b < batch; ++b) {
    int l = (int)lengths[b];
    l = l < 1 ? 1 : (l > seq ? seq : l);
    int t = exact ? l : max(1, (int)ceil((double)l * 0.64));
    t = t < mseq ? t : mseq;
    meta->src_len[b] = l;
    meta->tgt_len[b] = t;
    meta->src_off[b] = o0;
    meta->tgt_off[b] = o1;
    meta->samp_off[0][b] = s0;
    meta->samp_off[1][b] = s1;
    o0 += l;
    o1 += t;
    if (!exact && l > kSampleThreshold) s0 += (l + kSampleStride - 1) / kSampleStride;
    if (!exact && t > kSampleThreshold) s1 += (t + kSampleStride - 1) / kSampleStride;
  }
  meta->src_off[batch] = o0;
  meta->tgt_off[batch] = o1;
  meta->samp_off[0][batch] = s0;
  meta->samp_off[1][batch] = s1;
  meta->t0 = o0;
  meta->t1 = o1;
  meta->exact = exact;
}

// ops.ts:680-725: Q6_K row gather + decode, 8 columns per thread, 1 token per
// block. The f32 value (d * scale) * q is exact, then f16 round-to-nearest.
__global__ void __launch_bounds__(256) embedding_kernel(const uint32_t* __restrict__ ids,
                                                        const uint8_t* __restrict__ table, int vocab,
                                                        const Meta* __restrict__ meta, __half* x) {
  const int tok = blockIdx.x;
  if (tok >= meta->t0) return;
  const int b = find_request(meta->src_off, meta->batch, tok);
  const int p = tok - meta->src_off[b];
  uint32_t id = ids[(size_t)b * meta->seq + p];
  if (id >= (uint32_t)vocab) id = 0;  // host validates; keeps device reads in bounds
  const int c = threadIdx.x * 8;
  const int within = c & 255, half = within >> 7, position = within & 127;
  const int quad = position >> 5, lane = position & 31;
  const uint8_t* blk = table + ((size_t)id * (kHidden / 256) + (c >> 8)) * 210;
  const float d = ld_half(blk + 208);
  const int sc = (int)(int8_t)blk[192 + half * 8 + lane / 16 + quad * 2];
  const float ds = __fmul_rn(d, (float)sc);
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int lb = blk[half * 64 + lane + i + (quad & 1) * 32];
    const int lo = quad >= 2 ? (lb >> 4) : (lb & 15);
    const int hi = (blk[128 + half * 32 + lane + i] >> (quad * 2)) & 3;
    v[i] = __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
  }
  *reinterpret_cast<uint4*>(x + (size_t)tok * kHidden + c) = pack8(v);
}

// ops.ts:21-72: one row per block of 256 threads, 8 columns per thread.
__global__ void __launch_bounds__(256) rmsnorm_kernel(__half* x, const __half* __restrict__ residual,
                                                      const float* __restrict__ w, __half* norm,
                                                      const int* __restrict__ d_rows, float eps) {
  __shared__ float red[32];
  dev::pdl_launch_dependents();  // lets the next projection start streaming its weights
  const int row = blockIdx.x;
  if (row >= *d_rows) return;
  const int c = threadIdx.x * 8;
  __half* xr = x + (size_t)row * kHidden + c;
  float v[8];
  unpack8(*reinterpret_cast<const uint4*>(xr), v);
  if (residual) {
    float r[8];
    unpack8(*reinterpret_cast<const uint4*>(residual + (size_t)row * kHidden + c), r);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(v[i], r[i]);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  uint4 xs = pack8(v);  // x = f16(value)
  if (residual) *reinterpret_cast<uint4*>(xr) = xs;
  ss = block_sum_256(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)kHidden), eps));
  float xn[8];
  unpack8(xs, xn);
  const float4 w0 = *reinterpret_cast<const float4*>(w + c);
  const float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(xn[i], inv), wv[i]);
  *reinterpret_cast<uint4*>(norm + (size_t)row * kHidden + c) = pack8(o);
}

// rmsnorm_kernel after a GEMM launched with GemmEpi::part: when that GEMM
// split K, the residual is f16(its f32 parts summed in split order), the f16
// projection output an unsplit GEMM stores; otherwise its f16 output. One
// block per row. WIDE issues every split's loads before the first add (one
// round trip instead of one per split) at the cost of registers (2 blocks per
// SM): the launcher takes it when the plan's rows are few, which is also when
// the GEMM splits K.
template <bool WIDE>
__global__ void __launch_bounds__(256, WIDE ? 2 : 8) rmsnorm_parts_kernel(__half* x, const __half* __restrict__ residual,
                                                            const float* __restrict__ part,
                                                            const int* __restrict__ d_splits,
                                                            const float* __restrict__ w, __half* norm,
                                                            const int* __restrict__ d_rows, float eps) {
  __shared__ float red[32];
  dev::pdl_launch_dependents();
  const int row = blockIdx.x;
  const int M = *d_rows;
  if (row >= M) return;
  const int c = threadIdx.x * 8;
  __half* xr = x + (size_t)row * kHidden + c;
  // x, the f16 residual (always allocated; used with one split) and the
  // split count are loaded together
  const uint4 xv = *reinterpret_cast<const uint4*>(xr);
  const uint4 rv = __ldcg(reinterpret_cast<const uint4*>(residual + (size_t)row * kHidden + c));
  const int splits = *d_splits;
  float r[8];
  if (splits == 1) {
    unpack8(rv, r);
  } else if (WIDE) {
    float4 pa[kMaxKSplit], pb[kMaxKSplit];
#pragma unroll
    for (int sp = 0; sp < kMaxKSplit; ++sp) {
      if (sp < splits) {
        const float4* p = reinterpret_cast<const float4*>(part + ((size_t)sp * M + row) * kHidden + c);
        pa[sp] = __ldcg(p);
        pb[sp] = __ldcg(p + 1);
      }
    }
    r[0] = pa[0].x, r[1] = pa[0].y, r[2] = pa[0].z, r[3] = pa[0].w;
    r[4] = pb[0].x, r[5] = pb[0].y, r[6] = pb[0].z, r[7] = pb[0].w;
#pragma unroll
    for (int sp = 1; sp < kMaxKSplit; ++sp) {
      if (sp < splits) {
        const float u[8] = {pa[sp].x, pa[sp].y, pa[sp].z, pa[sp].w, pb[sp].x, pb[sp].y, pb[sp].z, pb[sp].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = __fadd_rn(r[i], u[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = __half2float(__float2half_rn(r[i]));
  } else {
    {
      const float4* p = reinterpret_cast<const float4*>(part + (size_t)row * kHidden + c);
      const float4 a = __ldcg(p), b = __ldcg(p + 1);
      r[0] = a.x, r[1] = a.y, r[2] = a.z, r[3] = a.w, r[4] = b.x, r[5] = b.y, r[6] = b.z, r[7] = b.w;
    }
    for (int sp = 1; sp < splits; ++sp) {
      const float4* p = reinterpret_cast<const float4*>(part + ((size_t)sp * M + row) * kHidden + c);
      const float4 a = __ldcg(p), b = __ldcg(p + 1);
      const float u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = __fadd_rn(r[i], u[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = __half2float(__float2half_rn(r[i]));
  }
  float v[8];
  unpack8(xv, v);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(v[i], r[i]);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  uint4 xs = pack8(v);  // x = f16(value)
  *reinterpret_cast<uint4*>(xr) = xs;
  ss = block_sum_256(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)kHidden), eps));
  float xn[8];
  unpack8(xs, xn);
  const float4 w0 = *reinterpret_cast<const float4*>(w + c);
  const float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(xn[i], inv), wv[i]);
  *reinterpret_cast<uint4*>(norm + (size_t)row * kHidden + c) = pack8(o);
}

// ops.ts:168-194: one thread per (token, head, pair); the position is the
// token's index within its (merged) row. A head group of nq q heads and nk kv
// heads: Q at columns [0, nq*128) and K at [nq*128, (nq+nk)*128) of qkv rows
// qkv_ld wide (the full model: 24, 8, 5120).
__global__ void __launch_bounds__(256) rope_kernel(const __half* __restrict__ qkv,
                                                   const float* __restrict__ table,
                                                   const Meta* __restrict__ meta, int merged, __half* q,
                                                   __half* k, int nq, int nk, int qkv_ld) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_tok = (nq + nk) * 64;
  const int tok = (int)(idx / per_tok);
  const int T = merged ? meta->t1 : meta->t0;
  if (tok >= T) return;
  const int hp = (int)(idx - (long long)tok * per_tok), head = hp >> 6, pair = hp & 63;
  const int* off = merged ? meta->tgt_off : meta->src_off;
  const int b = find_request(off, meta->batch, tok);
  const int pos = tok - off[b];
  const bool is_q = head < nq;
  const int col = head * kHeadDim;
  const __half2 in = *reinterpret_cast<const __half2*>(qkv + (size_t)tok * qkv_ld + col + pair * 2);
  const float2 cs = *reinterpret_cast<const float2*>(table + ((size_t)pos * 64 + pair) * 2);
  const float even = __low2float(in), odd = __high2float(in);
  const float first = __fsub_rn(__fmul_rn(even, cs.x), __fmul_rn(odd, cs.y));
  const float second = __fadd_rn(__fmul_rn(even, cs.y), __fmul_rn(odd, cs.x));
  const __half2 o = __halves2half2(__float2half_rn(first), __float2half_rn(second));
  if (is_q)
    *reinterpret_cast<__half2*>(q + ((size_t)tok * nq + head) * kHeadDim + pair * 2) = o;
  else
    *reinterpret_cast<__half2*>(k + ((size_t)tok * nk + head - nq) * kHeadDim + pair * 2) = o;
}

// ops.ts:74-89: out = f16(silu(g) * u), silu = g / (1 + exp(-g)).
__global__ void __launch_bounds__(256) swiglu_kernel(const __half* __restrict__ gu, const int* __restrict__ d_rows,
                                                     __half* out) {
  const int row = blockIdx.x;
  if (row >= *d_rows) return;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= kInter) return;
  float g[8], u[8], o[8];
  unpack8(*reinterpret_cast<const uint4*>(gu + (size_t)row * 2 * kInter + c), g);
  unpack8(*reinterpret_cast<const uint4*>(gu + (size_t)row * 2 * kInter + kInter + c), u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float silu = __fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i])));
    o[i] = __fmul_rn(silu, u[i]);
  }
  *reinterpret_cast<uint4*>(out + (size_t)row * kInter + c) = pack8(o);
}

// ops.ts:629-661: BOS-preserving adjacent-bin mean over both x and the
// normalised state; f32 sum in source order, f32 division, f16 store.
__global__ void __launch_bounds__(256) merge_kernel(const __half* __restrict__ x, const __half* __restrict__ nrm,
                                                    const Meta* __restrict__ meta, __half* xm, __half* nm) {
  const int tok = blockIdx.x;
  if (tok >= meta->t1) return;
  const int b = find_request(meta->tgt_off, meta->batch, tok);
  const uint32_t p = (uint32_t)(tok - meta->tgt_off[b]);
  const uint32_t sl = (uint32_t)meta->src_len[b], tl = (uint32_t)meta->tgt_len[b];
  uint32_t start = 0, end = 1;
  if (p > 0 && tl > 1) {
    const uint32_t st = sl - 1, tt = tl - 1;
    start = 1 + ((p - 1) * st) / tt;
    end = 1 + (p * st) / tt;
    end = max(end, start + 1);
    end = min(end, sl);
  }
  const int c = threadIdx.x * 8;
  float tx[8] = {0, 0, 0, 0, 0, 0, 0, 0}, tn[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const size_t base = (size_t)meta->src_off[b];
  for (uint32_t s = start; s < end; ++s) {
    float a[8], n[8];
    unpack8(*reinterpret_cast<const uint4*>(x + (base + s) * kHidden + c), a);
    unpack8(*reinterpret_cast<const uint4*>(nrm + (base + s) * kHidden + c), n);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      tx[i] = __fadd_rn(tx[i], a[i]);
      tn[i] = __fadd_rn(tn[i], n[i]);
    }
  }
  const float cnt = (float)(end - start);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    tx[i] = __fdiv_rn(tx[i], cnt);
    tn[i] = __fdiv_rn(tn[i], cnt);
  }
  *reinterpret_cast<uint4*>(xm + (size_t)tok * kHidden + c) = pack8(tx);
  *reinterpret_cast<uint4*>(nm + (size_t)tok * kHidden + c) = pack8(tn);
}

// ops.ts:596-616: mean over the valid merged rows, then L2 normalisation.
// One block of 1024 threads per request, two columns per thread: each column
// sums its rows in order with 32 row loads in flight (a 3200-row request is
// 100 dependent rounds instead of 200 with 8 columns per thread).
constexpr int kPoolThreads = kHidden / 2;
__global__ void __launch_bounds__(kPoolThreads) pool_kernel(const __half* __restrict__ nrm,
                                                            const Meta* __restrict__ meta, float* out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int len = meta->tgt_len[b];
  const size_t base = (size_t)meta->tgt_off[b];
  const int c = threadIdx.x * 2;
  float t0 = 0.f, t1 = 0.f;
  constexpr int kRows = 32;
  int p = 0;
  for (; p + kRows <= len; p += kRows) {
    __half2 u[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) u[r] = *reinterpret_cast<const __half2*>(nrm + (base + p + r) * kHidden + c);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const float2 a = __half22float2(u[r]);
      t0 = __fadd_rn(t0, a.x);
      t1 = __fadd_rn(t1, a.y);
    }
  }
  for (; p < len; ++p) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(nrm + (base + p) * kHidden + c));
    t0 = __fadd_rn(t0, a.x);
    t1 = __fadd_rn(t1, a.y);
  }
  t0 = __fdiv_rn(t0, (float)len);
  t1 = __fdiv_rn(t1, (float)len);
  const float ss = block_sum_256(__fadd_rn(__fmul_rn(t0, t0), __fmul_rn(t1, t1)), red);
  const float inv = rsqrtf(ss);
  *reinterpret_cast<float2*>(out + (size_t)b * kHidden + c) = make_float2(t0 * inv, t1 * inv);
}

// CUDA-core GEMM for validation: 64x64 tile, K step 32, 4x4 outputs/thread.
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                        __half* y, float* y32, const int* __restrict__ d_rows,
                                                        int n, int k) {
  __shared__ float xs[32][64 + 4];
  __shared__ float ws[32][64 + 4];
  const int M = *d_rows;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  if (m0 >= M) return;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += 32) {
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
      const int r = i / 32, kk = i % 32;
      xs[kk][r] = (m0 + r < M) ? __half2float(x[(size_t)(m0 + r) * k + k0 + kk]) : 0.f;
      ws[kk][r] = __half2float(w[(size_t)(n0 + r) * k + k0 + kk]);
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        bb[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * bb[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + ty * 4 + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int cidx = n0 + tx * 4 + j;
      y[(size_t)r * n + cidx] = __float2half_rn(acc[i][j]);
      if (y32) y32[(size_t)r * n + cidx] = acc[i][j];
    }
  }
}

inline int grid_for(long long work, int per_block, int cap = 148 * 16) {
  long long g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  return (int)(g > cap ? cap : g);
}

}  // namespace

cudaError_t launch_decode(int fmt, const uint8_t* src, int rows, int k, __half* out16, float* out32,
                          cudaStream_t s) {
  decode_kernel<<<grid_for((long long)rows * (k / 32), 256), 256, 0, s>>>(fmt, src, rows, k, out16, out32);
  return cudaGetLastError();
}

cudaError_t launch_meta(const uint32_t* lengths, int batch, int seq, const uint32_t* run_batch, Meta* meta,
                        cudaStream_t s, int exact) {
  meta_kernel<<<1, 32, 0, s>>>(lengths, batch, seq, run_batch, meta, exact);
  return cudaGetLastError();
}

cudaError_t launch_embedding(const uint32_t* ids, const uint8_t* table, int vocab, const Meta* meta,
                             int max_tokens, __half* x, cudaStream_t s) {
  embedding_kernel<<<max_tokens, 256, 0, s>>>(ids, table, vocab, meta, x);
  return cudaGetLastError();
}

cudaError_t launch_residual_rmsnorm(__half* x, const __half* residual, const float* w, __half* norm,
                                    const int* d_rows, int max_rows, cudaStream_t s) {
  rmsnorm_kernel<<<max_rows, 256, 0, s>>>(x, residual, w, norm, d_rows, kEpsilon);
  return cudaGetLastError();
}

cudaError_t launch_residual_rmsnorm_parts(__half* x, const __half* residual, const float* part, const int* d_splits,
                                          const float* w, __half* norm, const int* d_rows, int max_rows,
                                          cudaStream_t s) {
  if (!residual || !part || !d_splits) return cudaErrorInvalidValue;
  // (1280 rows: 10 row tiles, the most at which the O / down GEMMs still
  // split K by 8 on 148 SMs)
  if (max_rows <= 1280)
    rmsnorm_parts_kernel<true><<<max_rows, 256, 0, s>>>(x, residual, part, d_splits, w, norm, d_rows, kEpsilon);
  else
    rmsnorm_parts_kernel<false><<<max_rows, 256, 0, s>>>(x, residual, part, d_splits, w, norm, d_rows, kEpsilon);
  return cudaGetLastError();
}

cudaError_t launch_rope(const __half* qkv, const float* table, const Meta* meta, bool merged, int max_tokens,
                        __half* q, __half* k, cudaStream_t s) {
  return launch_rope_group(qkv, kQKVWidth, kQHeads, kKVHeads, table, meta, merged, max_tokens, q, k, s);
}

cudaError_t launch_rope_group(const __half* qkv, int qkv_ld, int nq, int nk, const float* table, const Meta* meta,
                              bool merged, int max_tokens, __half* q, __half* k, cudaStream_t s) {
  if (max_tokens <= 0) return cudaSuccess;
  const long long threads = (long long)max_tokens * (nq + nk) * 64;
  rope_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(qkv, table, meta, merged ? 1 : 0, q, k, nq, nk,
                                                                qkv_ld);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const __half* gate_up, const int* d_rows, int max_rows, __half* out, cudaStream_t s) {
  dim3 grid(max_rows, (kInter / 8 + 255) / 256);
  swiglu_kernel<<<grid, 256, 0, s>>>(gate_up, d_rows, out);
  return cudaGetLastError();
}

cudaError_t launch_merge(const __half* x, const __half* norm, const Meta* meta, int max_out, __half* xm,
                         __half* nm, cudaStream_t s) {
  merge_kernel<<<max_out, 256, 0, s>>>(x, norm, meta, xm, nm);
  return cudaGetLastError();
}

cudaError_t launch_mean_pool(const __half* norm, const Meta* meta, int batch, float* out, cudaStream_t s) {
  pool_kernel<<<batch, kPoolThreads, 0, s>>>(norm, meta, out);
  return cudaGetLastError();
}

cudaError_t launch_gemm_simt(const __half* x, const __half* w, __half* y, float* y32, const int* d_rows,
                             int max_rows, int n, int k, cudaStream_t s) {
  dim3 grid(n / 64, (max_rows + 63) / 64);
  gemm_simt_kernel<<<grid, 256, 0, s>>>(x, w, y, y32, d_rows, n, k);
  return cudaGetLastError();
}

}  // namespace nemo
