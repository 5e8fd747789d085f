// Bidirectional GQA attention (ops.ts:213-362) on CUDA cores: one block per
// (32-query tile, q head, request), 4 warps x 8 queries; K/V tiles of 32
// (sampled) keys staged in shared memory, one key per lane for Q.K, online
// softmax in f32, P.V accumulated in f32 (4 dims per lane).
//
// Semantics kept from the reference: keys are restricted to the request's
// valid length in this layer; when that length exceeds 2048 only every third
// key (positions 0, 3, 6, ...) is used (ops.ts:258-269); queries at positions
// >= 16384 get the temperature factor of ops.ts:241. Softmax scale 1/sqrt(128).
#include "kernels.cuh"

namespace nemo {
namespace {

constexpr int kQT = 32;  // queries per block
constexpr int kKT = 32;  // keys per tile

__global__ void __launch_bounds__(128) attention_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                                                        const __half* __restrict__ qkv, const Meta* __restrict__ meta,
                                                        int merged, __half* out) {
  __shared__ __align__(16) __half qs[kQT][kHeadDim];
  __shared__ __align__(16) float ks[kKT][kHeadDim + 4];
  __shared__ __align__(16) float vs[kKT][kHeadDim];
  dev::pdl_launch_dependents();  // lets the next projection start streaming its weights
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kQT;
  if (b >= meta->batch) return;
  const int* off = merged ? meta->tgt_off : meta->src_off;
  const int len = merged ? meta->tgt_len[b] : meta->src_len[b];
  if (q0 >= len) return;
  const int base = off[b];
  const int kvh = h / (kQHeads / kKVHeads);
  const int stride = !meta->exact && len > 2048 ? 3 : 1;
  const int nkeys = (len + stride - 1) / stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < kQT * kHeadDim / 8; i += 128) {
    const int r = i / (kHeadDim / 8), c = (i % (kHeadDim / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q0 + r < len) v = *reinterpret_cast<const uint4*>(q + ((size_t)(base + q0 + r) * kQHeads + h) * kHeadDim + c);
    *reinterpret_cast<uint4*>(&qs[r][c]) = v;
  }

  float m[8], l[8], acc[8][4], temp[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    const int pos = q0 + warp * 8 + i;
    temp[i] = pos >= 16384 ? logf(floorf((float)pos / 16384.0f) + 1.0f) * 0.1f + 1.0f : 1.0f;
  }
  const float scale = 0.08838834764831845f;

  for (int kt = 0; kt < nkeys; kt += kKT) {
    __syncthreads();
    for (int i = tid; i < kKT * kHeadDim / 8; i += 128) {
      const int r = i / (kHeadDim / 8), c = (i % (kHeadDim / 8)) * 8;
      float kv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, vv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (kt + r < nkeys) {
        const size_t kp = (size_t)base + (size_t)(kt + r) * stride;
        const uint4 ku = *reinterpret_cast<const uint4*>(k + (kp * kKVHeads + kvh) * kHeadDim + c);
        const uint4 vu = *reinterpret_cast<const uint4*>(qkv + kp * kQKVWidth + kQWidth + kKVWidth + kvh * kHeadDim + c);
        const __half2* kh = reinterpret_cast<const __half2*>(&ku);
        const __half2* vh = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = __half22float2(kh[j]), bb = __half22float2(vh[j]);
          kv[2 * j] = a.x;
          kv[2 * j + 1] = a.y;
          vv[2 * j] = bb.x;
          vv[2 * j + 1] = bb.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ks[r][c + j] = kv[j];
        vs[r][c + j] = vv[j];
      }
    }
    __syncthreads();
    const bool key_valid = kt + lane < nkeys;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int qi = warp * 8 + i;
      if (q0 + qi >= len) continue;
      // four independent partial sums (dimensions d mod 4), added at the end
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
      for (int d = 0; d < kHeadDim; d += 4) {
        const float4 kk = *reinterpret_cast<const float4*>(&ks[lane][d]);
        const __half2 qa = *reinterpret_cast<const __half2*>(&qs[qi][d]);
        const __half2 qb = *reinterpret_cast<const __half2*>(&qs[qi][d + 2]);
        const float2 fa = __half22float2(qa), fb = __half22float2(qb);
        s4[0] = fmaf(fa.x, kk.x, s4[0]);
        s4[1] = fmaf(fa.y, kk.y, s4[1]);
        s4[2] = fmaf(fb.x, kk.z, s4[2]);
        s4[3] = fmaf(fb.y, kk.w, s4[3]);
      }
      float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      s = key_valid ? s * scale * temp[i] : -INFINITY;
      float tmax = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mnew = fmaxf(m[i], tmax);
      const float p = expf(s - mnew);
      float psum = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      const float corr = expf(m[i] - mnew);
      l[i] = l[i] * corr + psum;
      float a0 = acc[i][0] * corr, a1 = acc[i][1] * corr, a2 = acc[i][2] * corr, a3 = acc[i][3] * corr;
#pragma unroll 8
      for (int j = 0; j < kKT; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float4 v4 = *reinterpret_cast<const float4*>(&vs[j][lane * 4]);
        a0 += pj * v4.x;
        a1 += pj * v4.y;
        a2 += pj * v4.z;
        a3 += pj * v4.w;
      }
      acc[i][0] = a0;
      acc[i][1] = a1;
      acc[i][2] = a2;
      acc[i][3] = a3;
      m[i] = mnew;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pos = q0 + warp * 8 + i;
    if (pos >= len) continue;
    const float inv = 1.0f / l[i];
    __half2 o[2] = {__floats2half2_rn(acc[i][0] * inv, acc[i][1] * inv),
                    __floats2half2_rn(acc[i][2] * inv, acc[i][3] * inv)};
    *reinterpret_cast<uint2*>(out + (size_t)(base + pos) * kQWidth + h * kHeadDim + lane * 4) =
        *reinterpret_cast<uint2*>(o);
  }
}

}  // namespace

cudaError_t launch_attention(const __half* q, const __half* k, const __half* qkv, const Meta* meta, bool merged,
                             int batch, int max_len, __half* out, cudaStream_t s) {
  if (max_len <= 0 || batch <= 0) return cudaSuccess;
  dim3 grid((max_len + kQT - 1) / kQT, kQHeads, batch);
  attention_kernel<<<grid, 128, 0, s>>>(q, k, qkv, meta, merged ? 1 : 0, out);
  return cudaGetLastError();
}

}  // namespace nemo
