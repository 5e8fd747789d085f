// CPU oracle: restatement of the reference's quantisation code and of the WGSL
// forward math of the Nemotron-3-Embed-1B encoder. TEST INFRASTRUCTURE ONLY:
// see oracle.h for what may use it. Built with -ffp-contract=off so every f32/f64
// expression rounds in the order written, as the JS and WGSL statements do.
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#if defined(__F16C__)
#include <immintrin.h>
#endif

namespace {

constexpr int kHidden = 2048;          // model.ts:19
constexpr int kInter = 6144;           // model.ts:20
constexpr int kQWidth = 3072;          // model.ts:21
constexpr int kKVWidth = 1024;         // model.ts:22
constexpr int kQKVWidth = 5120;        // model.ts:23
constexpr int kMergeAfterLayer = 4;    // model.ts:26
constexpr float kEpsilon = 1e-5f;      // model.ts:27
constexpr double kRopeTheta = 1000000.0;  // model.ts:28
constexpr int kQHeads = 24, kKVHeads = 8, kHeadDim = 128;  // model.ts:127-128
constexpr int kEmbedBlockBytes = 210;  // Q6_K block, ops.ts:690

void set_err(char* err, size_t errlen, const char* msg) {
  if (err && errlen) {
    snprintf(err, errlen, "%s", msg);
  }
}

inline float h2f(uint16_t h) { return orc_f16_to_f32(h); }
inline uint16_t f2h(float f) { return orc_f16_rne(f); }

size_t block_bytes(int type) {
  return type == ORC_Q4_K ? 144 : type == ORC_Q6_K ? 210 : type == ORC_Q4_0 ? 18 : 0;
}
int block_values(int type) { return type == ORC_Q4_0 ? 32 : 256; }

}  // namespace

extern "C" {

// quantization.ts:2-9
double orc_half_to_float(uint16_t bits) {
  const double sign = (bits & 0x8000) ? -1.0 : 1.0;
  const int exponent = (bits >> 10) & 0x1f;
  const int fraction = bits & 0x3ff;
  if (exponent == 0) return sign * ldexp(1.0, -14) * (fraction / 1024.0);
  if (exponent == 0x1f) return fraction ? NAN : sign * INFINITY;
  return sign * ldexp(1.0, exponent - 15) * (1.0 + fraction / 1024.0);
}

// f16.ts:4-25. The JS stores the number into a Float32Array first, then rounds
// the mantissa half-up (ties away from zero), not to nearest even.
uint16_t orc_float_to_half(double value) {
  const float f = (float)value;
  uint32_t bits;
  memcpy(&bits, &f, 4);
  const uint32_t sign = (bits >> 16) & 0x8000;
  int exponent = (int)((bits >> 23) & 0xff) - 127 + 15;
  uint32_t mantissa = bits & 0x7fffff;
  if (exponent <= 0) {
    if (exponent < -10) return (uint16_t)sign;
    mantissa = (mantissa | 0x800000) >> (1 - exponent);
    return (uint16_t)(sign | ((mantissa + 0x1000) >> 13));
  }
  if (exponent >= 31) return (uint16_t)(sign | 0x7c00);
  if (mantissa & 0x1000) {
    mantissa += 0x2000;
    if (mantissa & 0x800000) {
      mantissa = 0;
      exponent += 1;
      if (exponent >= 31) return (uint16_t)(sign | 0x7c00);
    }
  }
  return (uint16_t)(sign | ((uint32_t)exponent << 10) | (mantissa >> 13));
}

// The shader-side f16(x) conversion: IEEE round to nearest, ties to even.
uint16_t orc_f16_rne(float value) {
  uint32_t x;
  memcpy(&x, &value, 4);
  const uint32_t sign = (x >> 16) & 0x8000;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00);  // >= 65520 rounds to inf
  if (ax < 0x38800000u) {                                    // below 2^-14: subnormal half
    float a;
    memcpy(&a, &ax, 4);
    const float scaled = a * 16777216.0f;  // exact: multiply by 2^24
    return (uint16_t)(sign | (uint32_t)rintf(scaled));  // rintf: ties to even
  }
  const uint32_t e = (ax >> 23) - 112;
  const uint32_t m = ax & 0x7fffff;
  uint32_t half = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (half & 1))) half += 1;
  return (uint16_t)(sign | half);
}

float orc_f16_to_f32(uint16_t bits) { return (float)orc_half_to_float(bits); }

// quantization.ts:11-17
static void scale_and_min(const uint8_t* scales, int index, int* scale, int* min) {
  if (index < 4) {
    *scale = scales[index] & 63;
    *min = scales[index + 4] & 63;
    return;
  }
  *scale = (scales[index + 4] & 0x0f) | ((scales[index - 4] >> 6) << 4);
  *min = (scales[index + 4] >> 4) | ((scales[index] >> 6) << 4);
}

// quantization.ts:19-38
void orc_dequant_q4k_block(const uint8_t* block, float* out) {
  const double d = orc_half_to_float((uint16_t)(block[0] | (block[1] << 8)));
  const double dmin = orc_half_to_float((uint16_t)(block[2] | (block[3] << 8)));
  const uint8_t* scales = block + 4;
  const uint8_t* quants = block + 16;
  int scale_index = 0;
  for (int group = 0; group < 4; ++group) {
    int sl, ml, sh, mh;
    scale_and_min(scales, scale_index++, &sl, &ml);
    scale_and_min(scales, scale_index++, &sh, &mh);
    for (int lane = 0; lane < 32; ++lane) {
      const int packed = quants[group * 32 + lane];
      out[group * 64 + lane] = (float)(d * sl * (packed & 0x0f) - dmin * ml);
      out[group * 64 + lane + 32] = (float)(d * sh * (packed >> 4) - dmin * mh);
    }
  }
}

// quantization.ts:40-44
void orc_dequant_q40_block(const uint8_t* block, float* out) {
  const double d = orc_half_to_float((uint16_t)(block[0] | (block[1] << 8)));
  for (int lane = 0; lane < 16; ++lane) {
    const int packed = block[2 + lane];
    out[lane] = (float)(d * ((packed & 15) - 8));
    out[lane + 16] = (float)(d * ((packed >> 4) - 8));
  }
}

// quantization.ts:46-74
void orc_dequant_q6k_block(const uint8_t* block, float* out) {
  const uint8_t* ql = block;
  const uint8_t* qh = block + 128;
  const int8_t* scales = (const int8_t*)(block + 192);
  const double d = orc_half_to_float((uint16_t)(block[208] | (block[209] << 8)));
  for (int half = 0; half < 2; ++half) {
    const int lo = half * 64, ho = half * 32, so = half * 8, oo = half * 128;
    for (int lane = 0; lane < 32; ++lane) {
      const int sp = lane >> 4;
      const int high = qh[ho + lane];
      const int low_a = ql[lo + lane];
      const int low_b = ql[lo + lane + 32];
      const int q1 = (low_a & 15) | ((high & 3) << 4);
      const int q2 = (low_b & 15) | (((high >> 2) & 3) << 4);
      const int q3 = (low_a >> 4) | (((high >> 4) & 3) << 4);
      const int q4 = (low_b >> 4) | (((high >> 6) & 3) << 4);
      out[oo + lane] = (float)(d * scales[so + sp] * (q1 - 32));
      out[oo + lane + 32] = (float)(d * scales[so + sp + 2] * (q2 - 32));
      out[oo + lane + 64] = (float)(d * scales[so + sp + 4] * (q3 - 32));
      out[oo + lane + 96] = (float)(d * scales[so + sp + 6] * (q4 - 32));
    }
  }
}

// quantization.ts:77-98 (f64 arithmetic as in JS; the stored scale goes through
// Float32Array and the half-up floatToHalf).
void orc_quantize_q40_block(const float* values, uint8_t* out) {
  double signed_max = 0.0, max_abs = 0.0;
  for (int i = 0; i < 32; ++i) {
    const double v = values[i];
    const double a = fabs(v);
    if (a > max_abs) {
      max_abs = a;
      signed_max = v;
    }
  }
  const double scale = signed_max == 0.0 ? 0.0 : signed_max / -8.0;
  const double inverse = scale == 0.0 ? 0.0 : 1.0 / scale;
  const uint16_t bits = orc_float_to_half((double)(float)scale);
  out[0] = (uint8_t)(bits & 0xff);
  out[1] = (uint8_t)(bits >> 8);
  for (int i = 0; i < 16; ++i) {
    double lo = floor((double)values[i] * inverse + 8.5);
    double hi = floor((double)values[i + 16] * inverse + 8.5);
    lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
    hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
    out[i + 2] = (uint8_t)((int)lo | ((int)hi << 4));
  }
}

// quantization.ts:101-131
int orc_requantize_to_q40(const uint8_t* src, size_t src_bytes, int type, int k, int n,
                          uint8_t* out) {
  if (k % 256 != 0) return -1;
  if (type != ORC_Q4_K && type != ORC_Q6_K && type != ORC_Q4_0) return -2;
  const size_t bb = block_bytes(type);
  const int bv = block_values(type);
  const size_t expected = (size_t)n * (size_t)(k / bv) * bb;
  if (src_bytes != expected) return -3;
  float decoded[256];
  size_t so = 0, oo = 0;
  for (int row = 0; row < n; ++row) {
    for (int column = 0; column < k; column += bv) {
      if (type == ORC_Q4_K) orc_dequant_q4k_block(src + so, decoded);
      else if (type == ORC_Q6_K) orc_dequant_q6k_block(src + so, decoded);
      else orc_dequant_q40_block(src + so, decoded);
      for (int sub = 0; sub < bv; sub += 32) {
        orc_quantize_q40_block(decoded + sub, out + oo);
        oo += 18;
      }
      so += bb;
    }
  }
  return 0;
}

// format.ts:65-99
int orc_pack_q40_tile32(const uint8_t* const* parts, const int* part_rows, int nparts, int k,
                        uint8_t* out) {
  if (nparts <= 0 || k % 32 != 0) return -1;
  int n = 0;
  for (int p = 0; p < nparts; ++p) n += part_rows[p];
  const int kblocks = k / 32;
  const int ntiles = (n + 31) / 32;
  memset(out, 0, (size_t)ntiles * kblocks * 32 * 20);
  std::vector<int> row_part(n), row_local(n);
  for (int p = 0, r = 0; p < nparts; ++p)
    for (int i = 0; i < part_rows[p]; ++i, ++r) {
      row_part[r] = p;
      row_local[r] = i;
    }
  for (int tile = 0; tile < ntiles; ++tile)
    for (int kb = 0; kb < kblocks; ++kb)
      for (int lr = 0; lr < 32; ++lr) {
        const int orow = tile * 32 + lr;
        if (orow >= n) continue;
        const uint8_t* src = parts[row_part[orow]] + ((size_t)row_local[orow] * kblocks + kb) * 18;
        uint8_t* dst = out + (((size_t)tile * kblocks + kb) * 32 + lr) * 20;
        dst[0] = src[0];
        dst[1] = src[1];
        memcpy(dst + 4, src + 2, 16);
      }
  return 0;
}

int orc_decode_matrix(const uint8_t* bytes, size_t nbytes, int type, int compact, int k, int n,
                      float* out) {
  if (compact) {
    // format.ts:84-97 layout, decoded as quant-matmul.ts:99-108.
    if (type != ORC_Q4_0 || k % 32 != 0) return -1;
    const int kblocks = k / 32;
    const size_t need = (size_t)((n + 31) / 32) * kblocks * 32 * 20;
    if (nbytes < need) return -2;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
      const int tile = r / 32, lr = r % 32;
      for (int kb = 0; kb < kblocks; ++kb) {
        const uint8_t* b = bytes + (((size_t)tile * kblocks + kb) * 32 + lr) * 20;
        const double d = orc_half_to_float((uint16_t)(b[0] | (b[1] << 8)));
        float* o = out + (size_t)r * k + kb * 32;
        for (int j = 0; j < 16; ++j) {
          o[j] = (float)(d * ((b[4 + j] & 15) - 8));
          o[j + 16] = (float)(d * ((b[4 + j] >> 4) - 8));
        }
      }
    }
    return 0;
  }
  const size_t bb = block_bytes(type);
  const int bv = block_values(type);
  if (!bb || k % bv != 0) return -1;
  const int bpr = k / bv;
  if (nbytes < (size_t)n * bpr * bb) return -2;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n; ++r) {
    for (int b = 0; b < bpr; ++b) {
      const uint8_t* src = bytes + ((size_t)r * bpr + b) * bb;
      float* o = out + (size_t)r * k + (size_t)b * bv;
      if (type == ORC_Q4_K) orc_dequant_q4k_block(src, o);
      else if (type == ORC_Q6_K) orc_dequant_q6k_block(src, o);
      else orc_dequant_q40_block(src, o);
    }
  }
  return 0;
}

// model.ts:30-32: max(1, ceil(sequence * 0.64)) in f64.
uint32_t orc_merged_length(uint32_t sequence) {
  const double v = ceil((double)sequence * 0.64);
  return v < 1.0 ? 1u : (uint32_t)v;
}

int orc_num_threads(void) { return omp_get_max_threads(); }
void orc_set_num_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

// ---------------------------------------------------------------------------
// Forward-pass stages.

// ops.ts:680-725: x[t,:] = f16(dequantQ6K(token_embd[id_t,:])). The shader's f32
// product (d*scale)*q is exact, so it equals the CPU block decode.
void orc_embedding(const uint8_t* token_embd, int vocab, const uint32_t* ids, int tokens,
                   uint16_t* out) {
  (void)vocab;
  const int bpr = kHidden / 256;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < tokens; ++t) {
    float row[256];
    for (int b = 0; b < bpr; ++b) {
      orc_dequant_q6k_block(token_embd + ((size_t)ids[t] * bpr + b) * kEmbedBlockBytes, row);
      for (int j = 0; j < 256; ++j) out[(size_t)t * kHidden + b * 256 + j] = f2h(row[j]);
    }
  }
}

// ops.ts:21-72. value = f32(x) (+ f32(residual), stored back as f16); the sum
// of squares uses the unrounded f32 value; normalized = f16(f32(x) * inv * w).
void orc_residual_rmsnorm(uint16_t* x, const uint16_t* residual, const float* weight,
                          uint16_t* normalized, int rows, int width, float eps) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    uint16_t* xr = x + (size_t)r * width;
    double ss = 0.0;
    for (int c = 0; c < width; ++c) {
      float v = h2f(xr[c]);
      if (residual) {
        v = v + h2f(residual[(size_t)r * width + c]);
        xr[c] = f2h(v);
      }
      ss += (double)v * (double)v;
    }
    const float inv = (float)(1.0 / sqrt((double)(float)(ss / width) + (double)eps));
    for (int c = 0; c < width; ++c) {
      const float a = h2f(xr[c]) * inv;
      normalized[(size_t)r * width + c] = f2h(a * weight[c]);
    }
  }
}

static void f16_row_to_f32(const uint16_t* src, float* dst, int n) {
  int i = 0;
#if defined(__F16C__)
  for (; i + 8 <= n; i += 8) {
    __m128i h = _mm_loadu_si128((const __m128i*)(src + i));
    _mm256_storeu_ps(dst + i, _mm256_cvtph_ps(h));
  }
#endif
  for (; i < n; ++i) dst[i] = h2f(src[i]);
}

static float dot_f32(const float* a, const float* b, int k) {
  float s[16] = {0};
  int i = 0;
  for (; i + 16 <= k; i += 16)
    for (int j = 0; j < 16; ++j) s[j] += a[i + j] * b[i + j];
  float tail = 0.f;
  for (; i < k; ++i) tail += a[i] * b[i];
  double total = tail;
  for (int j = 0; j < 16; ++j) total += s[j];
  return (float)total;
}

// Y[m,n] = X[m,k] . W[n,k]^T with f16 operands, f32 accumulation; output f16
// (the projection kernels store f16, quant-matmul.ts:166-171).
void orc_matmul_f16(const uint16_t* x, const uint16_t* w, int m, int n, int k, float* out_f32,
                    uint16_t* out_f16) {
  std::vector<float> xf((size_t)m * k);
  for (int t = 0; t < m; ++t) f16_row_to_f32(x + (size_t)t * k, xf.data() + (size_t)t * k, k);
#pragma omp parallel
  {
    std::vector<float> wrow(k);
#pragma omp for schedule(static)
    for (int r = 0; r < n; ++r) {
      f16_row_to_f32(w + (size_t)r * k, wrow.data(), k);
      for (int t = 0; t < m; ++t) {
        const float v = dot_f32(xf.data() + (size_t)t * k, wrow.data(), k);
        if (out_f32) out_f32[(size_t)t * n + r] = v;
        if (out_f16) out_f16[(size_t)t * n + r] = f2h(v);
      }
    }
  }
}

// model.ts:95-107: YaRN-scaled table in f64, stored f32 (cos, sin) per
// (position, pair).
void orc_rope_table(int sequence, float* table) {
  const double frequency_scale = 1.0 / 16.0;
  auto correction = [](double beta) {
    return 128.0 * log(16384.0 / (beta * 2.0 * M_PI)) / (2.0 * log(kRopeTheta));
  };
  const double low = floor(correction(32.0));
  const double high = ceil(correction(1.0));
  for (int p = 0; p < sequence; ++p)
    for (int d = 0; d < 64; ++d) {
      double t = (d - low) / fmax(0.001, high - low);
      t = fmin(1.0, fmax(0.0, t));
      const double ramp = 1.0 - t;
      const double frequency = frequency_scale * (1.0 - ramp) + ramp;
      const double angle = p * pow(kRopeTheta, -d / 64.0) * frequency;
      table[((size_t)p * 64 + d) * 2] = (float)cos(angle);
      table[((size_t)p * 64 + d) * 2 + 1] = (float)sin(angle);
    }
}

// ops.ts:168-194: rotate pairs (2i, 2i+1) of each q and k head by the table
// entry of the token's position within its (merged) row.
void orc_rope(const uint16_t* qkv, const int* positions, int tokens, const float* table,
              uint16_t* q, uint16_t* k) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < tokens; ++t) {
    const float* rope = table + (size_t)positions[t] * 128;
    for (int h = 0; h < kQHeads + kKVHeads; ++h) {
      const bool is_q = h < kQHeads;
      const int head = is_q ? h : h - kQHeads;
      const int in_base = t * kQKVWidth + (is_q ? 0 : kQWidth) + head * kHeadDim;
      uint16_t* dst = is_q ? q + ((size_t)t * kQHeads + head) * kHeadDim
                           : k + ((size_t)t * kKVHeads + head) * kHeadDim;
      for (int pair = 0; pair < 64; ++pair) {
        const float c = rope[pair * 2], s = rope[pair * 2 + 1];
        const float even = h2f(qkv[in_base + pair * 2]);
        const float odd = h2f(qkv[in_base + pair * 2 + 1]);
        const float ec = even * c, os = odd * s, es = even * s, oc = odd * c;
        dst[pair * 2] = f2h(ec - os);
        dst[pair * 2 + 1] = f2h(es + oc);
      }
    }
  }
}

// ops.ts:213-362: bidirectional GQA attention over the valid keys of the row.
// Keys are sampled every third position when the row's valid length exceeds
// 2048 (ops.ts:258-269); queries at position >= 16384 get the temperature
// factor of ops.ts:241. Softmax in f64 (the reference keeps f32 stats and f16
// weights); output f16.
void orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, const int* offsets,
                   const uint32_t* lengths, int batch, uint16_t* out) {
  orc_attention_ex(q, k, qkv, offsets, lengths, batch, 1, out);
}

void orc_attention_ex(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, const int* offsets,
                      const uint32_t* lengths, int batch, int sample, uint16_t* out) {
  for (int b = 0; b < batch; ++b) {
    const int len = (int)lengths[b];
    const int base = offsets[b];
    const int stride = sample && len > 2048 ? 3 : 1;
    const int nkeys = (len + stride - 1) / stride;
#pragma omp parallel
    {
      std::vector<float> kf((size_t)nkeys * kHeadDim), vf((size_t)nkeys * kHeadDim);
      std::vector<double> scores(nkeys);
#pragma omp for schedule(static)
      for (int kvh = 0; kvh < kKVHeads; ++kvh) {
        for (int j = 0; j < nkeys; ++j) {
          const int kp = j * stride;
          for (int d = 0; d < kHeadDim; ++d) {
            kf[(size_t)j * kHeadDim + d] = h2f(k[((size_t)(base + kp) * kKVHeads + kvh) * kHeadDim + d]);
            vf[(size_t)j * kHeadDim + d] =
                h2f(qkv[(size_t)(base + kp) * kQKVWidth + kQWidth + kKVWidth + kvh * kHeadDim + d]);
          }
        }
        for (int g = 0; g < kQHeads / kKVHeads; ++g) {
          const int h = kvh * (kQHeads / kKVHeads) + g;
          for (int i = 0; i < len; ++i) {
            float qf[kHeadDim];
            for (int d = 0; d < kHeadDim; ++d)
              qf[d] = h2f(q[((size_t)(base + i) * kQHeads + h) * kHeadDim + d]);
            float temperature = 1.0f;
            if (i >= 16384) temperature = logf(floorf((float)i / 16384.0f) + 1.0f) * 0.1f + 1.0f;
            double mx = -INFINITY;
            for (int j = 0; j < nkeys; ++j) {
              const float dot = dot_f32(qf, kf.data() + (size_t)j * kHeadDim, kHeadDim);
              const double s = (double)(dot * 0.08838834764831845f * temperature);
              scores[j] = s;
              if (s > mx) mx = s;
            }
            double den = 0.0;
            double acc[kHeadDim] = {0};
            for (int j = 0; j < nkeys; ++j) {
              const double p = exp(scores[j] - mx);
              den += p;
              const float* vr = vf.data() + (size_t)j * kHeadDim;
              for (int d = 0; d < kHeadDim; ++d) acc[d] += p * vr[d];
            }
            for (int d = 0; d < kHeadDim; ++d)
              out[((size_t)(base + i) * kQHeads + h) * kHeadDim + d] = f2h((float)(acc[d] / den));
          }
        }
      }
    }
  }
}

// ops.ts:74-89: out = f16(silu(g) * u), silu = g / (1 + exp(-g)) in f32.
void orc_swiglu(const uint16_t* gate_up, int rows, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < kInter; ++c) {
      const float g = h2f(gate_up[(size_t)r * 2 * kInter + c]);
      const float u = h2f(gate_up[(size_t)r * 2 * kInter + kInter + c]);
      const float e = expf(-g);
      const float silu = g / (1.0f + e);
      out[(size_t)r * kInter + c] = f2h(silu * u);
    }
}

// ops.ts:629-661: BOS-preserving adjacent-bin mean. Position 0 is the BOS row
// alone; position p > 0 averages source rows [start, end) with integer
// division; the sum runs in f32 in source order.
void orc_token_merge(const uint16_t* in, const int* src_offsets, const uint32_t* src_lengths,
                     const int* dst_offsets, const uint32_t* dst_lengths, int batch,
                     uint16_t* out) {
  for (int b = 0; b < batch; ++b) {
    const uint32_t sl = src_lengths[b], tl = dst_lengths[b];
#pragma omp parallel for schedule(static)
    for (int p = 0; p < (int)tl; ++p) {
      uint32_t start = 0, end = 1;
      if (p > 0 && tl > 1) {
        const uint32_t st = sl - 1, tt = tl - 1;
        start = 1 + ((uint32_t)(p - 1) * st) / tt;
        end = 1 + ((uint32_t)p * st) / tt;
        if (end < start + 1) end = start + 1;
        if (end > sl) end = sl;
      }
      for (int c = 0; c < kHidden; ++c) {
        float total = 0.f;
        for (uint32_t s = start; s < end; ++s)
          total += h2f(in[((size_t)src_offsets[b] + s) * kHidden + c]);
        out[((size_t)dst_offsets[b] + p) * kHidden + c] = f2h(total / (float)(end - start));
      }
    }
  }
}

// ops.ts:596-616: mean over the valid rows (f32, in row order), then L2.
void orc_mean_pool(const uint16_t* in, const int* offsets, const uint32_t* lengths, int batch,
                   float* out) {
  for (int b = 0; b < batch; ++b) {
    double ss = 0.0;
    for (int c = 0; c < kHidden; ++c) {
      float total = 0.f;
      for (uint32_t p = 0; p < lengths[b]; ++p) total += h2f(in[((size_t)offsets[b] + p) * kHidden + c]);
      const float mean = total / (float)lengths[b];
      out[(size_t)b * kHidden + c] = mean;
      ss += (double)mean * mean;
    }
    const float inv = (float)(1.0 / sqrt(ss));
    for (int c = 0; c < kHidden; ++c) out[(size_t)b * kHidden + c] *= inv;
  }
}

// ---------------------------------------------------------------------------
// Model and forward.

}  // extern "C"

struct orc_model {
  int n_layers;
  int vocab;
  const uint8_t* token_embd;
  const float* attn_norm[16];
  const float* ffn_norm[16];
  const float* output_norm;
  std::vector<uint16_t> w[16][4];  // effective f16 weights, n x k row-major
};

static const int kProjN[4] = {kQKVWidth, kHidden, 2 * kInter, kHidden};
static const int kProjK[4] = {kHidden, kQWidth, kHidden, kInter};

extern "C" {

orc_model* orc_model_create(const orc_model_desc* desc, char* err, size_t errlen) {
  if (!desc || desc->n_layers < kMergeAfterLayer + 1 || desc->n_layers > 16) {
    set_err(err, errlen, "n_layers must be in [5, 16]");
    return nullptr;
  }
  if (!desc->token_embd || desc->vocab <= 0 ||
      desc->token_embd_bytes != (size_t)desc->vocab * 8 * kEmbedBlockBytes) {
    set_err(err, errlen, "token_embd must be Q6_K [2048 x vocab]");
    return nullptr;
  }
  orc_model* m = new orc_model();
  m->n_layers = desc->n_layers;
  m->vocab = desc->vocab;
  m->token_embd = desc->token_embd;
  m->output_norm = desc->output_norm;
  for (int l = 0; l < desc->n_layers; ++l) {
    m->attn_norm[l] = desc->attn_norm[l];
    m->ffn_norm[l] = desc->ffn_norm[l];
    const orc_proj* projs[4] = {&desc->qkv[l], &desc->o[l], &desc->gate_up[l], &desc->down[l]};
    for (int which = 0; which < 4; ++which) {
      const orc_proj* pr = projs[which];
      const int n = kProjN[which], k = kProjK[which];
      int rows = 0;
      for (int p = 0; p < pr->nparts; ++p) rows += pr->parts[p].n;
      if (rows != n) {
        char msg[128];
        snprintf(msg, sizeof msg, "layer %d projection %d has %d rows, expected %d", l, which, rows, n);
        set_err(err, errlen, msg);
        delete m;
        return nullptr;
      }
      m->w[l][which].resize((size_t)n * k);
      std::vector<float> tmp;
      int row0 = 0;
      for (int p = 0; p < pr->nparts; ++p) {
        const orc_part& part = pr->parts[p];
        if (part.k != k) {
          set_err(err, errlen, "projection part has the wrong K");
          delete m;
          return nullptr;
        }
        tmp.resize((size_t)part.n * k);
        if (orc_decode_matrix(part.data, part.nbytes, part.type, part.compact, k, part.n, tmp.data())) {
          set_err(err, errlen, "projection part could not be decoded");
          delete m;
          return nullptr;
        }
        uint16_t* dst = m->w[l][which].data() + (size_t)row0 * k;
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)part.n * k; ++i) dst[i] = f2h(tmp[i]);
        row0 += part.n;
      }
    }
  }
  return m;
}

void orc_model_destroy(orc_model* model) { delete model; }

int orc_model_weights_f16(const orc_model* model, int layer, int which, uint16_t* out) {
  if (!model || layer < 0 || layer >= model->n_layers || which < 0 || which > 3) return -1;
  memcpy(out, model->w[layer][which].data(), model->w[layer][which].size() * 2);
  return 0;
}

int orc_forward(const orc_model* m, int batch, int sequence, const uint32_t* ids,
                const uint32_t* lengths, float* out, uint16_t* x_dump, uint16_t* norm_dump,
                int* tokens_per_layer, char* err, size_t errlen) {
  return orc_forward_ex(m, batch, sequence, ids, lengths, 0, out, x_dump, norm_dump, tokens_per_layer, err, errlen);
}

int orc_forward_ex(const orc_model* m, int batch, int sequence, const uint32_t* ids,
                   const uint32_t* lengths, int exact, float* out, uint16_t* x_dump, uint16_t* norm_dump,
                   int* tokens_per_layer, char* err, size_t errlen) {
  if (!m || batch < 1 || sequence < 1) {
    set_err(err, errlen, "invalid plan shape");
    return -1;
  }
  for (int b = 0; b < batch; ++b)
    if (lengths[b] < 1 || lengths[b] > (uint32_t)sequence) {
      set_err(err, errlen, "lengths must be in [1, sequence]");
      return -1;
    }
  for (long long i = 0; i < (long long)batch * sequence; ++i)
    if (ids[i] >= (uint32_t)m->vocab) {
      set_err(err, errlen, "token id out of vocabulary");
      return -1;
    }
  // model.ts:226-233
  const uint32_t merged_seq = orc_merged_length((uint32_t)sequence);
  std::vector<uint32_t> tgt(batch);
  std::vector<int> off0(batch + 1, 0), off1(batch + 1, 0);
  for (int b = 0; b < batch; ++b) {
    const uint32_t src = lengths[b] < (uint32_t)sequence ? lengths[b] : (uint32_t)sequence;
    const uint32_t ml = orc_merged_length(src);
    tgt[b] = exact ? lengths[b] : (ml < merged_seq ? ml : merged_seq);
    off0[b + 1] = off0[b] + (int)lengths[b];
    off1[b + 1] = off1[b] + (int)tgt[b];
  }
  const int t0 = off0[batch], t1 = off1[batch];
  std::vector<uint32_t> packed_ids(t0);
  std::vector<int> pos0(t0), pos1(t1);
  for (int b = 0; b < batch; ++b) {
    for (uint32_t p = 0; p < lengths[b]; ++p) {
      packed_ids[off0[b] + p] = ids[(size_t)b * sequence + p];
      pos0[off0[b] + p] = (int)p;
    }
    for (uint32_t p = 0; p < tgt[b]; ++p) pos1[off1[b] + p] = (int)p;
  }
  std::vector<float> rope((size_t)sequence * 128);
  orc_rope_table(sequence, rope.data());

  std::vector<uint16_t> x((size_t)t0 * kHidden), norm((size_t)t0 * kHidden);
  std::vector<uint16_t> qkv((size_t)t0 * kQKVWidth), qb((size_t)t0 * kQWidth),
      kb((size_t)t0 * kKVWidth), attn((size_t)t0 * kQWidth), delta((size_t)t0 * kHidden),
      gu((size_t)t0 * 2 * kInter), ffn((size_t)t0 * kInter);

  orc_embedding(m->token_embd, m->vocab, packed_ids.data(), t0, x.data());
  orc_residual_rmsnorm(x.data(), nullptr, m->attn_norm[0], norm.data(), t0, kHidden, kEpsilon);

  int tokens = t0;
  const int* offsets = off0.data();
  const uint32_t* layer_len = lengths;
  const int* positions = pos0.data();
  for (int l = 0; l < m->n_layers; ++l) {
    if (l == kMergeAfterLayer && !exact) {  // model.ts:157, merge both x and normalized
      std::vector<uint16_t> xm((size_t)t1 * kHidden), nm((size_t)t1 * kHidden);
      orc_token_merge(x.data(), off0.data(), lengths, off1.data(), tgt.data(), batch, xm.data());
      orc_token_merge(norm.data(), off0.data(), lengths, off1.data(), tgt.data(), batch, nm.data());
      memcpy(x.data(), xm.data(), xm.size() * 2);
      memcpy(norm.data(), nm.data(), nm.size() * 2);
      tokens = t1;
      offsets = off1.data();
      layer_len = tgt.data();
      positions = pos1.data();
    }
    orc_matmul_f16(norm.data(), m->w[l][0].data(), tokens, kQKVWidth, kHidden, nullptr, qkv.data());
    orc_rope(qkv.data(), positions, tokens, rope.data(), qb.data(), kb.data());
    orc_attention_ex(qb.data(), kb.data(), qkv.data(), offsets, layer_len, batch, exact ? 0 : 1, attn.data());
    orc_matmul_f16(attn.data(), m->w[l][1].data(), tokens, kHidden, kQWidth, nullptr, delta.data());
    orc_residual_rmsnorm(x.data(), delta.data(), m->ffn_norm[l], norm.data(), tokens, kHidden, kEpsilon);
    orc_matmul_f16(norm.data(), m->w[l][2].data(), tokens, 2 * kInter, kHidden, nullptr, gu.data());
    orc_swiglu(gu.data(), tokens, ffn.data());
    orc_matmul_f16(ffn.data(), m->w[l][3].data(), tokens, kHidden, kInter, nullptr, delta.data());
    const float* next = l + 1 < m->n_layers ? m->attn_norm[l + 1] : m->output_norm;
    orc_residual_rmsnorm(x.data(), delta.data(), next, norm.data(), tokens, kHidden, kEpsilon);
    const size_t stride = (size_t)batch * sequence * kHidden;
    if (x_dump) memcpy(x_dump + (size_t)l * stride, x.data(), (size_t)tokens * kHidden * 2);
    if (norm_dump) memcpy(norm_dump + (size_t)l * stride, norm.data(), (size_t)tokens * kHidden * 2);
    if (tokens_per_layer) tokens_per_layer[l] = tokens;
  }
  orc_mean_pool(norm.data(), off1.data(), tgt.data(), batch, out);
  return 0;
}

}  // extern "C"
