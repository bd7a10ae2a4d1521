/* CPU oracle for the attention path (TEST INFRASTRUCTURE ONLY; see nbl_oracle.h).
 *
 * Build with -O2 -ffp-contract=off (oracle/Makefile): the reference compiles its scalar kernels the same way
 * (CMakeLists.txt:72-73), and contracting a*b+c into an FMA would change the rounding this file must share
 * with them. C's expf/exp/pow/cos/sin are the functions the reference's std:: overloads resolve to for the
 * same argument types, so results are bit-identical on the same libm.
 */
#include "nbl_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Widening: zeros, subnormals (renormalised into float normals), infinities and NaN payloads
 * (src/fp16.h:18-42). */
float orc_fp16_to_fp32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
  uint32_t man = (uint32_t)h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    int e = 113; /* a subnormal half is man * 2^-24: shift the leading one up to bit 10 */
    while ((man & 0x400u) == 0) {
      man <<= 1;
      --e;
    }
    bits = sign | ((uint32_t)e << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* Narrowing with round-to-nearest-even; overflow to infinity, underflow to signed zero, NaN kept quiet
 * (src/fp16.h:46-71). */
uint16_t orc_fp32_to_fp16(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof x);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t e = (x >> 23) & 0xFFu;
  uint32_t m = x & 0x7FFFFFu;
  if (e == 0xFFu) return (uint16_t)(sign | 0x7C00u | (m ? (0x200u | (m >> 13)) : 0u));
  const int exp = (int)e - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    m |= 0x800000u;
    const int shift = 14 - exp;
    uint32_t half = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) ++half;
    return (uint16_t)(sign | half);
  }
  uint32_t half = ((uint32_t)exp << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) ++half; /* a carry may reach infinity, as it should */
  return (uint16_t)(sign | half);
}

float orc_bf16_to_fp32(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

uint16_t orc_fp32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof x);
  if ((x & 0x7F800000u) == 0x7F800000u && (x & 0x7FFFFFu)) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7FFFu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

void orc_fp16_to_fp32_n(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_fp16_to_fp32(src[i]);
}
void orc_fp32_to_fp16_n(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_fp32_to_fp16(src[i]);
}
void orc_bf16_to_fp32_n(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_bf16_to_fp32(src[i]);
}
void orc_fp32_to_bf16_n(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = orc_fp32_to_bf16(src[i]);
}

/* Running max in the reference's comparison form (std::max keeps the first argument unless it is less),
 * exp of the max-subtracted float, double sum, one float reciprocal (src/backend/cpu/ref_ops.cpp:66-77). */
void orc_softmax_inplace(float* x, int64_t n) {
  if (n <= 0) return;
  float m = x[0];
  for (int64_t i = 1; i < n; ++i) m = (m < x[i]) ? x[i] : m;
  double sum = 0;
  for (int64_t i = 0; i < n; ++i) {
    x[i] = expf(x[i] - m);
    sum += x[i];
  }
  const float inv = (float)(1.0 / sum);
  for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

/* Pair (i, i+half) for NeoX, (2i, 2i+1) otherwise; angle and trig in double, rotation in float
 * (src/backend/cpu/ref_ops.cpp:166-185). */
void orc_rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, float freq_base, int neox,
              const float* freq_factors) {
  const int64_t half = head_dim / 2;
  for (int64_t t = 0; t < n; ++t) {
    const double pos = (double)(pos0 + t);
    for (int64_t h = 0; h < n_heads; ++h) {
      float* v = x + (t * n_heads + h) * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        double theta = pos * pow((double)freq_base, -2.0 * (double)i / (double)head_dim);
        if (freq_factors) theta /= freq_factors[i];
        const float c = (float)cos(theta), s = (float)sin(theta);
        float* a = neox ? &v[i] : &v[2 * i];
        float* b = neox ? &v[i + half] : &v[2 * i + 1];
        const float a0 = *a, b0 = *b;
        *a = a0 * c - b0 * s;
        *b = a0 * s + b0 * c;
      }
    }
  }
}

/* Scores with a left-to-right float dot, scaled by 1/sqrtf(head_dim); softmax; float accumulation of p*v
 * (src/backend/cpu/ref_ops.cpp:188-214). Query head h reads KV head h / (n_heads / n_kv_heads). */
void orc_attention_heads(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                         int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t head_begin, int64_t head_end,
                         float* scratch) {
  const int64_t group = n_heads / n_kv_heads;
  const float scale = 1.0f / sqrtf((float)head_dim);
  for (int64_t h = head_begin; h < head_end; ++h) {
    const int64_t kvh = h / group;
    for (int64_t t = 0; t < n; ++t) {
      const float* qh = q + (t * n_heads + h) * head_dim;
      const int64_t len = pos0 + t + 1;
      for (int64_t j = 0; j < len; ++j) {
        const float* kj = k + (j * n_kv_heads + kvh) * head_dim;
        float dot = 0;
        for (int64_t d = 0; d < head_dim; ++d) dot += qh[d] * kj[d];
        scratch[j] = dot * scale;
      }
      orc_softmax_inplace(scratch, len);
      float* o = out + (t * n_heads + h) * head_dim;
      for (int64_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
      for (int64_t j = 0; j < len; ++j) {
        const float* vj = v + (j * n_kv_heads + kvh) * head_dim;
        const float pj = scratch[j];
        for (int64_t d = 0; d < head_dim; ++d) o[d] += pj * vj[d];
      }
    }
  }
}

int orc_attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                  int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
  float* scratch = (float*)malloc((size_t)(pos0 + n) * sizeof(float));
  if (!scratch) return -1;
  orc_attention_heads(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, 0, n_heads, scratch);
  free(scratch);
  return 0;
}

void orc_add_bias(float* x, const float* bias, int64_t width, int64_t n) {
  for (int64_t t = 0; t < n; ++t)
    for (int64_t i = 0; i < width; ++i) x[t * width + i] += bias[i];
}

void orc_gather_pages(const uint16_t* pool, const int32_t* page_table, int64_t len, int64_t n_kv_heads,
                      int64_t head_dim, int64_t page_size, int bf16, float* k_out, float* v_out) {
  const int64_t block = n_kv_heads * page_size * head_dim; /* elements of one page's K (or V) half */
  for (int64_t j = 0; j < len; ++j) {
    const int64_t page = page_table[j / page_size], slot = j % page_size;
    for (int64_t h = 0; h < n_kv_heads; ++h) {
      const uint16_t* ks = pool + page * 2 * block + (h * page_size + slot) * head_dim;
      const uint16_t* vs = ks + block;
      float* kd = k_out + (j * n_kv_heads + h) * head_dim;
      float* vd = v_out + (j * n_kv_heads + h) * head_dim;
      for (int64_t d = 0; d < head_dim; ++d) {
        kd[d] = bf16 ? orc_bf16_to_fp32(ks[d]) : orc_fp16_to_fp32(ks[d]);
        vd[d] = bf16 ? orc_bf16_to_fp32(vs[d]) : orc_fp16_to_fp32(vs[d]);
      }
    }
  }
}

void orc_lse_merge(const float* part_o, const float* part_lse, int64_t n_parts, int64_t rows, int64_t head_dim,
                   float* out, float* lse_out) {
  for (int64_t r = 0; r < rows; ++r) {
    double mx = -INFINITY;
    for (int64_t p = 0; p < n_parts; ++p)
      if (part_lse[p * rows + r] > mx) mx = part_lse[p * rows + r];
    float* o = out + r * head_dim;
    if (mx == -INFINITY) {
      for (int64_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
      if (lse_out) lse_out[r] = -INFINITY;
      continue;
    }
    double wsum = 0;
    for (int64_t p = 0; p < n_parts; ++p) wsum += exp((double)part_lse[p * rows + r] - mx);
    for (int64_t d = 0; d < head_dim; ++d) {
      double acc = 0;
      for (int64_t p = 0; p < n_parts; ++p) {
        const double w = exp((double)part_lse[p * rows + r] - mx);
        if (w > 0) acc += w * part_o[(p * rows + r) * head_dim + d];
      }
      o[d] = (float)(acc / wsum);
    }
    if (lse_out) lse_out[r] = (float)(mx + log(wsum));
  }
}

/* ---- the model's other ops ---- */

static float orc_weight_at(const void* w, int dtype, int64_t i) {
  return dtype == 0 ? ((const float*)w)[i] : orc_fp16_to_fp32(((const uint16_t*)w)[i]);
}

int orc_embed(const void* table, int dtype, int64_t ne0, int64_t n_rows, const int32_t* ids, int64_t n, float* out) {
  for (int64_t t = 0; t < n; ++t) {
    const int64_t id = ids[t];
    if (id < 0 || id >= n_rows) return -1;
    for (int64_t k = 0; k < ne0; ++k) out[t * ne0 + k] = orc_weight_at(table, dtype, id * ne0 + k);
  }
  return 0;
}

void orc_matmul(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n) {
  for (int64_t t = 0; t < n; ++t) {
    const float* xt = x + t * ne0;
    for (int64_t r = 0; r < ne1; ++r) {
      float acc = 0;
      for (int64_t k = 0; k < ne0; ++k) acc += xt[k] * orc_weight_at(w, dtype, r * ne0 + k);
      y[t * ne1 + r] = acc;
    }
  }
}

void orc_rmsnorm(const float* x, const float* weight, float* y, int64_t n, int64_t d, float eps) {
  for (int64_t t = 0; t < n; ++t) {
    const float* xt = x + t * d;
    double ss = 0;
    for (int64_t i = 0; i < d; ++i) ss += (double)xt[i] * xt[i];
    const double scale = 1.0 / sqrt(ss / (double)d + (double)eps);
    for (int64_t i = 0; i < d; ++i) y[t * d + i] = (float)(xt[i] * scale * weight[i]);
  }
}

void orc_add(float* x, const float* y, int64_t count) {
  for (int64_t i = 0; i < count; ++i) x[i] += y[i];
}

void orc_silu_mul(float* gate, const float* up, int64_t count) {
  for (int64_t i = 0; i < count; ++i) {
    const float g = gate[i];
    gate[i] = g / (1.0f + expf(-g)) * up[i];
  }
}

/* ---- quantized weights (Q8_0-activation family) ---- */

static uint16_t orc_rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

void orc_quantize_q8_0(const float* x, uint8_t* blocks, int64_t n) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* xb = x + b * 32;
    uint8_t* o = blocks + b * 34;
    float amax = 0.f;
    int has_nan = 0;
    for (int j = 0; j < 32; ++j) {
      amax = fmaxf(amax, fabsf(xb[j]));
      has_nan |= isnan(xb[j]);
    }
    const float d = has_nan ? NAN : amax / 127.f;
    const float id = d != 0.f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; ++j) {
      const float r = roundf(xb[j] * id);
      o[2 + j] = (uint8_t)(int8_t)(r != r ? 0 : (int)fminf(127.f, fmaxf(-127.f, r)));
    }
    const uint16_t h = orc_fp32_to_fp16(d);
    o[0] = (uint8_t)(h & 0xFF);
    o[1] = (uint8_t)(h >> 8);
  }
}

static int64_t orc_block_bytes(int dtype) { return dtype == 2 ? 18 : dtype == 6 ? 22 : dtype == 8 ? 34 : 0; }

int orc_dequantize_row(int dtype, const void* src, float* dst, int64_t n) {
  const uint8_t* p = (const uint8_t*)src;
  const int64_t bb = orc_block_bytes(dtype);
  if (!bb) return -1;
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* blk = p + b * bb;
    const float d = orc_fp16_to_fp32(orc_rd16(blk));
    if (dtype == 8) {
      for (int j = 0; j < 32; ++j) dst[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
    } else if (dtype == 2) {
      for (int j = 0; j < 16; ++j) {
        dst[b * 32 + j] = (float)((blk[2 + j] & 0x0F) - 8) * d;
        dst[b * 32 + j + 16] = (float)((blk[2 + j] >> 4) - 8) * d;
      }
    } else {
      const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
      for (int j = 0; j < 16; ++j) {
        const int x0 = ((blk[6 + j] & 0x0F) | (((qh >> j) << 4) & 0x10)) - 16;
        const int x1 = ((blk[6 + j] >> 4) | ((qh >> (j + 12)) & 0x10)) - 16;
        dst[b * 32 + j] = (float)x0 * d;
        dst[b * 32 + j + 16] = (float)x1 * d;
      }
    }
  }
  return 0;
}

int orc_matmul_q(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n) {
  const int64_t bb = orc_block_bytes(dtype), nb = ne0 / 32;
  if (!bb) return -1;
  uint8_t* xa = (uint8_t*)malloc((size_t)(nb * 34));
  if (!xa) return -1;
  for (int64_t t = 0; t < n; ++t) {
    orc_quantize_q8_0(x + t * ne0, xa, ne0);
    for (int64_t r = 0; r < ne1; ++r) {
      const uint8_t* wr = (const uint8_t*)w + r * nb * bb;
      float sum = 0.f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* bw = wr + b * bb;
        const uint8_t* ba = xa + b * 34;
        const int8_t* aq = (const int8_t*)(ba + 2);
        const float dw = orc_fp16_to_fp32(orc_rd16(bw)), da = orc_fp16_to_fp32(orc_rd16(ba));
        if (dtype == 8) {
          int s = 0;
          for (int j = 0; j < 32; ++j) s += (int8_t)bw[2 + j] * aq[j];
          sum += (float)s * (dw * da);
        } else if (dtype == 2) {
          int s0 = 0, s1 = 0;
          for (int j = 0; j < 16; ++j) {
            s0 += ((bw[2 + j] & 0x0F) - 8) * aq[j];
            s1 += ((bw[2 + j] >> 4) - 8) * aq[j + 16];
          }
          sum += (float)(s0 + s1) * dw * da;
        } else {
          const uint32_t qh = (uint32_t)bw[2] | ((uint32_t)bw[3] << 8) | ((uint32_t)bw[4] << 16) | ((uint32_t)bw[5] << 24);
          int s0 = 0, s1 = 0;
          for (int j = 0; j < 16; ++j) {
            s0 += (((bw[6 + j] & 0x0F) | (((qh >> j) << 4) & 0x10)) - 16) * aq[j];
            s1 += (((bw[6 + j] >> 4) | ((qh >> (j + 12)) & 0x10)) - 16) * aq[j + 16];
          }
          sum += (dw * da) * (float)(s0 + s1);
        }
      }
      y[t * ne1 + r] = sum;
    }
  }
  free(xa);
  return 0;
}
