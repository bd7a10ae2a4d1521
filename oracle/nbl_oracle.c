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

static int orc_dequantize_row_ext(int dtype, const uint8_t* p, float* dst, int64_t n);
static int orc_matmul_q_ext(const uint8_t* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y,
                            int64_t n);

int orc_dequantize_row(int dtype, const void* src, float* dst, int64_t n) {
  const uint8_t* p = (const uint8_t*)src;
  const int64_t bb = orc_block_bytes(dtype);
  if (!bb) return orc_dequantize_row_ext(dtype, p, dst, n);
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

/* One weight row of nb Q4_0 / Q5_0 / Q8_0 blocks against nb Q8_0 activation blocks (src/quant.cpp:310-366). */
static float orc_dot_q8_0_family(int dtype, const uint8_t* wr, const uint8_t* xa, int64_t nb, int64_t bb) {
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
  return sum;
}

int orc_matmul_q(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n) {
  const int64_t bb = orc_block_bytes(dtype), nb = ne0 / 32;
  if (!bb) return orc_matmul_q_ext((const uint8_t*)w, dtype, ne0, ne1, x, y, n);
  uint8_t* xa = (uint8_t*)malloc((size_t)(nb * 34));
  if (!xa) return -1;
  for (int64_t t = 0; t < n; ++t) {
    orc_quantize_q8_0(x + t * ne0, xa, ne0);
    for (int64_t r = 0; r < ne1; ++r) y[t * ne1 + r] = orc_dot_q8_0_family(dtype, (const uint8_t*)w + r * nb * bb, xa, nb, bb);
  }
  free(xa);
  return 0;
}

/* ---- Q5_1 (Q8_1 activations) and the k-quants Q4_K / Q5_K / Q6_K (Q8_K activations), src/quant.h:50-99 ---- */

static int64_t orc_ext_block_bytes(int dtype) {
  return dtype == 7 ? 24 : dtype == 12 ? 144 : dtype == 13 ? 176 : dtype == 14 ? 210 : 0;
}

/* The j-th 6-bit scale and minimum of a Q4_K / Q5_K super-block's 12 packed bytes (src/quant.cpp:54-63): j < 4
 * in the low 6 bits of bytes j and j + 4; j >= 4 in the nibbles of byte j + 4 with their top two bits taken from
 * bits 6-7 of bytes j - 4 (scale) and j (minimum). */
static void orc_scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* The 256 integer values of a k-quant super-block in element order (src/quant.cpp:67-96). Q4_K: element 64c + l
 * is the low nibble of qs[32c + l], element 64c + 32 + l its high nibble; Q5_K adds 16 where bit (2c) resp.
 * (2c + 1) of qh[l] is set; Q6_K combines ql nibbles and qh bit pairs per 128-element half, minus 32. */
static void orc_expand_k(int dtype, const uint8_t* blk, int8_t a[256]) {
  if (dtype == 14) {
    for (int h = 0; h < 2; ++h)
      for (int l = 0; l < 32; ++l) {
        const uint8_t* ql = blk + 64 * h;
        const int qh = blk[128 + 32 * h + l];
        a[128 * h + l] = (int8_t)(((ql[l] & 0xF) | ((qh & 3) << 4)) - 32);
        a[128 * h + 32 + l] = (int8_t)(((ql[32 + l] & 0xF) | (((qh >> 2) & 3) << 4)) - 32);
        a[128 * h + 64 + l] = (int8_t)(((ql[l] >> 4) | (((qh >> 4) & 3) << 4)) - 32);
        a[128 * h + 96 + l] = (int8_t)(((ql[32 + l] >> 4) | (((qh >> 6) & 3) << 4)) - 32);
      }
    return;
  }
  const uint8_t* qs = blk + (dtype == 13 ? 48 : 16);
  const uint8_t* qh = blk + 16;
  for (int c = 0; c < 4; ++c)
    for (int l = 0; l < 32; ++l) {
      int lo = qs[32 * c + l] & 0xF, hi = qs[32 * c + l] >> 4;
      if (dtype == 13) {
        lo += (qh[l] >> (2 * c)) & 1 ? 16 : 0;
        hi += (qh[l] >> (2 * c + 1)) & 1 ? 16 : 0;
      }
      a[64 * c + l] = (int8_t)lo;
      a[64 * c + 32 + l] = (int8_t)hi;
    }
}

/* Dequantization (src/quant.cpp:98-115, :206-242): Q5_1 x = q * d + m; Q4_K / Q5_K x = (d * sc) * q - dmin * m per
 * 32-element sub-block; Q6_K x = (d * scale) * q per 16-element sub-block. Each product and sum rounded on its own. */
static int orc_dequantize_row_ext(int dtype, const uint8_t* p, float* dst, int64_t n) {
  const int64_t bb = orc_ext_block_bytes(dtype);
  if (!bb) return -1;
  if (dtype == 7) {
    for (int64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = p + b * bb;
      const float d = orc_fp16_to_fp32(orc_rd16(blk)), m = orc_fp16_to_fp32(orc_rd16(blk + 2));
      const uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
      for (int j = 0; j < 16; ++j) {
        const int x0 = (blk[8 + j] & 0x0F) | (((qh >> j) << 4) & 0x10);
        const int x1 = (blk[8 + j] >> 4) | ((qh >> (j + 12)) & 0x10);
        dst[b * 32 + j] = (float)x0 * d + m;
        dst[b * 32 + j + 16] = (float)x1 * d + m;
      }
    }
    return 0;
  }
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* blk = p + b * bb;
    int8_t a[256];
    orc_expand_k(dtype, blk, a);
    float* o = dst + b * 256;
    if (dtype == 14) {
      const float d = orc_fp16_to_fp32(orc_rd16(blk + 208));
      for (int k = 0; k < 16; ++k) {
        const float dk = d * (float)(int8_t)blk[192 + k];
        for (int l = 0; l < 16; ++l) o[16 * k + l] = dk * (float)a[16 * k + l];
      }
    } else {
      const float d = orc_fp16_to_fp32(orc_rd16(blk)), dmin = orc_fp16_to_fp32(orc_rd16(blk + 2));
      for (int k = 0; k < 8; ++k) {
        int sc, m;
        orc_scale_min_k4(k, blk + 4, &sc, &m);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        for (int l = 0; l < 32; ++l) o[32 * k + l] = d1 * (float)a[32 * k + l] - m1;
      }
    }
  }
  return 0;
}

/* Activations to Q8_1 blocks (36 bytes: fp16 d, fp16 s, 32 int8), src/quant.cpp:260-273: d and q as Q8_0, and
 * s = fp16(sum(q) * d) from the scale before its fp16 rounding. */
void orc_quantize_q8_1(const float* x, uint8_t* blocks, int64_t n) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* xb = x + b * 32;
    uint8_t* o = blocks + b * 36;
    float amax = 0.f;
    int has_nan = 0;
    for (int j = 0; j < 32; ++j) {
      amax = fmaxf(amax, fabsf(xb[j]));
      has_nan |= isnan(xb[j]);
    }
    const float d = has_nan ? NAN : amax / 127.f;
    const float id = d != 0.f ? 1.0f / d : 0.0f;
    int sum = 0;
    for (int j = 0; j < 32; ++j) {
      const float r = roundf(xb[j] * id);
      const int q = r != r ? 0 : (int)fminf(127.f, fmaxf(-127.f, r));
      o[4 + j] = (uint8_t)(int8_t)q;
      sum += q;
    }
    const uint16_t hd = orc_fp32_to_fp16(d), hs = orc_fp32_to_fp16((float)sum * d);
    o[0] = (uint8_t)(hd & 0xFF);
    o[1] = (uint8_t)(hd >> 8);
    o[2] = (uint8_t)(hs & 0xFF);
    o[3] = (uint8_t)(hs >> 8);
  }
}

/* Activations to Q8_K blocks (292 bytes: float d, 256 int8, 16 int16 sums of 16), src/quant.cpp:276-307: the
 * element of largest magnitude (the first on ties) gives iscale = -127 / max, q = round-half-even(iscale * x)
 * after clamping to [-127, 127] (NaN -> 0), d = 1 / iscale; an all-zero block stays zero; a NaN makes d NaN. */
void orc_quantize_q8_K(const float* x, uint8_t* blocks, int64_t n) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const float* xb = x + b * 256;
    uint8_t* o = blocks + b * 292;
    memset(o, 0, 292);
    float max = 0.f, amax = 0.f, d = 0.f;
    int has_nan = 0;
    for (int j = 0; j < 256; ++j) {
      const float ax = fabsf(xb[j]);
      if (ax > amax) {
        amax = ax;
        max = xb[j];
      }
      has_nan |= isnan(xb[j]);
    }
    int8_t* q = (int8_t*)(o + 4);
    if (amax != 0.f) {
      const float iscale = -127.f / max;
      for (int j = 0; j < 256; ++j) {
        const float v = iscale * xb[j];
        q[j] = (int8_t)(v != v ? 0 : (int)nearbyintf(fminf(127.f, fmaxf(-127.f, v))));
      }
      for (int g = 0; g < 16; ++g) {
        int sum = 0;
        for (int i = 0; i < 16; ++i) sum += q[16 * g + i];
        const int16_t s16 = (int16_t)sum;
        memcpy(o + 260 + 2 * g, &s16, 2);
      }
      d = 1.f / iscale;
    }
    if (has_nan) d = NAN;
    memcpy(o, &d, 4);
  }
}

/* y[t, r] for Q5_1 (per block (d_w * d_a) * sumi + m_w * s_a, then added to the row sum, src/quant.cpp:371-392)
 * and the k-quants (src/quant.cpp:117-146 and :399-418): per super-block eight int32 lanes (element e feeds lane
 * e % 8, each product scaled by its sub-block's scale), sums[l] += (d_w * d_a) * lane[l]; Q4_K / Q5_K also subtract
 * (dmin_w * d_a) * sum_k(bsum_k * m_k) from the running total; the eight lane sums are added to the total last. */
/* One weight row of nb Q5_1 blocks against Q8_1 ones, or of nb k-quant super-blocks against Q8_K ones. */
static float orc_dot_ext(int dtype, const uint8_t* wr, const uint8_t* xa, int64_t nb) {
  const int64_t bb = orc_ext_block_bytes(dtype);
  const int kq = dtype != 7;
  const int64_t ab = kq ? 292 : 36;
  float sum = 0.f, sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* bw = wr + b * bb;
    const uint8_t* ba = xa + b * ab;
    if (!kq) {
      const int8_t* aq = (const int8_t*)(ba + 4);
      const uint32_t qh = (uint32_t)bw[4] | ((uint32_t)bw[5] << 8) | ((uint32_t)bw[6] << 16) | ((uint32_t)bw[7] << 24);
      int s0 = 0, s1 = 0;
      for (int j = 0; j < 16; ++j) {
        s0 += ((bw[8 + j] & 0x0F) | (((qh >> j) << 4) & 0x10)) * aq[j];
        s1 += ((bw[8 + j] >> 4) | ((qh >> (j + 12)) & 0x10)) * aq[j + 16];
      }
      const float dw = orc_fp16_to_fp32(orc_rd16(bw)), mw = orc_fp16_to_fp32(orc_rd16(bw + 2));
      const float da = orc_fp16_to_fp32(orc_rd16(ba)), sa = orc_fp16_to_fp32(orc_rd16(ba + 2));
      sum += (dw * da) * (float)(s0 + s1) + mw * sa;
      continue;
    }
    float da;
    memcpy(&da, ba, 4);
    const int8_t* aq = (const int8_t*)(ba + 4);
    int8_t a[256];
    orc_expand_k(dtype, bw, a);
    int lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (dtype == 14) {
      for (int e = 0; e < 256; ++e) lane[e & 7] += (int8_t)bw[192 + e / 16] * (aq[e] * a[e]);
      const float d = orc_fp16_to_fp32(orc_rd16(bw + 208)) * da;
      for (int l = 0; l < 8; ++l) sums[l] += d * (float)lane[l];
    } else {
      int sumi = 0;
      for (int k = 0; k < 8; ++k) {
        int sc, m;
        int16_t b0, b1;
        orc_scale_min_k4(k, bw + 4, &sc, &m);
        memcpy(&b0, ba + 260 + 4 * k, 2);
        memcpy(&b1, ba + 262 + 4 * k, 2);
        sumi += (b0 + b1) * m;
        for (int e = 0; e < 32; ++e) lane[e & 7] += sc * (aq[32 * k + e] * a[32 * k + e]);
      }
      const float d = orc_fp16_to_fp32(orc_rd16(bw)) * da;
      for (int l = 0; l < 8; ++l) sums[l] += d * (float)lane[l];
      const float dmin = orc_fp16_to_fp32(orc_rd16(bw + 2)) * da;
      sum -= dmin * (float)sumi;
    }
  }
  if (kq)
    for (int l = 0; l < 8; ++l) sum += sums[l];
  return sum;
}

static int orc_matmul_q_ext(const uint8_t* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y,
                            int64_t n) {
  const int64_t bb = orc_ext_block_bytes(dtype);
  if (!bb) return -1;
  const int kq = dtype != 7;
  const int64_t be = kq ? 256 : 32, ab = kq ? 292 : 36, nb = ne0 / be;
  uint8_t* xa = (uint8_t*)malloc((size_t)(nb * ab));
  if (!xa) return -1;
  for (int64_t t = 0; t < n; ++t) {
    if (kq) orc_quantize_q8_K(x + t * ne0, xa, ne0);
    else orc_quantize_q8_1(x + t * ne0, xa, ne0);
    for (int64_t r = 0; r < ne1; ++r) y[t * ne1 + r] = orc_dot_ext(dtype, w + r * nb * bb, xa, nb);
  }
  free(xa);
  return 0;
}

float orc_vec_dot(int dtype, const void* w, const void* act, int64_t n_blocks) {
  const int64_t bb = orc_block_bytes(dtype);
  if (bb) return orc_dot_q8_0_family(dtype, (const uint8_t*)w, (const uint8_t*)act, n_blocks, bb);
  if (orc_ext_block_bytes(dtype)) return orc_dot_ext(dtype, (const uint8_t*)w, (const uint8_t*)act, n_blocks);
  return NAN;
}
