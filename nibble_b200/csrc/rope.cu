// Elementwise kernels of the attention path: bias add, in-place fp32 RoPE (Backend::rope), and the fused
// bias -> RoPE -> narrowing -> paged K/V append that replaces the reference's cache-row writes.
//
// Rotation arithmetic follows nibble's cpu::rope (src/backend/cpu/ref_ops.cpp:166-185): cos/sin come from a
// table the host evaluates in double exactly as the reference does, and a' = a*c - b*s, b' = a*s + b*c are
// computed as separately rounded float products and sums (no FMA contraction), so the result is bit-identical.
#include <algorithm>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

__device__ __forceinline__ void rotate(float a, float b, float2 cs, float& ra, float& rb) { rope_rotate(a, b, cs, ra, rb); }

// Pair i of a head_dim-wide head: element offsets of its two members (NeoX: i, i+half; else 2i, 2i+1).
__device__ __forceinline__ void pair_index(int i, int half, bool neox, int& ia, int& ib) {
  ia = neox ? i : 2 * i;
  ib = neox ? i + half : 2 * i + 1;
}

__global__ void add_bias_kernel(float* __restrict__ x, const float* __restrict__ bias, int64_t width, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x)
    x[i] = __fadd_rn(x[i], bias[i % width]);
}

// One thread per (row, head, pair).
__global__ void rope_f32_kernel(float* __restrict__ x, int64_t n, int64_t n_heads, int half, int64_t pos0, bool neox,
                                const float2* __restrict__ tab, int* err) {
  const int64_t total = n * n_heads * half;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % half);
    const int64_t rh = idx / half;  // row * n_heads + head
    const int64_t t = rh / n_heads;
    float* v = x + rh * 2 * half;
    int ia, ib;
    pair_index(i, half, neox, ia, ib);
    const float2 cs = tab[(pos0 + t) * half + i];
    float ra, rb;
    rotate(v[ia], v[ib], cs, ra, rb);
    v[ia] = ra;
    v[ib] = rb;
  }
}

template <int DT>
__device__ __forceinline__ float load_as_float(const void* p, int64_t i) {
  if constexpr (DT == NBL_F32) return static_cast<const float*>(p)[i];
  else if constexpr (DT == NBL_F16) return __half2float(static_cast<const __half*>(p)[i]);
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
template <int DT>
__device__ __forceinline__ void store_from_float(void* p, int64_t i, float v) {
  if constexpr (DT == NBL_F32) static_cast<float*>(p)[i] = v;
  else if constexpr (DT == NBL_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// One CTA per token. Threads walk the token's q pairs, k pairs and v elements. The token's page slot is
// resolved once; an out-of-range row/position/page id flags the error word and skips the K/V write. With
// tok_row/tok_pos NULL the tokens are one new token per row: token t is row row_base + t at position
// lens[row] - 1 (a decode step whose lengths already count the new token).
template <int IN, int QOUT, int KV>
__global__ void rope_kv_append_kernel(const void* __restrict__ q_in, const void* __restrict__ k_in,
                                      const void* __restrict__ v_in, const float* __restrict__ bq,
                                      const float* __restrict__ bk, const float* __restrict__ bv, void* q_out,
                                      const int32_t* __restrict__ tok_row, const int32_t* __restrict__ tok_pos,
                                      const int32_t* __restrict__ page_table, int32_t pt_stride, int n_heads,
                                      int n_kv_heads, int head_dim, int page_size, int64_t n_pages, bool neox,
                                      const float2* __restrict__ tab, int64_t tab_pos, void* pool, int* err,
                                      int32_t row_base, const int32_t* __restrict__ lens) {
  const int64_t r = blockIdx.x;
  const int half = head_dim / 2;
  const int32_t row = tok_row ? tok_row[r] : row_base + static_cast<int32_t>(r);
  const int32_t pos = tok_pos ? tok_pos[r] : lens[row] - 1;
  bool pos_ok = pos >= 0 && pos < tab_pos;
  int64_t page = -1;
  if (pos_ok && pos / page_size < pt_stride && row >= 0) {
    page = page_table[int64_t(row) * pt_stride + pos / page_size];
    if (page < 0 || page >= n_pages) {
      if (threadIdx.x == 0) flag_error(err, kErrPageId);
      page = -1;
    }
  } else if (threadIdx.x == 0) {
    flag_error(err, kErrLength);
  }
  if (!pos_ok) return;
  const float2* cs_row = tab + int64_t(pos) * half;
  const int slot = pos % page_size;
  const int64_t block = int64_t(n_kv_heads) * page_size * head_dim;  // elements of one K (or V) half-page

  // q: rope(q_in + bq) -> q_out
  const int nq = n_heads * half;
  for (int idx = threadIdx.x; idx < nq; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    int ia, ib;
    pair_index(i, half, neox, ia, ib);
    const int64_t base = (r * n_heads + h) * head_dim;
    float a = load_as_float<IN>(q_in, base + ia), b = load_as_float<IN>(q_in, base + ib);
    if (bq) {
      a = __fadd_rn(a, bq[h * head_dim + ia]);
      b = __fadd_rn(b, bq[h * head_dim + ib]);
    }
    float ra, rb;
    rotate(a, b, cs_row[i], ra, rb);
    store_from_float<QOUT>(q_out, base + ia, ra);
    store_from_float<QOUT>(q_out, base + ib, rb);
  }
  if (page < 0) return;
  // k: rope(k_in + bk) -> page K half
  const int nk = n_kv_heads * half;
  for (int idx = threadIdx.x; idx < nk; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    int ia, ib;
    pair_index(i, half, neox, ia, ib);
    const int64_t base = (r * n_kv_heads + h) * head_dim;
    float a = load_as_float<IN>(k_in, base + ia), b = load_as_float<IN>(k_in, base + ib);
    if (bk) {
      a = __fadd_rn(a, bk[h * head_dim + ia]);
      b = __fadd_rn(b, bk[h * head_dim + ib]);
    }
    float ra, rb;
    rotate(a, b, cs_row[i], ra, rb);
    const int64_t dst = page * 2 * block + (int64_t(h) * page_size + slot) * head_dim;
    store_from_float<KV>(pool, dst + ia, ra);
    store_from_float<KV>(pool, dst + ib, rb);
  }
  // v: v_in + bv -> page V half
  const int nv = n_kv_heads * head_dim;
  for (int idx = threadIdx.x; idx < nv; idx += blockDim.x) {
    const int h = idx / head_dim, d = idx % head_dim;
    float a = load_as_float<IN>(v_in, r * nv + idx);
    if (bv) a = __fadd_rn(a, bv[idx]);
    const int64_t dst = page * 2 * block + block + (int64_t(h) * page_size + slot) * head_dim + d;
    store_from_float<KV>(pool, dst, a);
  }
}

// Four consecutive elements as floats (16-bit types: one 8-byte load; fp32: one 16-byte load). The caller
// guarantees the alignment (vector path only).
template <int DT>
__device__ __forceinline__ void load4(const void* p, int64_t i, float (&v)[4]) {
  if constexpr (DT == NBL_F32) {
    const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  } else {
    const uint2 x = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i);
    const uint32_t w[2] = {x.x, x.y};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if constexpr (DT == NBL_F16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        v[2 * k] = f.x, v[2 * k + 1] = f.y;
      } else {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
        v[2 * k] = f.x, v[2 * k + 1] = f.y;
      }
    }
  }
}
template <int DT>
__device__ __forceinline__ void store4(void* p, int64_t i, const float (&v)[4]) {
  if constexpr (DT == NBL_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if constexpr (DT == NBL_F16) {
        const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p) + i) = make_uint2(w[0], w[1]);
  }
}

// Eight consecutive elements as floats (16-bit types: one 16-byte load; fp32: two).
template <int DT>
__device__ __forceinline__ void load8(const void* p, int64_t i, float (&lo)[4], float (&hi)[4]) {
  if constexpr (DT == NBL_F32) {
    load4<DT>(p, i, lo);
    load4<DT>(p, i + 4, hi);
  } else {
    const uint4 x = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f;
      if constexpr (DT == NBL_F16) f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
      float* dst = k < 2 ? lo : hi;
      dst[2 * (k & 1)] = f.x, dst[2 * (k & 1) + 1] = f.y;
    }
  }
}
template <int DT>
__device__ __forceinline__ void store8(void* p, int64_t i, const float (&lo)[4], const float (&hi)[4]) {
  if constexpr (DT == NBL_F32) {
    store4<DT>(p, i, lo);
    store4<DT>(p, i + 4, hi);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float* src = k < 2 ? lo : hi;
      const float a = src[2 * (k & 1)], b = src[2 * (k & 1) + 1];
      if constexpr (DT == NBL_F16) {
        const __half2 h = __floats2half2_rn(a, b);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        w[k] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Vector form of rope_kv_append_kernel for head_dim % 8 == 0 and 16-byte-aligned rows. Warps walk the tokens
// (grid-stride, kTokGroup tokens at a time whose position, row and page slot are resolved in one round of loads);
// for each token lane l takes 8-element chunks l, l+32, ... of its q heads, K heads and V heads in that order, so
// the warp reads and writes consecutive 16-byte pieces of each row. A chunk holds four rotation pairs: elements
// 8c..8c+7 (interleaved pairs) or 4c..4c+3 with their partners half+4c..half+4c+3 (NeoX). Checks, error flags and
// the NULL tok_row/tok_pos form are those of the scalar kernel; the per-pair arithmetic is identical, so are the
// results.
// Chunks per lane whose loads are issued together. One measured fastest on B200 (config-3 prefill append,
// 3.7 GB: 0.75 ms with 1, 0.96 ms with 2, 1.5 ms with 4): the registers a second chunk costs lower occupancy more
// than its extra load in flight gains.
constexpr int kInFlight = 1;
constexpr int kTokGroup = 8;  // most tokens whose metadata one warp resolves at once (<= 32)

template <int IN, int QOUT, int KV, bool NEOX>
__global__ void __launch_bounds__(256) rope_kv_append_vec_kernel(
    const void* __restrict__ q_in, const void* __restrict__ k_in, const void* __restrict__ v_in,
    const float* __restrict__ bq, const float* __restrict__ bk, const float* __restrict__ bv, void* q_out,
    const int32_t* __restrict__ tok_row, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ page_table,
    int32_t pt_stride, int n_heads, int n_kv_heads, int head_dim, int page_size, int64_t n_pages,
    const float2* __restrict__ tab, int64_t tab_pos, void* pool, int* err, int64_t n_tok, int32_t row_base,
    const int32_t* __restrict__ lens, int tok_group) {
  const int lane = threadIdx.x & 31;
  const int half = head_dim / 2;
  const int chunks = head_dim / 8;
  const int q_units = n_heads * chunks, k_units = n_kv_heads * chunks;
  const int units = q_units + 2 * k_units;
  const int64_t block = int64_t(n_kv_heads) * page_size * head_dim;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  // Tokens are taken tok_group (1..kTokGroup) at a time per warp: lane i < tok_group resolves token t0 + i
  // (position check, page lookup, error flags) in one round of loads, then the warp walks the group reading the
  // results by shuffle. Few tokens run one per warp, so a small launch spreads over as many warps as it has tokens.
  for (int64_t t0 = (blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5)) * tok_group; t0 < n_tok;
       t0 += warps * tok_group) {
    int32_t my_pos = -1;
    int64_t my_page = -1;
    if (lane < tok_group && t0 + lane < n_tok) {
      const int64_t t = t0 + lane;
      const int32_t row = tok_row ? tok_row[t] : row_base + static_cast<int32_t>(t);
      my_pos = tok_pos ? tok_pos[t] : lens[row] - 1;
      if (my_pos >= 0 && my_pos < tab_pos) {
        if (my_pos / page_size < pt_stride && row >= 0) {
          my_page = page_table[int64_t(row) * pt_stride + my_pos / page_size];
          if (my_page < 0 || my_page >= n_pages) {
            flag_error(err, kErrPageId);
            my_page = -1;
          }
        } else {
          flag_error(err, kErrLength);
        }
      } else {
        flag_error(err, kErrLength);
        my_pos = -1;  // skipped entirely
      }
    }
    const int n_here = static_cast<int>(std::min<int64_t>(tok_group, n_tok - t0));
#pragma unroll 1
    for (int ti = 0; ti < n_here; ++ti) {
      const int64_t r = t0 + ti;
      const int32_t pos = __shfl_sync(0xffffffffu, my_pos, ti);
      const int64_t page = __shfl_sync(0xffffffffu, my_page, ti);
      if (pos < 0) continue;
      const int slot = pos % page_size;
      const int u_end = page >= 0 ? units : q_units;  // no page: q only
      const float2* cs_row = tab + int64_t(pos) * half;
      const int64_t k_dst = page * 2 * block + int64_t(slot) * head_dim;  // + h * page_size * head_dim
#pragma unroll 1
      for (int u0 = lane; u0 < u_end; u0 += 32 * kInFlight) {
        float x[kInFlight][8];
        int kind[kInFlight], h[kInFlight], c[kInFlight];
#pragma unroll
        for (int i = 0; i < kInFlight; ++i) {  // issue every chunk's loads first
          const int u = u0 + 32 * i;
          kind[i] = u >= u_end ? -1 : (u < q_units ? 0 : (u < q_units + k_units ? 1 : 2));
          const int uu = kind[i] <= 0 ? u : (kind[i] == 1 ? u - q_units : u - q_units - k_units);
          h[i] = uu / chunks;
          c[i] = uu - h[i] * chunks;
          if (kind[i] < 0) continue;
          const void* src = kind[i] == 0 ? q_in : (kind[i] == 1 ? k_in : v_in);
          const int64_t base = (r * (kind[i] == 0 ? n_heads : n_kv_heads) + h[i]) * head_dim;
          float(&lo)[4] = *reinterpret_cast<float(*)[4]>(&x[i][0]);
          float(&hi)[4] = *reinterpret_cast<float(*)[4]>(&x[i][4]);
          if (NEOX && kind[i] < 2) {
            load4<IN>(src, base + 4 * c[i], lo);
            load4<IN>(src, base + half + 4 * c[i], hi);
          } else {
            load8<IN>(src, base + 8 * c[i], lo, hi);
          }
        }
#pragma unroll
        for (int i = 0; i < kInFlight; ++i) {
          if (kind[i] < 0) continue;
          const int ea = NEOX && kind[i] < 2 ? 4 * c[i] : 8 * c[i];
          const int eb = NEOX && kind[i] < 2 ? half + 4 * c[i] : 8 * c[i] + 4;
          const float* bias = kind[i] == 0 ? bq : (kind[i] == 1 ? bk : bv);
          float(&lo)[4] = *reinterpret_cast<float(*)[4]>(&x[i][0]);
          float(&hi)[4] = *reinterpret_cast<float(*)[4]>(&x[i][4]);
          if (bias) {
            const float4 ba = *reinterpret_cast<const float4*>(bias + h[i] * head_dim + ea);
            const float4 bb = *reinterpret_cast<const float4*>(bias + h[i] * head_dim + eb);
            lo[0] = __fadd_rn(lo[0], ba.x), lo[1] = __fadd_rn(lo[1], ba.y);
            lo[2] = __fadd_rn(lo[2], ba.z), lo[3] = __fadd_rn(lo[3], ba.w);
            hi[0] = __fadd_rn(hi[0], bb.x), hi[1] = __fadd_rn(hi[1], bb.y);
            hi[2] = __fadd_rn(hi[2], bb.z), hi[3] = __fadd_rn(hi[3], bb.w);
          }
          float ya[4], yb[4];
          if (kind[i] == 2) {  // V: no rotation
#pragma unroll
            for (int k = 0; k < 4; ++k) ya[k] = lo[k], yb[k] = hi[k];
          } else {
            // pairs 4c..4c+3: two 16-byte loads (the row starts at pos * half float2, half even)
            const float4 cs01 = *reinterpret_cast<const float4*>(cs_row + 4 * c[i]);
            const float4 cs23 = *reinterpret_cast<const float4*>(cs_row + 4 * c[i] + 2);
            const float2 cs[4] = {make_float2(cs01.x, cs01.y), make_float2(cs01.z, cs01.w), make_float2(cs23.x, cs23.y),
                                  make_float2(cs23.z, cs23.w)};
            if (NEOX) {  // pair 4c+k = (lo[k], hi[k])
#pragma unroll
              for (int k = 0; k < 4; ++k) rotate(lo[k], hi[k], cs[k], ya[k], yb[k]);
            } else {  // adjacent pairs
              rotate(lo[0], lo[1], cs[0], ya[0], ya[1]);
              rotate(lo[2], lo[3], cs[1], ya[2], ya[3]);
              rotate(hi[0], hi[1], cs[2], yb[0], yb[1]);
              rotate(hi[2], hi[3], cs[3], yb[2], yb[3]);
            }
          }
          if (kind[i] == 0) {
            const int64_t base = (r * n_heads + h[i]) * head_dim;
            if (NEOX) {
              store4<QOUT>(q_out, base + ea, ya);
              store4<QOUT>(q_out, base + eb, yb);
            } else {
              store8<QOUT>(q_out, base + ea, ya, yb);
            }
          } else {
            const int64_t dst = k_dst + (kind[i] == 2 ? block : 0) + int64_t(h[i]) * page_size * head_dim;
            if (NEOX && kind[i] == 1) {
              store4<KV>(pool, dst + ea, ya);
              store4<KV>(pool, dst + eb, yb);
            } else {
              store8<KV>(pool, dst + ea, ya, yb);
            }
          }
        }
      }
    }
  }
}

int grid_for(int64_t total, int threads) {
  const int64_t g = (total + threads - 1) / threads;
  return static_cast<int>(g < 1 ? 1 : (g > 1048576 ? 1048576 : g));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Resident CTAs of the vector kernel over the whole GPU, queried once per instance (one GPU type per process).
template <int IN, int QOUT, int KV, bool NEOX>
int64_t vec_resident() {
  static const int64_t r = [] {
    int dev = 0, sms = 148, per_sm = 1;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rope_kv_append_vec_kernel<IN, QOUT, KV, NEOX>,
                                                             256, 0),
               "occupancy");
    return int64_t(sms) * std::max(per_sm, 1);
  }();
  return r;
}

template <int IN, int QOUT, int KV>
void launch_kv(cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
               const float* bq, const float* bk, const float* bv, void* q_out, const int32_t* tok_row,
               const int32_t* tok_pos, const int32_t* page_table, int32_t pt_stride, int64_t n_tok, int n_heads,
               bool neox, const float2* tab, int64_t tab_pos, int* err, int32_t row_base, const int32_t* lens) {
  const auto& c = kv->cfg;
  // vector path: whole 8-element chunks, 16-byte aligned rows and bias (every row offset is a multiple of
  // head_dim elements, so aligned bases keep every chunk aligned)
  const bool vec = c.head_dim % 8 == 0 && aligned16(q_in) && aligned16(k_in) && aligned16(v_in) &&
                   aligned16(q_out) && aligned16(kv->pool) && (!bq || aligned16(bq)) && (!bk || aligned16(bk)) &&
                   (!bv || aligned16(bv));
  if (vec) {
    auto k = neox ? rope_kv_append_vec_kernel<IN, QOUT, KV, true> : rope_kv_append_vec_kernel<IN, QOUT, KV, false>;
    // 8 warps per CTA; one wave of resident CTAs walks all tokens, each warp tok_group tokens at a time (as few
    // as the resident warps allow, at most kTokGroup)
    const int64_t cap = neox ? vec_resident<IN, QOUT, KV, true>() : vec_resident<IN, QOUT, KV, false>();
    const int tok_group = static_cast<int>(std::min<int64_t>(kTokGroup, std::max<int64_t>(1, (n_tok + 8 * cap - 1) / (8 * cap))));
    const int64_t want = (n_tok + 8 * tok_group - 1) / (8 * tok_group);
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
    k<<<grid, 256, 0, st>>>(q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table, pt_stride, n_heads,
                            c.n_kv_heads, c.head_dim, c.page_size, c.n_pages, tab, tab_pos, kv->pool, err, n_tok,
                            row_base, lens, tok_group);
    return;
  }
  rope_kv_append_kernel<IN, QOUT, KV><<<dim3(static_cast<unsigned>(n_tok)), dim3(128), 0, st>>>(
      q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table, pt_stride, n_heads, c.n_kv_heads,
      c.head_dim, c.page_size, c.n_pages, neox, tab, tab_pos, kv->pool, err, row_base, lens);
}

template <int IN, int QOUT>
void dispatch_kv(cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                 const float* bq, const float* bk, const float* bv, void* q_out, const int32_t* tok_row,
                 const int32_t* tok_pos, const int32_t* page_table, int32_t pt_stride, int64_t n_tok, int n_heads,
                 bool neox, const float2* tab, int64_t tab_pos, int* err, int32_t row_base, const int32_t* lens) {
  if (kv->cfg.dtype == NBL_F16)
    launch_kv<IN, QOUT, NBL_F16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                 pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
  else
    launch_kv<IN, QOUT, NBL_BF16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                  pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
}

template <int IN>
void dispatch_qout(int q_out_dtype, cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in,
                   const void* v_in, const float* bq, const float* bk, const float* bv, void* q_out,
                   const int32_t* tok_row, const int32_t* tok_pos, const int32_t* page_table, int32_t pt_stride,
                   int64_t n_tok, int n_heads, bool neox, const float2* tab, int64_t tab_pos, int* err,
                   int32_t row_base, const int32_t* lens) {
  switch (q_out_dtype) {
    case NBL_F32:
      return dispatch_kv<IN, NBL_F32>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                      pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
    case NBL_F16:
      return dispatch_kv<IN, NBL_F16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                      pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
    default:
      return dispatch_kv<IN, NBL_BF16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                       pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
  }
}

}  // namespace

void launch_add_bias(cudaStream_t st, float* x, const float* bias, int64_t width, int64_t n) {
  const int64_t total = width * n;
  add_bias_kernel<<<grid_for(total, 256), 256, 0, st>>>(x, bias, width, total);
  check_cuda(cudaGetLastError(), "add_bias launch");
}

void launch_rope_f32(cudaStream_t st, float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0,
                     bool neox, const float2* tab, int* err) {
  const int64_t total = n * n_heads * (head_dim / 2);
  rope_f32_kernel<<<grid_for(total, 256), 256, 0, st>>>(x, n, n_heads, static_cast<int>(head_dim / 2), pos0, neox,
                                                         tab, err);
  check_cuda(cudaGetLastError(), "rope launch");
}

void launch_rope_kv_append(cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                           int in_dtype, const float* bq, const float* bk, const float* bv, void* q_out,
                           int q_out_dtype, const int32_t* tok_row, const int32_t* tok_pos,
                           const int32_t* page_table, int32_t pt_stride, int64_t n_tok, int n_heads, bool neox,
                           const float2* tab, int64_t tab_pos, int* err, int32_t row_base, const int32_t* lens) {
  switch (in_dtype) {
    case NBL_F32:
      dispatch_qout<NBL_F32>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                             pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
      break;
    case NBL_F16:
      dispatch_qout<NBL_F16>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                             pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
      break;
    default:
      dispatch_qout<NBL_BF16>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos,
                              page_table, pt_stride, n_tok, n_heads, neox, tab, tab_pos, err, row_base, lens);
  }
  check_cuda(cudaGetLastError(), "rope_kv_append launch");
}

}  // namespace nbl
