// Elementwise kernels of the attention path: bias add, in-place fp32 RoPE (Backend::rope), and the fused
// bias -> RoPE -> narrowing -> paged K/V append that replaces the reference's cache-row writes.
//
// Rotation arithmetic follows nibble's cpu::rope (src/backend/cpu/ref_ops.cpp:166-185): cos/sin come from a
// table the host evaluates in double exactly as the reference does, and a' = a*c - b*s, b' = a*s + b*c are
// computed as separately rounded float products and sums (no FMA contraction), so the result is bit-identical.
#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

__device__ __forceinline__ void rotate(float a, float b, float2 cs, float& ra, float& rb) {
  ra = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
  rb = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
}

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
// resolved once; an out-of-range row/position/page id flags the error word and skips the K/V write.
template <int IN, int QOUT, int KV>
__global__ void rope_kv_append_kernel(const void* __restrict__ q_in, const void* __restrict__ k_in,
                                      const void* __restrict__ v_in, const float* __restrict__ bq,
                                      const float* __restrict__ bk, const float* __restrict__ bv, void* q_out,
                                      const int32_t* __restrict__ tok_row, const int32_t* __restrict__ tok_pos,
                                      const int32_t* __restrict__ page_table, int32_t pt_stride, int n_heads,
                                      int n_kv_heads, int head_dim, int page_size, int64_t n_pages, bool neox,
                                      const float2* __restrict__ tab, int64_t tab_pos, void* pool, int* err) {
  const int64_t r = blockIdx.x;
  const int half = head_dim / 2;
  const int32_t pos = tok_pos[r];
  const int32_t row = tok_row[r];
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

int grid_for(int64_t total, int threads) {
  const int64_t g = (total + threads - 1) / threads;
  return static_cast<int>(g < 1 ? 1 : (g > 1048576 ? 1048576 : g));
}

template <int IN, int QOUT>
void dispatch_kv(cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                 const float* bq, const float* bk, const float* bv, void* q_out, const int32_t* tok_row,
                 const int32_t* tok_pos, const int32_t* page_table, int32_t pt_stride, int64_t n_tok, int n_heads,
                 bool neox, const float2* tab, int64_t tab_pos, int* err) {
  const auto& c = kv->cfg;
  const dim3 grid(static_cast<unsigned>(n_tok)), block(128);
  if (c.dtype == NBL_F16)
    rope_kv_append_kernel<IN, QOUT, NBL_F16><<<grid, block, 0, st>>>(
        q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table, pt_stride, n_heads, c.n_kv_heads,
        c.head_dim, c.page_size, c.n_pages, neox, tab, tab_pos, kv->pool, err);
  else
    rope_kv_append_kernel<IN, QOUT, NBL_BF16><<<grid, block, 0, st>>>(
        q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table, pt_stride, n_heads, c.n_kv_heads,
        c.head_dim, c.page_size, c.n_pages, neox, tab, tab_pos, kv->pool, err);
}

template <int IN>
void dispatch_qout(int q_out_dtype, cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in,
                   const void* v_in, const float* bq, const float* bk, const float* bv, void* q_out,
                   const int32_t* tok_row, const int32_t* tok_pos, const int32_t* page_table, int32_t pt_stride,
                   int64_t n_tok, int n_heads, bool neox, const float2* tab, int64_t tab_pos, int* err) {
  switch (q_out_dtype) {
    case NBL_F32:
      return dispatch_kv<IN, NBL_F32>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                      pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
    case NBL_F16:
      return dispatch_kv<IN, NBL_F16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                      pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
    default:
      return dispatch_kv<IN, NBL_BF16>(st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                                       pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
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
                           const float2* tab, int64_t tab_pos, int* err) {
  switch (in_dtype) {
    case NBL_F32:
      dispatch_qout<NBL_F32>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                             pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
      break;
    case NBL_F16:
      dispatch_qout<NBL_F16>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos, page_table,
                             pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
      break;
    default:
      dispatch_qout<NBL_BF16>(q_out_dtype, st, kv, q_in, k_in, v_in, bq, bk, bv, q_out, tok_row, tok_pos,
                              page_table, pt_stride, n_tok, n_heads, neox, tab, tab_pos, err);
  }
  check_cuda(cudaGetLastError(), "rope_kv_append launch");
}

}  // namespace nbl
