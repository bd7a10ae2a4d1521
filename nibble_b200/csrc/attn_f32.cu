// Backend::attention on fp32 device buffers with the reference's layout and semantics (src/backend/backend.h:66-69,
// CpuBackend::attention src/backend/cpu/cpu_backend.cpp:272-290): q,out [n, n_heads, head_dim], k,v
// [n_ctx, n_kv_heads, head_dim]; query row t (position pos0+t) attends keys 0..pos0+t; query head h reads KV
// head h / (n_heads / n_kv_heads).
//
// This is the drop-in path for a Transformer that keeps nibble's flat fp32 caches; the paged fp16/bf16 kernels
// (decode.cu, prefill.cu) are the fast paths. One warp per (row, head): keys in chunks of 32 (one per lane)
// with an online softmax, then the chunk's p_j * v_j accumulated with lanes over head dimensions. Scores are
// q.k * (1/sqrtf(head_dim)) like the reference; exp is expf; sums are fp32 (the reference sums the softmax
// denominator in double), so results agree to ~1e-6 relative.
#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxDimPerLane = 8;  // head_dim <= 256

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kWarps * 32) attention_f32_kernel(const float* __restrict__ q,
                                                                    const float* __restrict__ k,
                                                                    const float* __restrict__ v,
                                                                    float* __restrict__ out, int64_t n, int64_t pos0,
                                                                    int64_t n_heads, int64_t n_kv_heads, int head_dim,
                                                                    float scale) {
  extern __shared__ float q_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t idx = int64_t(blockIdx.x) * kWarps + warp;
  if (idx >= n * n_heads) return;
  const int64_t t = idx / n_heads, h = idx % n_heads;
  const int64_t kvh = h / (n_heads / n_kv_heads);
  float* qw = q_smem + warp * head_dim;
  for (int d = lane; d < head_dim; d += 32) qw[d] = q[idx * head_dim + d];
  __syncwarp();

  const int64_t len = pos0 + t + 1;
  const int64_t kv_stride = n_kv_heads * head_dim;
  const float* kbase = k + kvh * head_dim;
  const float* vbase = v + kvh * head_dim;
  float m = -INFINITY, l = 0.f;
  float o[kMaxDimPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) o[i] = 0.f;

  for (int64_t j0 = 0; j0 < len; j0 += 32) {
    const int64_t j = j0 + lane;
    float s = -INFINITY;
    if (j < len) {
      const float* kj = kbase + j * kv_stride;
      float dot = 0.f;
      if ((head_dim & 1) == 0) {  // rows start on 8-byte boundaries: paired loads
        const float2* k2 = reinterpret_cast<const float2*>(kj);
        const float2* q2 = reinterpret_cast<const float2*>(qw);
        for (int d = 0; d < head_dim / 2; ++d) {
          const float2 kk = k2[d], qq = q2[d];
          dot = fmaf(qq.x, kk.x, dot);
          dot = fmaf(qq.y, kk.y, dot);
        }
      } else {
        for (int d = 0; d < head_dim; ++d) dot = fmaf(qw[d], kj[d], dot);
      }
      s = dot * scale;
    }
    const float m_new = fmaxf(m, warp_max(s));  // finite: lane 0's key is always valid
    const float alpha = expf(m - m_new);
    const float p = (j < len) ? expf(s - m_new) : 0.f;
    l = l * alpha + p;
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) o[i] *= alpha;
    const int cnt = static_cast<int>(len - j0 < 32 ? len - j0 : 32);
    for (int jj = 0; jj < cnt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const float* vj = vbase + (j0 + jj) * kv_stride;
#pragma unroll
      for (int i = 0; i < kMaxDimPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < head_dim) o[i] = fmaf(pj, vj[d], o[i]);
      }
    }
    m = m_new;
  }
  const float inv = 1.f / warp_sum(l);
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < head_dim) out[idx * head_dim + d] = o[i] * inv;
  }
}

}  // namespace

void launch_attention_f32(cudaStream_t st, const float* q, const float* k, const float* v, float* out, int64_t n,
                          int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float scale) {
  const int64_t pairs = n * n_heads;
  const int64_t blocks = (pairs + kWarps - 1) / kWarps;
  if (blocks > 0x7fffffff) fail(NBL_E_INVALID, "attention: n * n_heads too large");
  const size_t smem = size_t(kWarps) * head_dim * sizeof(float);
  attention_f32_kernel<<<static_cast<unsigned>(blocks), kWarps * 32, smem, st>>>(
      q, k, v, out, n, pos0, n_heads, n_kv_heads, static_cast<int>(head_dim), scale);
  check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace nbl
