// Backend::attention on fp32 device buffers with the reference's layout and semantics (src/backend/backend.h:66-69,
// CpuBackend::attention src/backend/cpu/cpu_backend.cpp:272-290): q,out [n, n_heads, head_dim], k,v
// [n_ctx, n_kv_heads, head_dim]; query row t (position pos0+t) attends keys 0..pos0+t; query head h reads KV
// head h / (n_heads / n_kv_heads).
//
// This is the drop-in path for a Transformer that keeps nibble's flat fp32 caches; the paged fp16/bf16 kernels
// (decode.cu, prefill.cu) are the fast paths. Prefill chunks (16 rows or more, head_dim 64 or 128) run the
// query-tiled kernel below; otherwise one CTA per (row, head); its warps take the row's keys in chunks of
// 32 (warp w: chunks w, w + W, ...). A warp stages its chunk of K and V in shared memory with coalesced 16-byte
// loads (K rows padded by one float, so lane i reading key i is conflict-free), each lane scores one key, an online
// softmax keeps (m, l, o) per warp, and the chunk's p_j * v_j is accumulated with lanes over head dimensions. The
// warps' states are merged at the end. Scores are q.k * (1/sqrtf(head_dim)) accumulated over d in
// order like the reference; exp is expf; sums are fp32 (the reference sums the softmax denominator in double), so
// results agree to ~1e-6 relative.
#include <atomic>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

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

// Shared memory: q [head_dim], per warp a K chunk [32][head_dim + 1], a V chunk [32][head_dim] and its final
// (m, l, o[head_dim]).
__host__ __device__ constexpr size_t attn_smem_floats(int warps, int head_dim) {
  return size_t(head_dim) + size_t(warps) * (32 * (2 * head_dim + 1) + head_dim + 2);
}

// Copies `cnt` rows of head_dim floats (global row stride `stride`) into shared rows of stride ld, with 16-byte loads
// when every row start is 16-byte aligned and head_dim % 4 == 0.
__device__ __forceinline__ void stage_rows(float* dst, int ld, const float* src, int64_t stride, int cnt,
                                           int head_dim, bool vec, int lane) {
  if (vec) {
    const int q4 = head_dim / 4;
    for (int e = lane; e < cnt * q4; e += 32) {
      const int row = e / q4, c = e - row * q4;
      const float4 x = __ldg(reinterpret_cast<const float4*>(src + row * stride) + c);
      float* o = dst + row * ld + 4 * c;
      o[0] = x.x, o[1] = x.y, o[2] = x.z, o[3] = x.w;
    }
  } else {
    for (int e = lane; e < cnt * head_dim; e += 32) {
      const int row = e / head_dim, d = e - row * head_dim;
      dst[row * ld + d] = __ldg(src + row * stride + d);
    }
  }
}

template <int W>
__global__ void __launch_bounds__(W * 32) attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, float* __restrict__ out,
                                                               int64_t n, int64_t pos0, int64_t n_heads,
                                                               int64_t n_kv_heads, int head_dim, float scale,
                                                               bool vec) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t idx = blockIdx.x;  // (row t, head h)
  const int64_t t = idx / n_heads, h = idx % n_heads;
  const int64_t kvh = h / (n_heads / n_kv_heads);
  const int ldk = head_dim + 1;
  float* q_s = smem;
  float* k_s = smem + head_dim + size_t(warp) * 32 * (2 * head_dim + 1);
  float* v_s = k_s + 32 * ldk;
  float* st = smem + head_dim + size_t(W) * 32 * (2 * head_dim + 1);  // per warp: m, l, o[head_dim]
  for (int d = threadIdx.x; d < head_dim; d += W * 32) q_s[d] = q[idx * head_dim + d];
  __syncthreads();

  const int64_t len = pos0 + t + 1;
  const int64_t kv_stride = n_kv_heads * head_dim;
  const float* kbase = k + kvh * head_dim;
  const float* vbase = v + kvh * head_dim;
  float m = -INFINITY, l = 0.f;
  float o[kMaxDimPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) o[i] = 0.f;

  for (int64_t j0 = int64_t(warp) * 32; j0 < len; j0 += W * 32) {
    const int cnt = static_cast<int>(len - j0 < 32 ? len - j0 : 32);
    stage_rows(k_s, ldk, kbase + j0 * kv_stride, kv_stride, cnt, head_dim, vec, lane);
    stage_rows(v_s, head_dim, vbase + j0 * kv_stride, kv_stride, cnt, head_dim, vec, lane);
    __syncwarp();
    float s = -INFINITY;
    if (lane < cnt) {
      const float* kr = k_s + lane * ldk;  // row stride head_dim + 1: lanes hit distinct banks
      float dot = 0.f;
      for (int d = 0; d < head_dim; ++d) dot = fmaf(q_s[d], kr[d], dot);
      s = dot * scale;
    }
    const float m_new = fmaxf(m, warp_max(s));  // finite: lane 0's key is always valid
    const float alpha = expf(m - m_new);
    const float p = lane < cnt ? expf(s - m_new) : 0.f;
    l = l * alpha + p;
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) o[i] *= alpha;
#pragma unroll 4
    for (int jj = 0; jj < cnt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const float* vj = v_s + jj * head_dim;
#pragma unroll
      for (int i = 0; i < kMaxDimPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < head_dim) o[i] = fmaf(pj, vj[d], o[i]);
      }
    }
    m = m_new;
    __syncwarp();  // the chunk buffers are reused by the next chunk
  }
  // merge the warps: M = max m_w, out = sum_w o_w e^(m_w - M) / sum_w l_w e^(m_w - M)
  float* my = st + size_t(warp) * (head_dim + 2);
  const float lw = warp_sum(l);
  if (lane == 0) {
    my[0] = m;
    my[1] = lw;
  }
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < head_dim) my[2 + d] = o[i];
  }
  __syncthreads();
  float big = -INFINITY;
#pragma unroll
  for (int w = 0; w < W; ++w) big = fmaxf(big, st[size_t(w) * (head_dim + 2)]);
  float den = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const float mw = st[size_t(w) * (head_dim + 2)];
    if (mw != -INFINITY) den += st[size_t(w) * (head_dim + 2) + 1] * expf(mw - big);
  }
  const float inv = 1.f / den;
  for (int d = threadIdx.x; d < head_dim; d += W * 32) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float mw = st[size_t(w) * (head_dim + 2)];
      if (mw != -INFINITY) acc += st[size_t(w) * (head_dim + 2) + 2 + d] * expf(mw - big);
    }
    out[idx * head_dim + d] = acc * inv;
  }
}

// ---------------------------------------------------------------- query tiles (prefill chunks)
// A CTA takes 64 query rows of one head (and, when there are more tiles than SMs, then the mirror tile from the end
// of the chunk, so that every CTA has about the same causal work) and walks their keys in chunks of 64 staged in shared memory, so each K/V
// row is read once per 64 queries instead of once per query. Thread (ty, tx) (16 x 16) owns query rows ty + 16 i and,
// for the scores, key columns tx + 16 j (i, j < 4): each score is the same in-order fmaf chain over d as above, built
// from 16-byte shared loads (K rows padded to head_dim + 4 floats, so eight lanes reading eight rows miss no bank).
// The online softmax of a row reduces over the 16 lanes that hold it; p goes to shared memory and the thread
// accumulates o for its rows over head-dim columns 4 tx + 64 c with 16-byte loads of V.
constexpr int kTileQ = 64, kTileK = 64, kTileThreads = 256;

template <int D>
__host__ __device__ constexpr size_t tiled_smem_floats() {
  return size_t(kTileQ) * (D + 4) + size_t(kTileK) * (D + 4) + size_t(kTileK) * D + size_t(kTileQ) * (kTileK + 4);
}

template <int D>
__global__ void __launch_bounds__(kTileThreads) attention_f32_tiled_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ out,
    int64_t n, int64_t pos0, int64_t n_heads, int64_t n_kv_heads, float scale, bool paired) {
  constexpr int LD = D + 4, LP = kTileK + 4, C4 = D / 64;  // C4: float4 column groups of o per thread
  extern __shared__ __align__(16) float tsm[];
  float* qs = tsm;                    // [64][LD]
  float* ks = qs + kTileQ * LD;       // [64][LD]
  float* vs = ks + kTileK * LD;       // [64][D]
  float* ps = vs + kTileK * D;        // [64][LP]
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t h = blockIdx.y, kvh = h / (n_heads / n_kv_heads);
  const int64_t q_stride = n_heads * D, kv_stride = n_kv_heads * D;
  // tiles x and n_tiles - 1 - x: under the causal mask their key counts add up to the same total for every CTA
  const int64_t n_tiles = (n + kTileQ - 1) / kTileQ;
  for (int which = 0; which < 2; ++which) {
    const int64_t tile = which == 0 ? int64_t(blockIdx.x) : n_tiles - 1 - int64_t(blockIdx.x);
    if (which == 1 && (!paired || tile <= int64_t(blockIdx.x))) break;
    const int64_t q0 = tile * kTileQ;
    __syncthreads();  // the previous tile's shared data is no longer read
    // the query tile (rows past n read as zero and are never written)
    for (int e = tid; e < kTileQ * D / 4; e += kTileThreads) {
      const int r = e / (D / 4), c = e - r * (D / 4);
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q0 + r < n) x = __ldg(reinterpret_cast<const float4*>(q + (q0 + r) * q_stride + h * D) + c);
      *reinterpret_cast<float4*>(qs + r * LD + 4 * c) = x;
    }
    float m[4], l[4], o[4][C4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.f;
#pragma unroll
      for (int c = 0; c < C4; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[i][c][e] = 0.f;
    }
    const int64_t last = (q0 + kTileQ < n ? q0 + kTileQ : n) - 1;
    const int64_t keys = pos0 + last + 1;  // the tile's longest causal range
    for (int64_t j0 = 0; j0 < keys; j0 += kTileK) {
      __syncthreads();  // the previous chunk's K, V and p are no longer read
      for (int e = tid; e < kTileK * D / 4; e += kTileThreads) {
        const int r = e / (D / 4), c = e - r * (D / 4);
        float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
        if (j0 + r < keys) {
          kx = __ldg(reinterpret_cast<const float4*>(k + (j0 + r) * kv_stride + kvh * D) + c);
          vx = __ldg(reinterpret_cast<const float4*>(v + (j0 + r) * kv_stride + kvh * D) + c);
        }
        *reinterpret_cast<float4*>(ks + r * LD + 4 * c) = kx;
        *reinterpret_cast<float4*>(vs + r * D + 4 * c) = vx;
      }
      __syncthreads();
      float sc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
      for (int d = 0; d < D; d += 4) {
        float4 qa[4], kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(qs + (ty + 16 * i) * LD + d);
#pragma unroll
        for (int j = 0; j < 4; ++j) kb[j] = *reinterpret_cast<const float4*>(ks + (tx + 16 * j) * LD + d);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sc[i][j] = fmaf(qa[i].x, kb[j].x, sc[i][j]);
            sc[i][j] = fmaf(qa[i].y, kb[j].y, sc[i][j]);
            sc[i][j] = fmaf(qa[i].z, kb[j].z, sc[i][j]);
            sc[i][j] = fmaf(qa[i].w, kb[j].w, sc[i][j]);
          }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t qpos = pos0 + q0 + ty + 16 * i;  // keys 0..qpos
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t key = j0 + tx + 16 * j;
          sc[i][j] = key <= qpos ? sc[i][j] * scale : -INFINITY;
          mx = fmaxf(mx, sc[i][j]);
        }
#pragma unroll
        for (int off = 8; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float m_new = fmaxf(m[i], mx);  // finite: key 0 lies in every row's first chunk
        const float alpha = expf(m[i] - m_new);
        float rs = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float p = sc[i][j] == -INFINITY ? 0.f : expf(sc[i][j] - m_new);
          ps[(ty + 16 * i) * LP + tx + 16 * j] = p;
          rs += p;
        }
#pragma unroll
        for (int off = 8; off; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
        l[i] = l[i] * alpha + rs;
        m[i] = m_new;
#pragma unroll
        for (int c = 0; c < C4; ++c)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[i][c][e] *= alpha;
      }
      __syncthreads();
      const int jn = keys - j0 < kTileK ? static_cast<int>(keys - j0) : kTileK;
#pragma unroll 4
      for (int j = 0; j < jn; ++j) {
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pr[i] = ps[(ty + 16 * i) * LP + j];
#pragma unroll
        for (int c = 0; c < C4; ++c) {
          const float4 vv = *reinterpret_cast<const float4*>(vs + j * D + 64 * c + 4 * tx);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            o[i][c][0] = fmaf(pr[i], vv.x, o[i][c][0]);
            o[i][c][1] = fmaf(pr[i], vv.y, o[i][c][1]);
            o[i][c][2] = fmaf(pr[i], vv.z, o[i][c][2]);
            o[i][c][3] = fmaf(pr[i], vv.w, o[i][c][3]);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = q0 + ty + 16 * i;
      if (row < n) {
        const float inv = 1.f / l[i];
#pragma unroll
        for (int c = 0; c < C4; ++c) {
          const float4 y = make_float4(o[i][c][0] * inv, o[i][c][1] * inv, o[i][c][2] * inv, o[i][c][3] * inv);
          *reinterpret_cast<float4*>(out + row * q_stride + h * D + 64 * c + 4 * tx) = y;
        }
      }
    }
  }
}

template <int D>
void launch_tiled(cudaStream_t st, const float* q, const float* k, const float* v, float* out, int64_t n,
                  int64_t pos0, int64_t n_heads, int64_t n_kv_heads, float scale, int num_sms) {
  const size_t smem = tiled_smem_floats<D>() * sizeof(float);
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(attention_f32_tiled_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)),
               "attention smem attribute");
    configured.fetch_or(bit);
  }
  // pairs of tiles per CTA only when one tile per CTA would be more CTAs than SMs (otherwise the pairs idle SMs)
  const int64_t n_tiles = (n + kTileQ - 1) / kTileQ;
  const bool paired = n_tiles * n_heads > num_sms;
  const dim3 grid(static_cast<unsigned>(paired ? (n_tiles + 1) / 2 : n_tiles), static_cast<unsigned>(n_heads));
  attention_f32_tiled_kernel<D><<<grid, kTileThreads, smem, st>>>(q, k, v, out, n, pos0, n_heads, n_kv_heads, scale,
                                                                   paired);
}

// The widest head each warp count is launched for (shared memory stays under ~140 KB).
template <int W>
constexpr int max_dim_for() { return W == 8 ? 64 : W == 4 ? 128 : 256; }

template <int W>
void launch_w(cudaStream_t st, const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
              int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float scale) {
  const size_t smem = attn_smem_floats(W, static_cast<int>(head_dim)) * sizeof(float);
  static std::atomic<uint64_t> configured{0};  // the attribute is per device: set it once on each
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(attention_f32_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(attn_smem_floats(W, max_dim_for<W>()) * sizeof(float))),
               "attention smem attribute");
    configured.fetch_or(bit);
  }
  const bool vec = head_dim % 4 == 0 && ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
  attention_f32_kernel<W><<<static_cast<unsigned>(n * n_heads), W * 32, smem, st>>>(
      q, k, v, out, n, pos0, n_heads, n_kv_heads, static_cast<int>(head_dim), scale, vec);
}

}  // namespace

void launch_attention_f32(cudaStream_t st, const float* q, const float* k, const float* v, float* out, int64_t n,
                          int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float scale,
                          int num_sms) {
  if (n * n_heads > 0x7fffffff) fail(NBL_E_INVALID, "attention: n * n_heads too large");
  // Prefill chunks with head_dim 64 or 128 and 16-byte-aligned rows: 64-query tiles.
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  if (n >= 16 && aligned && n_heads <= 65535 && (head_dim == 64 || head_dim == 128)) {
    if (head_dim == 64) launch_tiled<64>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, scale, num_sms);
    else launch_tiled<128>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, scale, num_sms);
    check_cuda(cudaGetLastError(), "attention launch");
    return;
  }
  // Many (row, head) CTAs (prefill chunks): 2 warps each, small enough that several CTAs share an SM. Few (decode):
  // as many warps as their K/V chunks fit in shared memory -- 8 up to head_dim 64, 4 up to 128, 2 up to 256.
  if (n * n_heads >= 4 * int64_t(num_sms))
    launch_w<2>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scale);
  else if (head_dim <= max_dim_for<8>()) launch_w<8>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scale);
  else if (head_dim <= max_dim_for<4>()) launch_w<4>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scale);
  else launch_w<2>(st, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scale);
  check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace nbl
