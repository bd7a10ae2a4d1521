// Quantized weight matmuls and embedding rows on the GPU for the weight types nibble pairs with Q8_1 or Q8_K
// activations -- Q5_1 and the k-quants Q4_K, Q5_K, Q6_K -- bit-identical to nibble's CPU kernels (src/quant.h:50-99;
// src/quant.cpp:54-146 (k-quant scales, unpacking, dequantization and dots), :206-242 (dequantize_row), :260-307
// (the Q8_1 / Q8_K activation quantizers), :371-418 (the Q5_1 and Q6_K dots)).
//
// Arithmetic kept from the reference, operation by operation (every float operation is an uncontracted _rn
// intrinsic, the file is built with -fmad=false as well):
//  * Q8_1 activations: d = max|x| / 127, q = roundf(x * (1 / d)) clamped to [-127, 127], s = fp16(sum(q) * d) from
//    the unrounded d. Q8_K: iscale = -127 / x_max, x_max the element of largest magnitude (the first on ties),
//    q = round-half-even(iscale * x) clamped, d = 1 / iscale, 16 sums of 16 values.
//  * Q5_1 x Q8_1: per block sum += (d_w * d_a) * sumi + m_w * s_a, in block order.
//  * k-quants x Q8_K: per super-block eight int32 lanes (element e feeds lane e % 8, each product scaled by its
//    sub-block's scale), sums[l] += (d_w * d_a) * lane[l]; Q4_K / Q5_K subtract (dmin_w * d_a) * sum_k(bsum_k * m_k)
//    from the running total per super-block; the eight lane sums are added to the total last, lane 0 first.
// The integer parts are exact in any order, so they are spread over the warp: for a k-quant lane i takes elements
// i + 32 j (j = 0..7, all in accumulator lane i % 8, sub-block j), and lanes i, i^8, i^16, i^24 add up accumulator
// lane i % 8. Every lane then carries the float chain of its accumulator lane (and the min-term chain) through the
// super-blocks in order, and the eight chains are added to the total at the end exactly as the reference does.
// Q5_1 gives each lane one 32-element block (dp4a on the 5-bit values) and adds the block terms to the row's sum
// one block at a time, broadcast from the lane that holds it.
//
// Decode (n <= 8 activation rows) splits the two parts between the warps of a CTA: the integer dots of a CTA's
// (weight row, super-block) items run on all its warps at once into shared memory, then one warp per weight row runs
// the float chains over a chunk of super-blocks in order. More rows run one warp per (weight row, 4 activation rows).
//
// Layouts: a weight stays in its GGUF block layout on the device (ne1 rows of ne0 / block-elements blocks). Q8_1
// activations of n rows are int8 values [n][ne0], scales fp32 [n][blocks] and sums s fp32 [n][blocks]. Q8_K
// activations are stored lane-major, int8 [n][blocks][32 lanes][8] (lane i's bytes are elements i + 32 j), with the
// scales fp32 [n][blocks] and the eight 32-element sub-block sums (bsums[2k] + bsums[2k + 1], the pair the dots use)
// int32 [n][blocks][8].
#include <algorithm>

#include "model_ops.h"
#include "nbl_device.cuh"
#include "quant_common.cuh"

namespace nbl {
namespace {

constexpr int kRowsPerWarp = 4;  // activation rows one warp takes against its weight row
constexpr int kWarps = 8;        // weight rows per CTA
constexpr unsigned kFull = 0xffffffffu;

__host__ __device__ constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

__device__ __forceinline__ float f16_at(const uint8_t* p) {  // p is 2-byte aligned
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}

// ggml's get_scale_min_k4 (src/quant.cpp:54-63): the j-th 6-bit scale and minimum of the 12 packed bytes q.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// ---------------------------------------------------------------- activation quantizers (one warp per block)
// Q8_1: lane i quantizes element i of block `blk`.
__global__ void quantize_q8_1_kernel(const float* __restrict__ x, int64_t blocks, int8_t* __restrict__ qs,
                                     float* __restrict__ d, float* __restrict__ s) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < blocks;
       blk += warps) {
    const float v = x[blk * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
    const bool nan = __any_sync(kFull, v != v);
    const float dd = nan ? __int_as_float(0x7fc00000) : __fdiv_rn(amax, 127.f);
    const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
    const float r = roundf(__fmul_rn(v, id));
    const int q = r != r ? 0 : static_cast<int>(fminf(127.f, fmaxf(-127.f, r)));
    qs[blk * 32 + lane] = static_cast<int8_t>(q);
    int sum = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    if (lane == 0) {
      d[blk] = __half2float(__float2half_rn(dd));
      s[blk] = __half2float(__float2half_rn(__fmul_rn(static_cast<float>(sum), dd)));
    }
  }
}

// Q8_K: lane i quantizes elements i + 32 j (j = 0..7) of 256-element block `blk`.
__global__ void quantize_q8_K_kernel(const float* __restrict__ x, int64_t blocks, uint2* __restrict__ qs,
                                     float* __restrict__ d, int* __restrict__ bsums) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < blocks;
       blk += warps) {
    float v[8];
    float amax = 0.f, mx = 0.f;
    int idx = 256;
    bool nan = false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = x[blk * 256 + lane + 32 * j];
      const float ax = fabsf(v[j]);
      if (ax > amax) {  // NaN never wins, as in the reference's scan
        amax = ax;
        mx = v[j];
        idx = lane + 32 * j;
      }
      nan = nan || v[j] != v[j];
    }
    // largest magnitude, the smallest element index among equal ones: the reference's first maximum
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oa = __shfl_xor_sync(kFull, amax, o);
      const float om = __shfl_xor_sync(kFull, mx, o);
      const int oi = __shfl_xor_sync(kFull, idx, o);
      if (oa > amax || (oa == amax && oi < idx)) {
        amax = oa;
        mx = om;
        idx = oi;
      }
    }
    nan = __any_sync(kFull, nan);
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float dout = 0.f;
    if (amax != 0.f) {
      const float iscale = __fdiv_rn(-127.f, mx);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float w = __fmul_rn(iscale, v[j]);
        q[j] = w != w ? 0 : __float2int_rn(fminf(127.f, fmaxf(-127.f, w)));
      }
      dout = __fdiv_rn(1.f, iscale);
    }
    if (nan) dout = __int_as_float(0x7fc00000);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo |= (static_cast<uint32_t>(q[j]) & 0xFFu) << (8 * j);
      hi |= (static_cast<uint32_t>(q[j + 4]) & 0xFFu) << (8 * j);
    }
    qs[blk * 32 + lane] = make_uint2(lo, hi);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int g = q[j];  // sub-block j: element lane + 32 j of every lane
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) g += __shfl_xor_sync(kFull, g, o);
      if (lane == j) bsums[blk * 8 + j] = g;
    }
    if (lane == 0) d[blk] = dout;
  }
}

// ---------------------------------------------------------------- k-quant block dots
template <int DT>
struct KTraits;
template <>
struct KTraits<NBL_Q4_K> {
  static constexpr int kBytes = 144;
  static constexpr bool kMin = true;
};
template <>
struct KTraits<NBL_Q5_K> {
  static constexpr int kBytes = 176;
  static constexpr bool kMin = true;
};
template <>
struct KTraits<NBL_Q6_K> {
  static constexpr int kBytes = 210;
  static constexpr bool kMin = false;
};

// The values of elements lane + 32 j (j = 0..7) of a super-block and their sub-block scales (sub-block j for Q4_K /
// Q5_K, 16-element sub-block 2 j + lane / 16 for Q6_K).
template <int DT>
__device__ __forceinline__ void decode_k(const uint8_t* blk, int lane, int (&wq)[8], int (&sc)[8]) {
  if constexpr (DT == NBL_Q6_K) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int qh = blk[128 + 32 * h + lane];
      const int ql0 = blk[64 * h + lane], ql1 = blk[64 * h + 32 + lane];
      wq[4 * h + 0] = ((ql0 & 0xF) | ((qh & 3) << 4)) - 32;
      wq[4 * h + 1] = ((ql1 & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
      wq[4 * h + 2] = ((ql0 >> 4) | (((qh >> 4) & 3) << 4)) - 32;
      wq[4 * h + 3] = ((ql1 >> 4) | (((qh >> 6) & 3) << 4)) - 32;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j] = static_cast<int8_t>(blk[192 + 2 * j + (lane >> 4)]);
  } else {
    constexpr int kQs = DT == NBL_Q5_K ? 48 : 16;
    const int qh = DT == NBL_Q5_K ? blk[16 + lane] : 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int byte = blk[kQs + 32 * c + lane];
      wq[2 * c] = (byte & 0xF) + (((qh >> (2 * c)) & 1) << 4);
      wq[2 * c + 1] = (byte >> 4) + (((qh >> (2 * c + 1)) & 1) << 4);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int m;
      scale_min_k4(j, blk + 4, sc[j], m);
    }
  }
}

// This lane's integer share of accumulator lane (lane % 8): sum_j sc[j] * (a * w) over its elements lane + 32 j,
// then the lanes holding the same accumulator lane (lane, lane ^ 8, lane ^ 16, lane ^ 24) added together.
__device__ __forceinline__ int kdot(const uint2 av, const int (&wq)[8], const int (&sc)[8]) {
  int p = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int a = static_cast<int8_t>(((j < 4 ? av.x : av.y) >> (8 * (j & 3))) & 0xFFu);
    p += sc[j] * (a * wq[j]);
  }
  p += __shfl_xor_sync(kFull, p, 8);
  return p + __shfl_xor_sync(kFull, p, 16);
}

// The Q4_K / Q5_K min-term integer of one super-block: sum_k (bsums[2k] + bsums[2k + 1]) * m[k], lane k % 8 taking
// term k and three shuffles adding them (every lane ends with the sum). `sums` points at the block's 8 pair sums.
__device__ __forceinline__ int kmin_sum(const uint8_t* blk, const int* sums, int lane) {
  int sck, mk;
  scale_min_k4(lane & 7, blk + 4, sck, mk);
  int v = sums[lane & 7] * mk;
  v += __shfl_xor_sync(kFull, v, 1);
  v += __shfl_xor_sync(kFull, v, 2);
  return v + __shfl_xor_sync(kFull, v, 4);
}

// One warp per (weight row, up to kRowsPerWarp activation rows); CTAs of kWarps weight rows.
template <int DT>
__global__ void __launch_bounds__(kWarps * 32) kquant_matmul_kernel(
    const uint8_t* __restrict__ w, int64_t ne1, int nb, const uint2* __restrict__ aqs, const float* __restrict__ ad,
    const int* __restrict__ asum, float* __restrict__ y, int64_t n) {
  using Tr = KTraits<DT>;
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (r >= ne1) return;  // the whole warp leaves together
  const uint8_t* wrow = w + r * nb * Tr::kBytes;
  for (int64_t t0 = static_cast<int64_t>(blockIdx.y) * kRowsPerWarp; t0 < n;
       t0 += static_cast<int64_t>(gridDim.y) * kRowsPerWarp) {
    const int nt = n - t0 < kRowsPerWarp ? static_cast<int>(n - t0) : kRowsPerWarp;
    float sums[kRowsPerWarp], tot[kRowsPerWarp];
#pragma unroll
    for (int tt = 0; tt < kRowsPerWarp; ++tt) sums[tt] = tot[tt] = 0.f;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* blk = wrow + static_cast<int64_t>(b) * Tr::kBytes;
      int wq[8], sc[8];
      decode_k<DT>(blk, lane, wq, sc);
      const float dw = f16_at(blk + (DT == NBL_Q6_K ? 208 : 0));
      const float dminw = Tr::kMin ? f16_at(blk + 2) : 0.f;
#pragma unroll
      for (int tt = 0; tt < kRowsPerWarp; ++tt) {
        if (tt < nt) {
          const int64_t t = t0 + tt;
          const int p = kdot(aqs[(t * nb + b) * 32 + lane], wq, sc);  // accumulator lane (lane % 8)
          const float da = ad[t * nb + b];
          sums[tt] = __fadd_rn(sums[tt], __fmul_rn(__fmul_rn(dw, da), static_cast<float>(p)));
          if constexpr (Tr::kMin) {
            const int sumi = kmin_sum(blk, asum + (t * nb + b) * 8, lane);
            tot[tt] = __fsub_rn(tot[tt], __fmul_rn(__fmul_rn(dminw, da), static_cast<float>(sumi)));
          }
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < kRowsPerWarp; ++tt) {
      if (tt < nt) {
        float res = tot[tt];
#pragma unroll
        for (int l = 0; l < 8; ++l) res = __fadd_rn(res, __shfl_sync(kFull, sums[tt], l));
        if (lane == 0) y[(t0 + tt) * ne1 + r] = res;
      }
    }
  }
}

// Decode: CTAs of kWarps warps over `rows_per_cta` weight rows and all n <= kGemvMaxRows activation rows. Per chunk
// of up to kChunk super-blocks, phase 1 spreads the (row, super-block) items over the warps and leaves each item's
// eight accumulator-lane dots and min-term integer in shared memory; phase 2 has warp r carry row r's float chains
// (lanes 0-7 the accumulator lanes, lane 8 the min-term total; one per activation row) through the chunk in order.
constexpr int kChunk = 16;
template <int DT>
__global__ void __launch_bounds__(kWarps * 32) kquant_gemv_kernel(
    const uint8_t* __restrict__ w, int64_t ne1, int nb, const uint2* __restrict__ aqs, const float* __restrict__ ad,
    const int* __restrict__ asum, float* __restrict__ y, int n, int rows_per_cta) {
  using Tr = KTraits<DT>;
  extern __shared__ int part[];  // [n][rows_per_cta][kChunk][9]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int rows = ne1 - r0 < rows_per_cta ? static_cast<int>(ne1 - r0) : rows_per_cta;
  float st[kGemvMaxRows];
#pragma unroll
  for (int t = 0; t < kGemvMaxRows; ++t) st[t] = 0.f;
  for (int b0 = 0; b0 < nb; b0 += kChunk) {
    const int cb = nb - b0 < kChunk ? nb - b0 : kChunk;
    for (int it = warp; it < rows * cb; it += kWarps) {
      const int r = it / cb, bb = it - r * cb;
      const int64_t b = b0 + bb;
      const uint8_t* blk = w + ((r0 + r) * nb + b) * Tr::kBytes;
      int wq[8], sc[8];
      decode_k<DT>(blk, lane, wq, sc);
      for (int t = 0; t < n; ++t) {
        const int p = kdot(aqs[(static_cast<int64_t>(t) * nb + b) * 32 + lane], wq, sc);
        int* slot = part + ((t * rows_per_cta + r) * kChunk + bb) * 9;
        if (lane < 8) slot[lane] = p;
        if constexpr (Tr::kMin) {
          const int sumi = kmin_sum(blk, asum + (static_cast<int64_t>(t) * nb + b) * 8, lane);
          if (lane == 8) slot[8] = sumi;
        }
      }
    }
    __syncthreads();
    if (warp < rows && lane < (Tr::kMin ? 9 : 8)) {
      const uint8_t* wrow = w + (r0 + warp) * nb * Tr::kBytes;
#pragma unroll
      for (int t = 0; t < kGemvMaxRows; ++t) {
        if (t < n) {
          for (int bb = 0; bb < cb; ++bb) {
            const uint8_t* blk = wrow + static_cast<int64_t>(b0 + bb) * Tr::kBytes;
            const float da = ad[static_cast<int64_t>(t) * nb + b0 + bb];
            const float v = static_cast<float>(part[((t * rows_per_cta + warp) * kChunk + bb) * 9 + lane]);
            if (lane < 8)
              st[t] = __fadd_rn(st[t], __fmul_rn(__fmul_rn(f16_at(blk + (DT == NBL_Q6_K ? 208 : 0)), da), v));
            else
              st[t] = __fsub_rn(st[t], __fmul_rn(__fmul_rn(f16_at(blk + 2), da), v));
          }
        }
      }
    }
    __syncthreads();
  }
  if (warp < rows) {
#pragma unroll
    for (int t = 0; t < kGemvMaxRows; ++t) {
      if (t < n) {
        float res = Tr::kMin ? __shfl_sync(kFull, st[t], 8) : 0.f;
#pragma unroll
        for (int l = 0; l < 8; ++l) res = __fadd_rn(res, __shfl_sync(kFull, st[t], l));
        if (lane == 0) y[static_cast<int64_t>(t) * ne1 + r0 + warp] = res;
      }
    }
  }
}

// ---------------------------------------------------------------- Q5_1 block dots
__global__ void __launch_bounds__(kWarps * 32) q5_1_matmul_kernel(
    const uint8_t* __restrict__ w, int64_t ne1, int nb, const int8_t* __restrict__ aqs, const float* __restrict__ ad,
    const float* __restrict__ as, float* __restrict__ y, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (r >= ne1) return;
  const int64_t ne0 = static_cast<int64_t>(nb) * 32;
  const uint8_t* wrow = w + r * nb * 24;
  for (int64_t t0 = static_cast<int64_t>(blockIdx.y) * kRowsPerWarp; t0 < n;
       t0 += static_cast<int64_t>(gridDim.y) * kRowsPerWarp) {
    const int nt = n - t0 < kRowsPerWarp ? static_cast<int>(n - t0) : kRowsPerWarp;
    float tot[kRowsPerWarp];
#pragma unroll
    for (int tt = 0; tt < kRowsPerWarp; ++tt) tot[tt] = 0.f;
    for (int b0 = 0; b0 < nb; b0 += 32) {
      const int b = b0 + lane, in_row = nb - b0 < 32 ? nb - b0 : 32;
      int lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
      float dw = 0.f, mw = 0.f;
      if (b < nb) {
        const uint8_t* blk = wrow + static_cast<int64_t>(b) * 24;
        dw = f16_at(blk);
        mw = f16_at(blk + 2);
        const uint32_t qh = *reinterpret_cast<const uint32_t*>(blk + 4);
        const uint2 q0 = *reinterpret_cast<const uint2*>(blk + 8), q1 = *reinterpret_cast<const uint2*>(blk + 16);
        unpack_nibbles(make_uint4(q0.x, q0.y, q1.x, q1.y), lo, hi);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo[i] |= high_bits4(qh, 4 * i);
          hi[i] |= high_bits4(qh, 16 + 4 * i);
        }
      }
#pragma unroll
      for (int tt = 0; tt < kRowsPerWarp; ++tt) {
        if (tt < nt) {
          const int64_t t = t0 + tt;
          float term = 0.f;
          if (b < nb) {
            const int4* a = reinterpret_cast<const int4*>(aqs + t * ne0 + static_cast<int64_t>(b) * 32);
            const int4 a0 = a[0], a1 = a[1];
            int s = __dp4a(lo[0], a0.x, 0);
            s = __dp4a(lo[1], a0.y, s);
            s = __dp4a(lo[2], a0.z, s);
            s = __dp4a(lo[3], a0.w, s);
            s = __dp4a(hi[0], a1.x, s);
            s = __dp4a(hi[1], a1.y, s);
            s = __dp4a(hi[2], a1.z, s);
            s = __dp4a(hi[3], a1.w, s);
            const float da = ad[t * nb + b], sa = as[t * nb + b];
            term = __fadd_rn(__fmul_rn(__fmul_rn(dw, da), static_cast<float>(s)), __fmul_rn(mw, sa));
          }
          for (int u = 0; u < in_row; ++u) tot[tt] = __fadd_rn(tot[tt], __shfl_sync(kFull, term, u));
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < kRowsPerWarp; ++tt)
      if (tt < nt && lane == 0) y[(t0 + tt) * ne1 + r] = tot[tt];
  }
}

// ---------------------------------------------------------------- embedding rows (dequantize_row)
// One thread per output element; the reference's per-element float operations (src/quant.cpp:98-115, :206-242).
template <int DT>
__global__ void embed_qblock_kernel(const uint8_t* __restrict__ table, int64_t ne0, const int32_t* __restrict__ ids,
                                    int64_t n, float* __restrict__ out) {
  constexpr int kElems = DT == NBL_Q5_1 ? 32 : 256;
  constexpr int kBytes = DT == NBL_Q5_1 ? 24 : DT == NBL_Q4_K ? 144 : DT == NBL_Q5_K ? 176 : 210;
  const int64_t total = n * ne0, nb = ne0 / kElems;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / ne0, e = idx - t * ne0;
    const uint8_t* blk = table + (static_cast<int64_t>(ids[t]) * nb + e / kElems) * kBytes;
    const int i = static_cast<int>(e % kElems);
    float v;
    if constexpr (DT == NBL_Q5_1) {
      const int j = i & 15, byte = blk[8 + j];
      const uint32_t qh = *reinterpret_cast<const uint32_t*>(blk + 4);
      const int q = i < 16 ? (byte & 0x0F) | (((qh >> j) << 4) & 0x10) : (byte >> 4) | ((qh >> (j + 12)) & 0x10);
      v = __fadd_rn(__fmul_rn(static_cast<float>(q), f16_at(blk)), f16_at(blk + 2));
    } else if constexpr (DT == NBL_Q6_K) {
      const int h = i >> 7, g = (i >> 5) & 3, l = i & 31;
      const int ql = blk[64 * h + 32 * (g & 1) + l], qh = blk[128 + 32 * h + l];
      const int q = ((g < 2 ? ql & 0xF : ql >> 4) | (((qh >> (2 * g)) & 3) << 4)) - 32;
      const float dk = __fmul_rn(f16_at(blk + 208), static_cast<float>(static_cast<int8_t>(blk[192 + (i >> 4)])));
      v = __fmul_rn(dk, static_cast<float>(q));
    } else {
      const int k = i >> 5, l = i & 31;
      const int byte = blk[(DT == NBL_Q5_K ? 48 : 16) + 32 * (k >> 1) + l];
      int q = (k & 1) ? byte >> 4 : byte & 0xF;
      if constexpr (DT == NBL_Q5_K) q += ((blk[16 + l] >> k) & 1) << 4;
      int sc, m;
      scale_min_k4(k, blk + 4, sc, m);
      const float d1 = __fmul_rn(f16_at(blk), static_cast<float>(sc));
      const float m1 = __fmul_rn(f16_at(blk + 2), static_cast<float>(m));
      v = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
    out[idx] = v;
  }
}

}  // namespace

bool is_qblock(int32_t dtype) {
  return dtype == NBL_Q5_1 || dtype == NBL_Q4_K || dtype == NBL_Q5_K || dtype == NBL_Q6_K;
}

int64_t qblock_elems(int32_t dtype) { return dtype == NBL_Q5_1 ? 32 : 256; }

int64_t qblock_bytes(int32_t dtype) {
  return dtype == NBL_Q5_1 ? 24 : dtype == NBL_Q4_K ? 144 : dtype == NBL_Q5_K ? 176 : dtype == NBL_Q6_K ? 210 : 0;
}

size_t qblock_act_bytes(int32_t dtype, int64_t n, int64_t ne0) {
  const int64_t nb = ne0 / qblock_elems(dtype);
  return align256(static_cast<size_t>(n * ne0)) + align256(static_cast<size_t>(n * nb) * sizeof(float)) +
         static_cast<size_t>(n * nb) * (dtype == NBL_Q5_1 ? sizeof(float) : 8 * sizeof(int));
}

void launch_qblock_matmul(cudaStream_t st, const Weight& w, float* y, const float* x, int64_t n, void* act,
                          int num_sms) {
  const int64_t nb = w.ne0 / qblock_elems(w.dtype), blocks = n * nb;
  auto* base = static_cast<uint8_t*>(act);
  auto* d = reinterpret_cast<float*>(base + align256(static_cast<size_t>(n * w.ne0)));
  void* extra = reinterpret_cast<uint8_t*>(d) + align256(static_cast<size_t>(blocks) * sizeof(float));
  const unsigned qgrid =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((blocks + 7) / 8, int64_t(num_sms) * 16)));
  const auto* wb = static_cast<const uint8_t*>(w.dev);
  const int inb = static_cast<int>(nb);
  if (w.dtype == NBL_Q5_1) {
    auto* qs = reinterpret_cast<int8_t*>(base);
    quantize_q8_1_kernel<<<qgrid, 256, 0, st>>>(x, blocks, qs, d, static_cast<float*>(extra));
    const dim3 grid(static_cast<unsigned>((w.ne1 + kWarps - 1) / kWarps),
                    static_cast<unsigned>(std::min<int64_t>((n + kRowsPerWarp - 1) / kRowsPerWarp, 65535)));
    q5_1_matmul_kernel<<<grid, kWarps * 32, 0, st>>>(wb, w.ne1, inb, qs, d, static_cast<const float*>(extra), y, n);
    return;
  }
  auto* qs = reinterpret_cast<uint2*>(base);
  const auto* sums = static_cast<const int*>(extra);
  quantize_q8_K_kernel<<<qgrid, 256, 0, st>>>(x, blocks, qs, d, static_cast<int*>(extra));
  if (n <= kGemvMaxRows) {
    // weight rows per CTA: the most of 8, 4, 2 that still gives every SM four CTAs, else 1
    int per = 8;
    while (per > 1 && (w.ne1 + per - 1) / per < 4LL * num_sms) per >>= 1;
    const unsigned grid = static_cast<unsigned>((w.ne1 + per - 1) / per);
    const size_t smem = static_cast<size_t>(n) * per * kChunk * 9 * sizeof(int);
    const int in = static_cast<int>(n);
    switch (w.dtype) {
      case NBL_Q4_K:
        kquant_gemv_kernel<NBL_Q4_K><<<grid, kWarps * 32, smem, st>>>(wb, w.ne1, inb, qs, d, sums, y, in, per);
        break;
      case NBL_Q5_K:
        kquant_gemv_kernel<NBL_Q5_K><<<grid, kWarps * 32, smem, st>>>(wb, w.ne1, inb, qs, d, sums, y, in, per);
        break;
      default:
        kquant_gemv_kernel<NBL_Q6_K><<<grid, kWarps * 32, smem, st>>>(wb, w.ne1, inb, qs, d, sums, y, in, per);
        break;
    }
    return;
  }
  const dim3 grid(static_cast<unsigned>((w.ne1 + kWarps - 1) / kWarps),
                  static_cast<unsigned>(std::min<int64_t>((n + kRowsPerWarp - 1) / kRowsPerWarp, 65535)));
  switch (w.dtype) {
    case NBL_Q4_K: kquant_matmul_kernel<NBL_Q4_K><<<grid, kWarps * 32, 0, st>>>(wb, w.ne1, inb, qs, d, sums, y, n); break;
    case NBL_Q5_K: kquant_matmul_kernel<NBL_Q5_K><<<grid, kWarps * 32, 0, st>>>(wb, w.ne1, inb, qs, d, sums, y, n); break;
    default: kquant_matmul_kernel<NBL_Q6_K><<<grid, kWarps * 32, 0, st>>>(wb, w.ne1, inb, qs, d, sums, y, n); break;
  }
}

void launch_embed_qblock(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out,
                         int num_sms) {
  const int64_t total = n * table.ne0;
  const unsigned grid =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, int64_t(num_sms) * 8)));
  const auto* tb = static_cast<const uint8_t*>(table.dev);
  switch (table.dtype) {
    case NBL_Q5_1: embed_qblock_kernel<NBL_Q5_1><<<grid, 256, 0, st>>>(tb, table.ne0, ids, n, out); break;
    case NBL_Q4_K: embed_qblock_kernel<NBL_Q4_K><<<grid, 256, 0, st>>>(tb, table.ne0, ids, n, out); break;
    case NBL_Q5_K: embed_qblock_kernel<NBL_Q5_K><<<grid, 256, 0, st>>>(tb, table.ne0, ids, n, out); break;
    default: embed_qblock_kernel<NBL_Q6_K><<<grid, 256, 0, st>>>(tb, table.ne0, ids, n, out); break;
  }
}

}  // namespace nbl
