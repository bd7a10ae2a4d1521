// Quantized weight matmuls and embedding rows on the GPU, bit-identical to nibble's CPU kernels for the weight types
// whose activations are Q8_0 blocks: Q4_0, Q5_0 and Q8_0 (src/quant.h:1-20, src/quant.cpp:37-51 (activation
// quantizer), :158-205 (dequantize_row), :310-366 (block dots)).
//
// The reference never dequantizes a weight for a matmul: it quantizes each activation row to Q8_0 blocks (d =
// max|x| / 127 rounded to fp16, q = roundf(x / d)), takes the integer dot of each weight block with the activation
// block, turns it into a float term with the two fp16 scales (the operation order differs per type and is kept
// exactly: Q4_0 sumi * d_w * d_a, Q8_0 sumi * (d_w * d_a), Q5_0 (d_w * d_a) * sumi), and adds the terms to the row's
// sum in block order. Here the activation quantizer runs one warp per block, the integer dots run four products per
// dp4a instruction, every float operation is an uncontracted _rn intrinsic, and one row's terms are added in block
// order (lanes hold consecutive blocks; their terms are broadcast to the whole warp one block at a time), so every
// output equals the CPU's bit for bit.
//
// Device layouts (made at upload, nbl_weight_create): the GGUF blocks of a row are split into aligned arrays --
// fp16 scale bits [rows][blocks], the value bytes [rows][blocks][16 or 32] (16-byte aligned per block) and, for
// Q5_0, the 32 high bits [rows][blocks] -- so a lane reads its block with one or two 16-byte loads. Activations are
// quantized into int8 values [n][ne0] and the fp32 value of each block's fp16-rounded scale [n][ne0 / 32].
#include <algorithm>

#include "model_ops.h"
#include "nbl_device.cuh"

namespace nbl {
namespace {

// ---------------------------------------------------------------- activations to Q8_0
// One warp per 32-element block: amax by a max reduction (fmaxf skips NaN like std::fmax; a NaN anywhere makes d
// NaN), d = amax / 127, q = roundf(x * (1 / d)) clamped to [-127, 127] (NaN -> 0); the scale is kept as the fp32
// value of its fp16 rounding, which is what the dot products read.
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int8_t* __restrict__ qs, float* __restrict__ d,
                                     int64_t n_blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (b >= n_blocks) return;
  const float v = x[b * 32 + lane];
  float amax = fabsf(v);
  bool nan = v != v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  nan = __any_sync(0xffffffffu, nan);
  const float dd = nan ? __int_as_float(0x7fc00000) : __fdiv_rn(amax, 127.f);
  const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
  const float r = roundf(__fmul_rn(v, id));
  qs[b * 32 + lane] = static_cast<int8_t>(r != r ? 0 : static_cast<int>(fminf(127.f, fmaxf(-127.f, r))));
  if (lane == 0) d[b] = __half2float(__float2half_rn(dd));
}

// ---------------------------------------------------------------- block dots
// The 4-bit / 5-bit value bytes of a Q4_0 / Q5_0 block widened to the int8 values dp4a takes, in element order:
// lo[i] holds elements 4i..4i+3 (low nibbles of bytes 4i..4i+3), hi[i] elements 16+4i..16+4i+3.
__device__ __forceinline__ void unpack_nibbles(const uint4 q, int (&lo)[4], int (&hi)[4]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo[i] = static_cast<int>(w[i] & 0x0F0F0F0Fu);
    hi[i] = static_cast<int>((w[i] >> 4) & 0x0F0F0F0Fu);
  }
}

// Spreads bits [first, first + 4) of qh to bit 4 of four bytes (the fifth bit of four Q5_0 elements).
__device__ __forceinline__ int high_bits4(uint32_t qh, int first) {
  const uint32_t b = qh >> first;
  return static_cast<int>(((b & 1u) << 4) | ((b & 2u) << 11) | ((b & 4u) << 18) | ((b & 8u) << 25));
}

template <int T>
struct QTraits;
template <>
struct QTraits<NBL_Q4_0> {
  static constexpr int kQsBytes = 16;
};
template <>
struct QTraits<NBL_Q5_0> {
  static constexpr int kQsBytes = 16;
};
template <>
struct QTraits<NBL_Q8_0> {
  static constexpr int kQsBytes = 32;
};

// The float term of one block for activation row a (values av[8] as int8x4 words, scale da).
template <int T>
__device__ __forceinline__ float block_term(const uint8_t* wq, uint32_t qh, float dw, const int (&av)[8], float da) {
  if constexpr (T == NBL_Q8_0) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(wq), w1 = *reinterpret_cast<const uint4*>(wq + 16);
    const int wv[8] = {int(w0.x), int(w0.y), int(w0.z), int(w0.w), int(w1.x), int(w1.y), int(w1.z), int(w1.w)};
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __dp4a(wv[i], av[i], s);
    return __fmul_rn(static_cast<float>(s), __fmul_rn(dw, da));  // sumi * (d_w * d_a)
  } else {
    int lo[4], hi[4];
    unpack_nibbles(*reinterpret_cast<const uint4*>(wq), lo, hi);
    int s = 0;
    if constexpr (T == NBL_Q4_0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s = __dp4a(static_cast<int>(__vsub4(lo[i], 0x08080808)), av[i], s);
        s = __dp4a(static_cast<int>(__vsub4(hi[i], 0x08080808)), av[4 + i], s);
      }
      return __fmul_rn(__fmul_rn(static_cast<float>(s), dw), da);  // sumi * d_w * d_a
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s = __dp4a(static_cast<int>(__vsub4(lo[i] | high_bits4(qh, 4 * i), 0x10101010)), av[i], s);
        s = __dp4a(static_cast<int>(__vsub4(hi[i] | high_bits4(qh, 16 + 4 * i), 0x10101010)), av[4 + i], s);
      }
      return __fmul_rn(__fmul_rn(dw, da), static_cast<float>(s));  // (d_w * d_a) * sumi
    }
  }
}

constexpr int kQThreads = 128;

// y_j[t][r] over up to kMaxMulti weights of type T sharing the quantized activations (rows numbered
// consecutively, as in the float GEMV). One warp per weight row with a grid stride; lane l takes blocks l, l + 32, ...
// For each round of 32 blocks the lanes' terms are added to the row's sum in block order.
template <int T, int NT>
__global__ void __launch_bounds__(kQThreads) gemv_q_kernel(const QBatch b, const int8_t* __restrict__ aq,
                                                           const float* __restrict__ ad, int64_t ne0) {
  constexpr int kQs = QTraits<T>::kQsBytes;
  const int lane = threadIdx.x & 31;
  const int64_t nb = ne0 / 32;
  int64_t total = b.row_end[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < b.count) total = b.row_end[i];
  const int64_t n_warps = int64_t(gridDim.x) * (kQThreads / 32);
  for (int64_t r = int64_t(blockIdx.x) * (kQThreads / 32) + (threadIdx.x >> 5); r < total; r += n_warps) {
    // this row's weight j (a static scan of the parameter block)
    QWeightView w = b.w[0];
    float* y = b.y[0];
    int64_t begin = 0, rows_j = b.row_end[0];
    bool found = r < b.row_end[0];
#pragma unroll
    for (int i = 1; i < kMaxMulti; ++i)
      if (i < b.count && !found && r < b.row_end[i]) {
        found = true;
        w = b.w[i];
        y = b.y[i];
        begin = b.row_end[i - 1];
        rows_j = b.row_end[i] - b.row_end[i - 1];
      }
    const int64_t lr = r - begin;
    float sum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) sum[t] = 0.f;
    for (int64_t k0 = 0; k0 < nb; k0 += 32) {
      const int64_t blk = k0 + lane;
      float term[NT];
      if (blk < nb) {
        const int64_t wb = lr * nb + blk;
        const float dw = __half2float(__ushort_as_half(w.d[wb]));
        const uint32_t qh = T == NBL_Q5_0 ? w.qh[wb] : 0u;
        const uint8_t* wq = w.qs + wb * kQs;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint4 a0 = *reinterpret_cast<const uint4*>(aq + t * ne0 + blk * 32);
          const uint4 a1 = *reinterpret_cast<const uint4*>(aq + t * ne0 + blk * 32 + 16);
          const int av[8] = {int(a0.x), int(a0.y), int(a0.z), int(a0.w), int(a1.x), int(a1.y), int(a1.z), int(a1.w)};
          term[t] = block_term<T>(wq, qh, dw, av, ad[t * nb + blk]);
        }
      } else {
#pragma unroll
        for (int t = 0; t < NT; ++t) term[t] = 0.f;
      }
      const int cnt = nb - k0 < 32 ? static_cast<int>(nb - k0) : 32;
      for (int j = 0; j < cnt; ++j)
#pragma unroll
        for (int t = 0; t < NT; ++t) sum[t] = __fadd_rn(sum[t], __shfl_sync(0xffffffffu, term[t], j));
    }
    if (lane == 0)
#pragma unroll
      for (int t = 0; t < NT; ++t) y[t * rows_j + lr] = sum[t];
  }
}

// ---------------------------------------------------------------- embedding rows
// out[t][k] = dequantized element k of row ids[t]: (value - offset) * d as one float product (src/quant.cpp:169-205).
template <int T>
__global__ void embed_q_kernel(const QWeightView w, const int32_t* __restrict__ ids, float* __restrict__ out,
                               int64_t ne0) {
  constexpr int kQs = QTraits<T>::kQsBytes;
  const int64_t t = blockIdx.y;
  const int64_t nb = ne0 / 32;
  const int64_t row = ids[t];
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < ne0; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t blk = e / 32, j = e % 32, wb = row * nb + blk;
    const float d = __half2float(__ushort_as_half(w.d[wb]));
    const uint8_t* q = w.qs + wb * kQs;
    int v;
    if constexpr (T == NBL_Q8_0) {
      v = static_cast<int8_t>(q[j]);
    } else {
      const int nib = j < 16 ? (q[j] & 0x0F) : (q[j - 16] >> 4);
      if constexpr (T == NBL_Q4_0) {
        v = nib - 8;
      } else {
        v = (nib | (((w.qh[wb] >> j) & 1u) << 4)) - 16;
      }
    }
    out[t * ne0 + e] = __fmul_rn(static_cast<float>(v), d);
  }
}

template <int T, int NT>
void gemv_q_t(cudaStream_t st, const QBatch& b, const int8_t* aq, const float* ad, int64_t ne0, int num_sms) {
  int64_t total = b.row_end[b.count - 1];
  const int64_t grid = std::min<int64_t>((total + kQThreads / 32 - 1) / (kQThreads / 32), int64_t(num_sms) * 8);
  gemv_q_kernel<T, NT><<<static_cast<unsigned>(grid), kQThreads, 0, st>>>(b, aq, ad, ne0);
}

template <int T>
void gemv_q_dispatch(cudaStream_t st, const QBatch& b, const int8_t* aq, const float* ad, int64_t ne0, int64_t n,
                     int sms) {
  switch (n) {
    case 1: return gemv_q_t<T, 1>(st, b, aq, ad, ne0, sms);
    case 2: return gemv_q_t<T, 2>(st, b, aq, ad, ne0, sms);
    case 3: return gemv_q_t<T, 3>(st, b, aq, ad, ne0, sms);
    case 4: return gemv_q_t<T, 4>(st, b, aq, ad, ne0, sms);
    case 5: return gemv_q_t<T, 5>(st, b, aq, ad, ne0, sms);
    case 6: return gemv_q_t<T, 6>(st, b, aq, ad, ne0, sms);
    case 7: return gemv_q_t<T, 7>(st, b, aq, ad, ne0, sms);
    default: return gemv_q_t<T, 8>(st, b, aq, ad, ne0, sms);
  }
}

}  // namespace

bool is_quant(int32_t dtype) { return dtype == NBL_Q4_0 || dtype == NBL_Q5_0 || dtype == NBL_Q8_0; }

int64_t quant_block_bytes(int32_t dtype) {
  return dtype == NBL_Q4_0 ? 18 : dtype == NBL_Q5_0 ? 22 : dtype == NBL_Q8_0 ? 34 : 0;
}

int64_t quant_qs_bytes(int32_t dtype) { return dtype == NBL_Q8_0 ? 32 : 16; }

void launch_quantize_q8_0(cudaStream_t st, const float* x, int8_t* qs, float* d, int64_t n_elems) {
  const int64_t blocks = n_elems / 32;
  const int64_t grid = (blocks * 32 + 255) / 256;
  quantize_q8_0_kernel<<<static_cast<unsigned>(grid), 256, 0, st>>>(x, qs, d, blocks);
}

void launch_gemv_q(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const int8_t* aq,
                   const float* ad, int64_t n, int num_sms) {
  const Weight& w0 = *ws[0];
  const int64_t ne0 = w0.ne0, nb = ne0 / 32;
  for (int64_t t0 = 0; t0 < n; t0 += kGemvMaxRows) {
    const int64_t nt = std::min<int64_t>(kGemvMaxRows, n - t0);
    QBatch b{};
    b.count = count;
    int64_t rows = 0;
    for (int i = 0; i < count; ++i) {
      b.w[i] = ws[i]->q;
      b.y[i] = ys[i] + t0 * ws[i]->ne1;
      rows += ws[i]->ne1;
      b.row_end[i] = rows;
    }
    const int8_t* a = aq + t0 * ne0;
    const float* d = ad + t0 * nb;
    switch (w0.dtype) {
      case NBL_Q4_0: gemv_q_dispatch<NBL_Q4_0>(st, b, a, d, ne0, nt, num_sms); break;
      case NBL_Q5_0: gemv_q_dispatch<NBL_Q5_0>(st, b, a, d, ne0, nt, num_sms); break;
      default: gemv_q_dispatch<NBL_Q8_0>(st, b, a, d, ne0, nt, num_sms); break;
    }
  }
}

void launch_embed_q(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out) {
  const int64_t per_row = std::max<int64_t>(1, std::min<int64_t>((table.ne0 + 255) / 256, 64));
  const dim3 grid(static_cast<unsigned>(per_row), static_cast<unsigned>(n));
  switch (table.dtype) {
    case NBL_Q4_0: embed_q_kernel<NBL_Q4_0><<<grid, 256, 0, st>>>(table.q, ids, out, table.ne0); break;
    case NBL_Q5_0: embed_q_kernel<NBL_Q5_0><<<grid, 256, 0, st>>>(table.q, ids, out, table.ne0); break;
    default: embed_q_kernel<NBL_Q8_0><<<grid, 256, 0, st>>>(table.q, ids, out, table.ne0); break;
  }
}

}  // namespace nbl
