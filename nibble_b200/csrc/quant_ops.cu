// Quantized weight matmuls and embedding rows on the GPU, bit-identical to nibble's CPU kernels for the weight types
// whose activations are Q8_0 blocks: Q4_0, Q5_0 and Q8_0 (src/quant.h:1-20, src/quant.cpp:37-51 (activation
// quantizer), :158-205 (dequantize_row), :310-366 (block dots)).
//
// The reference never dequantizes a weight for a matmul: it quantizes each activation row to Q8_0 blocks (d =
// max|x| / 127 rounded to fp16, q = roundf(x / d)), takes the integer dot of each weight block with the activation
// block, turns it into a float term with the two fp16 scales (the operation order differs per type and is kept
// exactly: Q4_0 sumi * d_w * d_a, Q8_0 sumi * (d_w * d_a), Q5_0 (d_w * d_a) * sumi), and adds the terms to the row's
// sum in block order. Here the activation rows are quantized once per call (one warp per block, the same
// arithmetic, so the same bits), the integer dots run four products per dp4a instruction, every float operation is
// an uncontracted _rn intrinsic, and one row's terms are added in block order (lanes hold consecutive blocks; their
// terms are broadcast to the whole warp one block at a time), so every output equals the CPU's bit for bit.
//
// Device layouts (made at upload, nbl_weight_create): the GGUF blocks of a row are split into aligned arrays --
// fp16 scale bits [rows][blocks], the value bytes [rows][blocks][16 or 32] (16-byte aligned per block) and, for
// Q5_0, the 32 high bits [rows][blocks] -- so a lane reads its block with one or two 16-byte loads. Quantized
// activations are int8 values [n][ne0] and the fp32 value of each block's fp16-rounded scale [n][blocks].
#include <algorithm>
#include <atomic>

#include "model_ops.h"
#include "nbl_device.cuh"
#include "qkv_epilogue.cuh"
#include "quant_common.cuh"

namespace nbl {
namespace {

// ---------------------------------------------------------------- block dots
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
constexpr int kQRegBlocks = 8;  // single-row decode: a lane keeps up to 8 activation blocks (ne0 <= 8192) in registers

// The activation rows of a GEMV quantized to Q8_0 blocks once per call (one warp per block, the reference's
// arithmetic): int8 values [n][ne0] and the fp32 value of each block's fp16 scale [n][ne0 / 32]. Launched with
// programmatic stream serialization: it waits for x, then lets the GEMV launch and start streaming its weights.
__global__ void quantize_rows_kernel(const float* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ d,
                                     int64_t n_blocks) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t blk = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (blk >= n_blocks) return;
  const float dd = quantize_block(x[blk * 32 + lane], &q[blk * 32 + lane]);
  if (lane == 0) d[blk] = dd;
}

// y_j[t][r] over up to kMaxMulti weights of type T (rows numbered consecutively, as in the float GEMV), from the NT
// quantized activation rows (aq, ad). One warp per weight row, grid-stride, lane l taking blocks l, l + 32, ...;
// each round of 32 block terms is added to the row's sum in block order. The warp's first row is prefetched into
// L2 before the kernel waits for the quantizer. REG (NT == 1, at most kQRegBlocks blocks per lane): each lane
// keeps its activation blocks in registers across rows.
// EPI: the fused Q/K/V projection (launch_gemv_q_qkv): a warp takes the two rows of a RoPE pair (qkv_row) one after
// the other and, once both sums are done, lanes 0..NT-1 run the epilogue of one activation row each.
template <int T, int NT, bool REG, bool EPI = false>
__global__ void __launch_bounds__(kQThreads) gemv_q_kernel(const QBatch b, const int8_t* __restrict__ aq,
                                                           const float* __restrict__ ad, int64_t ne0,
                                                           const QkvEpilogue e) {
  constexpr int kQs = QTraits<T>::kQsBytes;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nb = ne0 / 32;
  int64_t total = b.row_end[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < b.count) total = b.row_end[i];
  const int64_t n_warps = int64_t(gridDim.x) * (kQThreads / 32);
  const int64_t r0 = int64_t(blockIdx.x) * (kQThreads / 32) + warp;
  // this row's weight j (a static scan of the parameter block)
  auto locate = [&](int64_t r, QWeightView& w, float*& y, int64_t& lr, int64_t& rows_j) {
    w = b.w[0];
    y = b.y[0];
    int64_t begin = 0;
    rows_j = b.row_end[0];
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
    lr = r - begin;
  };
  const int64_t n_items = EPI ? total / 2 : total;  // rows, or RoPE pairs of rows
  int region = 0, head = 0, pair = 0;
  if (r0 < n_items) {
    QWeightView w;
    float* y;
    int64_t lr, rows_j;
    locate(EPI ? qkv_row(2 * r0, e, region, head, pair) : r0, w, y, lr, rows_j);
    for (int64_t blk = lane; blk < nb; blk += 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(w.qs + (lr * nb + blk) * kQs));
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the quantized activations
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  int areg[REG ? kQRegBlocks : 1][8];
  float dreg[REG ? kQRegBlocks : 1];
  if constexpr (REG) {
#pragma unroll
    for (int i = 0; i < kQRegBlocks; ++i) {
      const int64_t blk = lane + 32 * i;
      if (blk < nb) {
        const uint4 a0 = *reinterpret_cast<const uint4*>(aq + blk * 32);
        const uint4 a1 = *reinterpret_cast<const uint4*>(aq + blk * 32 + 16);
        areg[i][0] = int(a0.x), areg[i][1] = int(a0.y), areg[i][2] = int(a0.z), areg[i][3] = int(a0.w);
        areg[i][4] = int(a1.x), areg[i][5] = int(a1.y), areg[i][6] = int(a1.z), areg[i][7] = int(a1.w);
        dreg[i] = ad[blk];
      }
    }
  }
  for (int64_t item = r0; item < n_items; item += n_warps) {
  float first[EPI ? NT : 1];
#pragma unroll 1
  for (int member = 0; member < (EPI ? 2 : 1); ++member) {
    const int64_t r = EPI ? qkv_row(2 * item + member, e, region, head, pair) : item;
    QWeightView w;
    float* y;
    int64_t lr, rows_j;
    locate(r, w, y, lr, rows_j);
    float sum[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) sum[t] = 0.f;
#pragma unroll(REG ? kQRegBlocks : 1)
    for (int round = 0; round < (REG ? kQRegBlocks : 1 << 30); ++round) {
      const int64_t k0 = int64_t(round) * 32;
      if (k0 >= nb) break;
      const int64_t blk = k0 + lane;
      float term[NT];
      if (blk < nb) {
        const int64_t wb = lr * nb + blk;
        const float dw = __half2float(__ushort_as_half(w.d[wb]));
        const uint32_t qh = T == NBL_Q5_0 ? w.qh[wb] : 0u;
        const uint8_t* wq = w.qs + wb * kQs;
        if constexpr (REG) {
          term[0] = block_term<T>(wq, qh, dw, areg[round], dreg[round]);
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint4 a0 = *reinterpret_cast<const uint4*>(aq + t * ne0 + blk * 32);
            const uint4 a1 = *reinterpret_cast<const uint4*>(aq + t * ne0 + blk * 32 + 16);
            const int av[8] = {int(a0.x), int(a0.y), int(a0.z), int(a0.w), int(a1.x), int(a1.y), int(a1.z), int(a1.w)};
            term[t] = block_term<T>(wq, qh, dw, av, ad[t * nb + blk]);
          }
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
    if constexpr (!EPI) {
      if (lane == 0)
#pragma unroll
        for (int t = 0; t < NT; ++t) y[t * rows_j + lr] = sum[t];
    } else if (member == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) first[t] = sum[t];  // every lane holds every row's sum
    } else {
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (lane == t) qkv_store(e, region, head, pair, t, first[t], sum[t]);
    }
  }
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

cudaLaunchAttribute pdl_attr() {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}

// Both launches use programmatic stream serialization (each kernel waits for its predecessor before reading).
template <int T, int NT, bool REG, bool EPI = false>
void gemv_q_t(cudaStream_t st, const QBatch& b, const int8_t* aq, const float* ad, int64_t ne0, int num_sms,
              const QkvEpilogue& e = QkvEpilogue{}) {
  const int64_t total = EPI ? b.row_end[b.count - 1] / 2 : b.row_end[b.count - 1];
  int per_sm = 0;
  check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_q_kernel<T, NT, REG, EPI>, kQThreads, 0),
             "quant gemv occupancy");
  const int64_t grid = std::min<int64_t>((total + kQThreads / 32 - 1) / (kQThreads / 32),
                                         int64_t(num_sms) * std::max(1, std::min(per_sm, 8)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kQThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1] = {pdl_attr()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, gemv_q_kernel<T, NT, REG, EPI>, b, aq, ad, ne0, e), "quant gemv launch");
}

template <int T, bool EPI = false>
void gemv_q_dispatch(cudaStream_t st, const QBatch& b, const int8_t* aq, const float* ad, int64_t ne0, int64_t n,
                     int sms, const QkvEpilogue& e = QkvEpilogue{}) {
  if (n == 1 && ne0 / 32 <= 32 * kQRegBlocks) return gemv_q_t<T, 1, true, EPI>(st, b, aq, ad, ne0, sms, e);
  switch (n) {
    case 1: return gemv_q_t<T, 1, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 2: return gemv_q_t<T, 2, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 3: return gemv_q_t<T, 3, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 4: return gemv_q_t<T, 4, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 5: return gemv_q_t<T, 5, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 6: return gemv_q_t<T, 6, false, EPI>(st, b, aq, ad, ne0, sms, e);
    case 7: return gemv_q_t<T, 7, false, EPI>(st, b, aq, ad, ne0, sms, e);
    default: return gemv_q_t<T, 8, false, EPI>(st, b, aq, ad, ne0, sms, e);
  }
}

// The activation rows quantized to Q8_0 blocks into act (int8 values, then the block scales): one launch.
void quantize_act(cudaStream_t st, const float* x, int64_t nt, int64_t ne0, int8_t* aq, float* ad) {
  const int64_t nb = ne0 / 32;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((nt * nb + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1] = {pdl_attr()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, quantize_rows_kernel, x, aq, ad, nt * nb), "quantize activations launch");
}

}  // namespace

bool is_quant(int32_t dtype) { return dtype == NBL_Q4_0 || dtype == NBL_Q5_0 || dtype == NBL_Q8_0; }

int64_t quant_block_bytes(int32_t dtype) {
  return dtype == NBL_Q4_0 ? 18 : dtype == NBL_Q5_0 ? 22 : dtype == NBL_Q8_0 ? 34 : 0;
}

int64_t quant_qs_bytes(int32_t dtype) { return dtype == NBL_Q8_0 ? 32 : 16; }

size_t gemv_q_act_bytes(int64_t ne0) {
  return static_cast<size_t>(kGemvMaxRows * ne0) + static_cast<size_t>(kGemvMaxRows * (ne0 / 32)) * sizeof(float);
}

void launch_gemv_q(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x, int64_t n,
                   void* act, int num_sms) {
  const Weight& w0 = *ws[0];
  const int64_t ne0 = w0.ne0, nb = ne0 / 32;
  int8_t* aq = static_cast<int8_t*>(act);
  float* ad = reinterpret_cast<float*>(aq + kGemvMaxRows * ne0);
  (void)nb;
  for (int64_t t0 = 0; t0 < n; t0 += kGemvMaxRows) {
    const int64_t nt = std::min<int64_t>(kGemvMaxRows, n - t0);
    quantize_act(st, x + t0 * ne0, nt, ne0, aq, ad);
    QBatch b{};
    b.count = count;
    int64_t rows = 0;
    for (int i = 0; i < count; ++i) {
      b.w[i] = ws[i]->q;
      b.y[i] = ys[i] + t0 * ws[i]->ne1;
      rows += ws[i]->ne1;
      b.row_end[i] = rows;
    }
    switch (w0.dtype) {
      case NBL_Q4_0: gemv_q_dispatch<NBL_Q4_0>(st, b, aq, ad, ne0, nt, num_sms); break;
      case NBL_Q5_0: gemv_q_dispatch<NBL_Q5_0>(st, b, aq, ad, ne0, nt, num_sms); break;
      default: gemv_q_dispatch<NBL_Q8_0>(st, b, aq, ad, ne0, nt, num_sms); break;
    }
  }
}

bool gemv_q_qkv_ok(const Weight* const* ws, int64_t n, int64_t n_heads, int64_t n_kv_heads) {
  const Weight &wq = *ws[0], &wk = *ws[1], &wv = *ws[2];
  return n >= 1 && n <= kGemvMaxRows && is_quant(wq.dtype) && wk.dtype == wq.dtype && wv.dtype == wq.dtype &&
         wq.ne0 == wk.ne0 && wq.ne0 == wv.ne0 && n_heads > 0 && n_kv_heads > 0 && wq.ne1 == n_heads * 64 &&
         wk.ne1 == n_kv_heads * 64 && wv.ne1 == wk.ne1;
}

bool launch_gemv_q_qkv(cudaStream_t st, const Weight* const* ws, const float* x, int64_t n, void* act,
                       const QkvEpilogue& e, int num_sms) {
  if (!gemv_q_qkv_ok(ws, n, e.n_heads, e.n_kv_heads)) return false;
  const int64_t ne0 = ws[0]->ne0;
  int8_t* aq = static_cast<int8_t*>(act);
  float* ad = reinterpret_cast<float*>(aq + kGemvMaxRows * ne0);
  quantize_act(st, x, n, ne0, aq, ad);
  QBatch b{};
  b.count = 3;
  int64_t rows = 0;
  for (int i = 0; i < 3; ++i) {
    b.w[i] = ws[i]->q;
    b.y[i] = nullptr;  // the epilogue stores instead
    rows += ws[i]->ne1;
    b.row_end[i] = rows;
  }
  switch (ws[0]->dtype) {
    case NBL_Q4_0: gemv_q_dispatch<NBL_Q4_0, true>(st, b, aq, ad, ne0, n, num_sms, e); break;
    case NBL_Q5_0: gemv_q_dispatch<NBL_Q5_0, true>(st, b, aq, ad, ne0, n, num_sms, e); break;
    default: gemv_q_dispatch<NBL_Q8_0, true>(st, b, aq, ad, ne0, n, num_sms, e); break;
  }
  return true;
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
