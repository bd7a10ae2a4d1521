// Float-weight matmul for many activation rows (prefill chunks, batched decode steps) on the tcgen05 tensor cores at
// fp32 accuracy: y[t][r] = sum_k w[r][k] * x[t][k], the reference's matmul (ref_ops.cpp:109-136 and the tiled SIMD
// GEMM of cpu_backend.cpp:146-233 for F16 / F32 weights), accumulated in fp32.
//
// The tensor core takes 11-significant-bit inputs (fp16, tf32), so the fp32 activations are split into two terms
// exact in the operand type and the products are summed in one fp32 accumulator:
//   F16 weights are read as they are (kind::f16); each activation row is scaled by a power of two so its largest
//   magnitude is below 2^14 and split into fp16 t1 + t2 (the remainder below 2^-22 of an element), w * t1 + w * t2
//   per K-step (2 MMAs), the accumulator multiplied back by the power of two (exact);
//   F32 weights and the activations are split into tf32 terms, w_hi * x_hi + w_hi * x_lo + w_lo * x_hi (kind::tf32,
//   3 MMAs per step; the dropped w_lo * x_lo is below 2^-22 of the product).
// Each product of 11-bit values is exact in fp32, so the result carries fp32 accumulation error only, like the
// reference's (a different summation order).
//
// Kernel: a tile is 128 weight rows (MMA M, TMEM lanes) x BN activation rows (MMA N). Per stage TMA brings one
// 128-byte swizzle row of K (64 fp16 or 32 fp32) of every operand term; one elected thread issues 4 K-steps x the
// terms of tcgen05.mma into the tile's TMEM accumulator (two accumulators, so a tile's epilogue overlaps the next
// tile's MMAs); four epilogue warps move the accumulator to y with tcgen05.ld, each thread one weight row (stores
// coalesced across the warp). Persistent CTAs walk the tiles with the activation tiles of one weight-row tile
// adjacent, so the weight tile is read from L2 by all of them. Up to kMaxMulti weights sharing x (matmul_multi's
// Q/K/V, gate/up) run as one launch, their row tiles numbered consecutively.
#include <algorithm>
#include <atomic>

#include "model_ops.h"
#include "nbl_device.cuh"

namespace nbl {
namespace {

constexpr int kBM = 128;
constexpr int kAccs = 2;     // TMEM accumulators (tiles in flight)
// Two operand modes. TERMS == 3: F32 weights, tf32 terms (4-byte elements, 32 of K per 128-byte swizzle row, K = 8
// per kind::tf32 MMA). TERMS == 2: F16 weights read as they are and fp16 activation terms (2-byte elements, 64 of
// K per row, K = 16 per kind::f16 MMA). A K-step is 32 bytes of a row in both.
template <int TERMS>
constexpr int kKStageOf = TERMS == 3 ? 32 : 64;
template <int TERMS>
constexpr int kKMmaOf = TERMS == 3 ? 8 : 16;
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpEpi0 = 2, kEpiWarps = 4;
constexpr int kThreads = 32 * (kWarpEpi0 + kEpiWarps);

template <int TERMS, int BN>
struct FCfg {
  static constexpr int kATerms = TERMS == 3 ? 2 : 1;  // weight terms in shared memory (hi, lo; or the F16 weight)
  static constexpr int kStages = TERMS == 3 ? 3 : 4;
  static constexpr uint32_t kATile = kBM * 128, kBTile = BN * 128;
  static constexpr uint32_t kStageBytes = kATerms * kATile + 2 * kBTile;
  static_assert(kStageBytes % 1024 == 0, "stages must keep the 1024-byte alignment of the swizzled tiles");
  static constexpr int kBarFull = 0, kBarEmpty = kStages, kBarTFull = 2 * kStages, kBarTEmpty = 2 * kStages + kAccs,
                       kBarDrain = 2 * kStages + 2 * kAccs, kNumBars = kBarDrain + 1;
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
  static constexpr uint32_t kSmemBytes = kOffTmemSlot + 16;
  static constexpr uint32_t kTmemCols = kAccs * BN;
};

// Instruction descriptor for kind::tf32: tf32 A and B, fp32 accumulator, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (2u << 7) | (2u << 10)                   // A, B: tf32
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

struct FGemmMaps {
  CUtensorMap a_hi[kMaxMulti], a_lo[kMaxMulti];  // weights fp32 [rows][ne0] (a_lo: F32 weights), box 32 x 128
  CUtensorMap b_hi, b_lo;                        // activations fp32 [n][ne0], box 32 x BN
};
struct FGemmArgs {
  float* dst[kMaxMulti];        // y_j [n][rows_j], or weight j's split-K partials [k_splits][n][rows_j]
  const float* scale;           // TERMS == 2: the power of two each activation row was scaled down by
  int rows[kMaxMulti];
  int tiles_end[kMaxMulti];     // cumulative tile counts (output tiles x K splits) per weight
  int k_splits[kMaxMulti];      // weight j's K split into k_splits ranges of kc_per_split stages (1: no split)
  int kc_per_split[kMaxMulti];
  int count, n, ne0, n_tt, n_tiles;
  int* err;
};

// Tile t -> weight j, weight-row tile, activation tile, K split (the splits of one output tile adjacent).
struct FTile {
  int j, rows, row0, tok0, kc0, kc1;
  float* dst;
};
template <int BN>
__device__ __forceinline__ FTile ftile_of(const FGemmArgs& a, int t, int n_kc) {
  FTile f;
  f.j = 0;
  int begin = 0;
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < a.count && t >= a.tiles_end[i - 1]) {
      f.j = i;
      begin = a.tiles_end[i - 1];
    }
  float* dst = a.dst[0];
  f.rows = a.rows[0];
  int splits = a.k_splits[0], per = a.kc_per_split[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (f.j == i) dst = a.dst[i], f.rows = a.rows[i], splits = a.k_splits[i], per = a.kc_per_split[i];
  const int local = t - begin, ks = local % splits, ot = local / splits;
  f.row0 = (ot / a.n_tt) * kBM;
  f.tok0 = (ot % a.n_tt) * BN;
  f.kc0 = ks * per;
  f.kc1 = min(n_kc, f.kc0 + per);
  f.dst = dst + static_cast<int64_t>(ks) * a.n * f.rows;
  return f;
}

template <int TERMS, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    fgemm_kernel(const __grid_constant__ FGemmMaps maps, const FGemmArgs a) {
  using C = FCfg<TERMS, BN>;
  constexpr int kStages = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (smem_u32(smem) & 1023u) {  // swizzled tiles need 1024-byte alignment; never expected to trip
    if (threadIdx.x == 0) flag_error(a.err, kErrSmemAlign);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[C::kBarFull + s], 1);
      mbar_init(&bars[C::kBarEmpty + s], 1);
    }
    for (int b = 0; b < kAccs; ++b) {
      mbar_init(&bars[C::kBarTFull + b], 1);
      mbar_init(&bars[C::kBarTEmpty + b], kEpiWarps);
    }
    mbar_init(&bars[C::kBarDrain], 1);
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr int kKStage = kKStageOf<TERMS>, kKMma = kKMmaOf<TERMS>;
  const int n_kc = (a.ne0 + kKStage - 1) / kKStage;
  // stage s: [A_hi][A_lo (TERMS == 3)][B_hi][B_lo]
  auto a_tile = [&](int s, int term) { return smem + s * C::kStageBytes + term * C::kATile; };
  auto b_tile = [&](int s, int term) { return smem + s * C::kStageBytes + C::kATerms * C::kATile + term * C::kBTile; };

  if (warp == kWarpTma) {
    if (lane == 0) {
      int kt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
        const FTile f = ftile_of<BN>(a, t, n_kc);
        const int row0 = f.row0, tok0 = f.tok0;
        const CUtensorMap* ahi = &maps.a_hi[0];
        const CUtensorMap* alo = &maps.a_lo[0];
#pragma unroll
        for (int i = 1; i < kMaxMulti; ++i)
          if (f.j == i) ahi = &maps.a_hi[i], alo = &maps.a_lo[i];
        for (int kc = f.kc0; kc < f.kc1; ++kc, ++kt) {
          const int s = kt % kStages;
          if (kt >= kStages && !mbar_wait(&bars[C::kBarEmpty + s], ((kt / kStages) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          uint64_t* full = &bars[C::kBarFull + s];
          mbar_arrive_expect_tx(full, C::kStageBytes);
          tma_load_2d(a_tile(s, 0), ahi, kc * kKStage, row0, full);
          if constexpr (TERMS == 3) tma_load_2d(a_tile(s, 1), alo, kc * kKStage, row0, full);
          tma_load_2d(b_tile(s, 0), &maps.b_hi, kc * kKStage, tok0, full);
          tma_load_2d(b_tile(s, 1), &maps.b_lo, kc * kKStage, tok0, full);
        }
      }
      for (int k = std::max(0, kt - kStages); k < kt; ++k)  // copies in flight after an early exit
        mbar_wait(&bars[C::kBarFull + k % kStages], (k / kStages) & 1, a.err);
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = TERMS == 3 ? make_idesc_tf32(kBM, BN) : make_idesc_f16(kBM, BN, false, false, false);
      int kt = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x, ++tc) {
        const int acc = tc % kAccs;
        if (tc >= kAccs && !mbar_wait(&bars[C::kBarTEmpty + acc], ((tc / kAccs) & 1) ^ 1, a.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        const FTile f = ftile_of<BN>(a, t, n_kc);
        for (int kc = f.kc0; kc < f.kc1; ++kc, ++kt) {
          const int s = kt % kStages;
          if (!mbar_wait(&bars[C::kBarFull + s], (kt / kStages) & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ah = smem_u32(a_tile(s, 0)), al = smem_u32(a_tile(s, TERMS == 3 ? 1 : 0));
          const uint32_t bh = smem_u32(b_tile(s, 0)), bl = smem_u32(b_tile(s, 1));
#pragma unroll
          for (int kk = 0; kk < kKStage / kKMma; ++kk) {
            const uint32_t off = kk * 32;  // 32 bytes per K-step inside the 128-byte swizzle row
            const uint32_t first = (kc > f.kc0 || kk > 0) ? 1u : 0u;
            if constexpr (TERMS == 3) {
              tc_mma_tf32(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bh + off, 16, 1024, 2), idesc, first);
              tc_mma_tf32(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bl + off, 16, 1024, 2), idesc, 1u);
              tc_mma_tf32(d, make_sdesc(al + off, 16, 1024, 2), make_sdesc(bh + off, 16, 1024, 2), idesc, 1u);
            } else {
              tc_mma_ss(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bh + off, 16, 1024, 2), idesc, first);
              tc_mma_ss(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bl + off, 16, 1024, 2), idesc, 1u);
            }
          }
          tc_commit(&bars[C::kBarEmpty + s]);
        }
        if (ok) tc_commit(&bars[C::kBarTFull + acc]);
      }
      tc_commit(&bars[C::kBarDrain]);  // every MMA has completed before TMEM is released
      mbar_wait(&bars[C::kBarDrain], 0, a.err);
    }
  } else {
    // epilogue: warp (quarter q) owns TMEM lanes 32q..32q+31 = weight rows row0 + 32q + lane
    const int quarter = warp & 3;
    const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
    int tc = 0;
    for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x, ++tc) {
      const int acc = tc % kAccs;
      if (!warp_wait_all(&bars[C::kBarTFull + acc], (tc / kAccs) & 1, a.err)) break;
      tc_fence_after();
      const FTile f = ftile_of<BN>(a, t, n_kc);
      const int row = f.row0 + quarter * 32 + lane, tok0 = f.tok0;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + t_lane + acc * BN + c0, v);
        tc_wait_ld();
        if (row < f.rows) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int tok = tok0 + c0 + j;
            if (tok < a.n) {
              float r = __uint_as_float(v[j]);
              if constexpr (TERMS == 2) r = __fmul_rn(r, a.scale[tok]);  // a power of two: exact
              f.dst[static_cast<int64_t>(tok) * f.rows + row] = r;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[C::kBarTEmpty + acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// x -> (tf32(x), tf32(x - tf32(x))), round to nearest (ties away) like cvt.rna; the difference is exact in fp32.
__device__ __forceinline__ float to_tf32(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t count) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x) {
    const float v = x[i];
    const float h = to_tf32(v);
    hi[i] = h;
    lo[i] = to_tf32(v - h);
  }
}

// One activation row (a CTA each) scaled by a power of two so its largest magnitude lies in [2^13, 2^14), then split
// into two fp16 terms: x * 2^-s = t1 + t2 + r with t1 = fp16(x * 2^-s), t2 = fp16(x * 2^-s - t1) (the difference
// is exact in fp32) and |r| <= 2^-12 |x * 2^-s - t1|, below 2^-22 of the element or 2^-38 of the row's largest one
// where t2 is subnormal. scale[row] = 2^s undoes the scaling exactly in the epilogue.
__global__ void split_f16_rows_kernel(const float* __restrict__ x, __half* __restrict__ t1, __half* __restrict__ t2,
                                      float* __restrict__ scale, int64_t ne0) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float* p = x + row * ne0;
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x) m = fmaxf(m, fabsf(p[i]));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  m = red[0];
  int e = 0;
  if (m > 0.f && m <= 3.4e38f) frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
  const int sh = m > 0.f && m <= 3.4e38f ? e - 14 : 0;
  const float down = ldexpf(1.f, -sh);
  if (threadIdx.x == 0) scale[row] = ldexpf(1.f, sh);
  for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x) {
    const float v = __fmul_rn(p[i], down);
    const __half h1 = __float2half_rn(v);
    t1[row * ne0 + i] = h1;
    t2[row * ne0 + i] = __float2half_rn(__fsub_rn(v, __half2float(h1)));
  }
}

// y[i] = sum over the K splits of partial[s][i], in split order.
__global__ void splitk_sum_kernel(const float* __restrict__ partial, float* __restrict__ y, int64_t count, int splits) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x) {
    float acc = partial[i];
    for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, partial[s * count + i]);
    y[i] = acc;
  }
}

// Rows of 4-byte (tf32 terms) or 2-byte (fp16) elements; a box is one 128-byte swizzle row of K x box_rows.
void encode_rows(CUtensorMap* m, const void* base, int elem, int64_t ne0, int64_t rows, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(ne0), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ne0) * elem};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem), static_cast<cuuint32_t>(box_rows)};
  encode_tmap(m, elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
              const_cast<void*>(base), dims, strides, box);
}

template <int TERMS, int BN>
void launch_t(cudaStream_t st, const FGemmMaps& maps, const FGemmArgs& a, int grid) {
  using C = FCfg<TERMS, BN>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(fgemm_kernel<TERMS, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::kSmemBytes),
               "float gemm smem attribute");
    configured.fetch_or(bit);
  }
  fgemm_kernel<TERMS, BN><<<grid, kThreads, C::kSmemBytes, st>>>(maps, a);
}

int64_t pad_rows(int64_t n) { return (n + 63) / 64 * 64; }  // keeps the partials 256-byte aligned

}  // namespace

// TMA rows must be whole 16-byte multiples: 4 fp32 (tf32 terms of an F32 matrix) or 8 fp16 (an F16 matrix).
bool fgemm_supported(int32_t dtype, int64_t ne0) { return ne0 % (dtype == NBL_F16 ? 8 : 4) == 0; }

constexpr int kMaxSplits = 16;
constexpr int kMinStagesPerSplit = 8;  // 8 128-byte rows of K per split at least

size_t fgemm_act_bytes(int64_t n, int64_t rows, int64_t ne0) {
  // the two activation terms (fp32 for F32 weights; fp16 for F16 weights, which use half), the activation rows'
  // scales, then room for the split-K partials
  return static_cast<size_t>(2 * n * ne0 + pad_rows(n) + kMaxSplits * n * rows) * sizeof(float);
}

void split_tf32(cudaStream_t st, const float* x, float* hi, float* lo, int64_t count, int num_sms) {
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((count + 255) / 256, int64_t(num_sms) * 8));
  split_tf32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(x, hi, lo, count);
  check_cuda(cudaGetLastError(), "tf32 split launch");
}

void launch_fgemm(cudaStream_t st, const void* const* w_hi, const float* const* w_lo, const int64_t* rows,
                  float* const* ys, int count, int64_t ne0, const float* x, int64_t n, void* act, int num_sms,
                  int* err) {
  const bool f16 = w_lo[0] == nullptr;  // F16 weights as they are; else the tf32 terms of F32 weights
  const int elem = f16 ? 2 : 4;
  float* xh = static_cast<float*>(act);  // activation term 1, then term 2, of elem bytes each
  void* b1 = xh;
  void* b2 = static_cast<uint8_t*>(act) + static_cast<size_t>(n * ne0) * elem;
  float* scale = xh + 2 * n * ne0;
  float* partial = scale + pad_rows(n);
  if (f16) {
    split_f16_rows_kernel<<<static_cast<unsigned>(n), 256, 0, st>>>(x, static_cast<__half*>(b1),
                                                                      static_cast<__half*>(b2), scale, ne0);
    check_cuda(cudaGetLastError(), "fp16 split launch");
  } else {
    split_tf32(st, x, static_cast<float*>(b1), static_cast<float*>(b2), n * ne0, num_sms);
  }
  // the tile shape and each weight's K split depend on n and that weight alone, never on the group, so a
  // matmul_multi launch gives every weight the bits a separate call gives it
  const int bn = n <= 64 ? 64 : 128;
  FGemmArgs a{};
  a.count = count;
  a.n = static_cast<int>(n);
  a.ne0 = static_cast<int>(ne0);
  a.n_tt = static_cast<int>((n + bn - 1) / bn);
  a.scale = scale;
  // for decode-sized n (<= 128 activation rows), a weight whose output tiles cannot cover the SMs alone splits K
  // (partials summed in split order by a second launch); prefill chunks keep whole K per tile, where the partials'
  // extra traffic and launch cost more than the idle SMs (measured: pp512 75.8k -> 80.3k tok/s without them)
  const int64_t k_row = 128 / elem, n_kc = (ne0 + k_row - 1) / k_row;
  a.err = err;
  FGemmMaps maps;
  int tiles = 0;
  int64_t part_off = 0;
  for (int i = 0; i < kMaxMulti; ++i) {
    const int w = i < count ? i : 0;
    if (i < count) {
      const int64_t out_tiles = (rows[i] + kBM - 1) / kBM * a.n_tt;
      int splits = 1;
      if (out_tiles < num_sms && n <= 128)
        splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({(num_sms + out_tiles - 1) / out_tiles,
                                                                           n_kc / kMinStagesPerSplit, kMaxSplits})));
      a.kc_per_split[i] = static_cast<int>((n_kc + splits - 1) / splits);
      a.k_splits[i] = static_cast<int>((n_kc + a.kc_per_split[i] - 1) / a.kc_per_split[i]);
      a.rows[i] = static_cast<int>(rows[i]);
      a.dst[i] = a.k_splits[i] > 1 ? partial + part_off : ys[i];
      if (a.k_splits[i] > 1) part_off += static_cast<int64_t>(a.k_splits[i]) * n * rows[i];
      tiles += static_cast<int>(out_tiles) * a.k_splits[i];
    } else {
      a.rows[i] = 0;
      a.dst[i] = nullptr;
      a.k_splits[i] = 1;
      a.kc_per_split[i] = static_cast<int>(n_kc);
    }
    a.tiles_end[i] = tiles;
    encode_rows(&maps.a_hi[i], w_hi[w], elem, ne0, rows[w], kBM);
    encode_rows(&maps.a_lo[i], w_lo[w] ? static_cast<const void*>(w_lo[w]) : w_hi[w], elem, ne0, rows[w], kBM);
  }
  a.n_tiles = tiles;
  encode_rows(&maps.b_hi, b1, elem, ne0, n, bn);
  encode_rows(&maps.b_lo, b2, elem, ne0, n, bn);
  const int grid = static_cast<int>(std::min<int64_t>(a.n_tiles, num_sms));
  if (!f16) {
    if (bn == 64) launch_t<3, 64>(st, maps, a, grid);
    else launch_t<3, 128>(st, maps, a, grid);
  } else {
    if (bn == 64) launch_t<2, 64>(st, maps, a, grid);
    else launch_t<2, 128>(st, maps, a, grid);
  }
  check_cuda(cudaGetLastError(), "float gemm launch");
  part_off = 0;
  for (int i = 0; i < count; ++i) {
    if (a.k_splits[i] == 1) continue;
    const int64_t cnt = n * rows[i];
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((cnt + 255) / 256, int64_t(num_sms) * 8));
    splitk_sum_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(partial + part_off, ys[i], cnt, a.k_splits[i]);
    check_cuda(cudaGetLastError(), "float gemm split-K sum");
    part_off += static_cast<int64_t>(a.k_splits[i]) * cnt;
  }
}

}  // namespace nbl
