// Float-weight matmul for many activation rows (prefill chunks, batched decode steps) on the tcgen05 tensor cores at
// fp32 accuracy: y[t][r] = sum_k w[r][k] * x[t][k], the reference's matmul (ref_ops.cpp:109-136 and the tiled SIMD
// GEMM of cpu_backend.cpp:146-233 for F16 / F32 weights), accumulated in fp32.
//
// The tensor core's fp32-class input is tf32 (11 significant bits), so each operand is split into terms that are
// exact in tf32 and the products that matter are summed in one fp32 accumulator:
//   F16 weights are exact in tf32 (11 significant bits, and every fp16 exponent fits), x = x_hi + x_lo with
//   x_hi = tf32(x), x_lo = tf32(x - x_hi) (|x - x_hi - x_lo| <= 2^-24 |x|):  w * x_hi + w * x_lo   (2 MMAs per step);
//   F32 weights likewise split, w_hi * x_hi + w_hi * x_lo + w_lo * x_hi        (3 MMAs per step; the dropped
//   w_lo * x_lo is below 2^-22 of the product).
// Each product of tf32 values is exact in fp32, so the result carries fp32 accumulation error only, like the
// reference's (a different summation order).
//
// Kernel: a tile is 128 weight rows (MMA M, TMEM lanes) x BN activation rows (MMA N). Per stage TMA brings 32 fp32
// of K (one 128-byte swizzle row) of every operand term; one elected thread issues 4 K-steps (K = 8) x the terms of
// tcgen05.mma kind::tf32 into the tile's TMEM accumulator (two accumulators, so a tile's epilogue overlaps the next
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
constexpr int kKStage = 32;  // fp32 elements of K per stage: one 128-byte swizzle row
constexpr int kKMma = 8;     // K of one kind::tf32 MMA
constexpr int kAccs = 2;     // TMEM accumulators (tiles in flight)
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpEpi0 = 2, kEpiWarps = 4;
constexpr int kThreads = 32 * (kWarpEpi0 + kEpiWarps);

template <int TERMS, int BN>
struct FCfg {
  static constexpr int kATerms = TERMS == 3 ? 2 : 1;  // weight terms in shared memory (hi, lo)
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
      constexpr uint32_t idesc = make_idesc_tf32(kBM, BN);
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
            const uint32_t off = kk * kKMma * 4;  // 32 bytes per K-step inside the 128-byte swizzle row
            tc_mma_tf32(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bh + off, 16, 1024, 2), idesc,
                        (kc > f.kc0 || kk > 0) ? 1u : 0u);
            tc_mma_tf32(d, make_sdesc(ah + off, 16, 1024, 2), make_sdesc(bl + off, 16, 1024, 2), idesc, 1u);
            if constexpr (TERMS == 3)
              tc_mma_tf32(d, make_sdesc(al + off, 16, 1024, 2), make_sdesc(bh + off, 16, 1024, 2), idesc, 1u);
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
      const FTile f = ftile_of<BN>(a, t, (a.ne0 + kKStage - 1) / kKStage);
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
            if (tok < a.n) f.dst[static_cast<int64_t>(tok) * f.rows + row] = __uint_as_float(v[j]);
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

// y[i] = sum over the K splits of partial[s][i], in split order.
__global__ void splitk_sum_kernel(const float* __restrict__ partial, float* __restrict__ y, int64_t count, int splits) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x) {
    float acc = partial[i];
    for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, partial[s * count + i]);
    y[i] = acc;
  }
}

void encode_rows(CUtensorMap* m, const float* base, int64_t ne0, int64_t rows, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(ne0), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ne0) * 4};
  const cuuint32_t box[2] = {kKStage, static_cast<cuuint32_t>(box_rows)};
  encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box);
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

}  // namespace

bool fgemm_supported(int64_t ne0) { return ne0 % 4 == 0; }

constexpr int kMaxSplits = 16;
constexpr int kMinStagesPerSplit = 8;  // 256 K per split at least

size_t fgemm_act_bytes(int64_t n, int64_t rows, int64_t ne0) {
  // the two activation terms, then room for the split-K partials
  return static_cast<size_t>(2 * n * ne0 + kMaxSplits * n * rows) * sizeof(float);
}

void split_tf32(cudaStream_t st, const float* x, float* hi, float* lo, int64_t count, int num_sms) {
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((count + 255) / 256, int64_t(num_sms) * 8));
  split_tf32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(x, hi, lo, count);
  check_cuda(cudaGetLastError(), "tf32 split launch");
}

void launch_fgemm(cudaStream_t st, const float* const* w_hi, const float* const* w_lo, const int64_t* rows,
                  float* const* ys, int count, int64_t ne0, const float* x, int64_t n, void* act, int num_sms,
                  int* err) {
  float* xh = static_cast<float*>(act);
  float* xl = xh + n * ne0;
  float* partial = xl + n * ne0;
  split_tf32(st, x, xh, xl, n * ne0, num_sms);
  // the tile shape and each weight's K split depend on n and that weight alone, never on the group, so a
  // matmul_multi launch gives every weight the bits a separate call gives it
  const int bn = n <= 64 ? 64 : 128;
  FGemmArgs a{};
  a.count = count;
  a.n = static_cast<int>(n);
  a.ne0 = static_cast<int>(ne0);
  a.n_tt = static_cast<int>((n + bn - 1) / bn);
  // a weight whose output tiles cannot cover the SMs alone splits K (partials summed in split order by a second
  // launch)
  const int64_t n_kc = (ne0 + kKStage - 1) / kKStage;
  a.err = err;
  FGemmMaps maps;
  int tiles = 0;
  int64_t part_off = 0;
  for (int i = 0; i < kMaxMulti; ++i) {
    const int w = i < count ? i : 0;
    if (i < count) {
      const int64_t out_tiles = (rows[i] + kBM - 1) / kBM * a.n_tt;
      int splits = 1;
      if (out_tiles < num_sms)
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
    encode_rows(&maps.a_hi[i], w_hi[w], ne0, rows[w], kBM);
    encode_rows(&maps.a_lo[i], w_lo[w] ? w_lo[w] : w_hi[w], ne0, rows[w], kBM);
  }
  a.n_tiles = tiles;
  encode_rows(&maps.b_hi, xh, ne0, n, bn);
  encode_rows(&maps.b_lo, xl, ne0, n, bn);
  const int grid = static_cast<int>(std::min<int64_t>(a.n_tiles, num_sms));
  if (w_lo[0]) {
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
