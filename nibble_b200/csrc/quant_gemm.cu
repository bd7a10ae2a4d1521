// Quantized-weight matmul for many activation rows (prefill chunks) on the tcgen05 tensor cores, bit-identical to
// the reference's CPU matmul.
//
// The reference (src/backend/cpu/cpu_backend.cpp:146-233 with the block dots of src/quant.cpp:310-366) quantizes
// every activation row to Q8_0 blocks and forms each output as a sum, in block order, of one float term per
// 32-element block: the block's integer dot sumi converted to float and multiplied by the two fp16 block scales
// (Q4_0: sumi * d_w * d_a; Q8_0: sumi * (d_w * d_a); Q5_0: (d_w * d_a) * sumi). The integer dots are exact, so
// they can come from anywhere; the float ops and their order cannot change.
//
// So here the tensor core computes the integer dots and nothing else: for a tile of 128 weight rows x BN (128 or
// 64) activation rows, one tcgen05.mma kind::i8 (K = 32 = one block) per block writes that block's 128 x BN int32
// dots into its own TMEM buffer (4 buffers of BN columns, a ring), and the epilogue warps read each buffer back
// and add the block's terms to per-output running sums, in block order, with the reference's rounding: every
// multiply and add rounded on its own. (The exact int-to-float conversion and the first product run as packed
// f32x2 operations; the product that feeds the add and the add itself are the scalar _rn intrinsics, since the
// assembler fused a packed multiply with the packed add consuming it, even with .rn and -fmad=false.) The epilogue
// -- about four issue slots per output and block -- bounds the kernel, not the MMA.
//
// Operands (made once per weight, on its first multi-row matmul): the weight's values as int8 [rows][ne0] (Q8_0's
// device values as they are; Q4_0 and Q5_0 unpacked to value - 8 / value - 16) and its scales as fp32
// [blocks][rows]; the activations quantized per call into int8 [n][ne0] and fp32 scales [blocks][n]. All four
// arrive by TMA: per stage, 4 blocks (128 bytes of K) of 128 weight rows and of BN activation rows (128-byte
// swizzle, the canonical K-major layout the MMA reads) plus the 4 x 128 and 4 x BN scales.
#include <algorithm>
#include <atomic>

#include "model_ops.h"
#include "nbl_device.cuh"
#include "quant_common.cuh"

namespace nbl {
namespace {

constexpr int kBM = 128;                     // weight rows per tile: MMA M, TMEM lanes
constexpr int kBlocksPerStage = 4;           // 4 blocks of 32 int8 = one 128-byte swizzle row
constexpr int kStages = 4;
constexpr int kTmemBufs = 4;                 // a ring of kTmemBufs int32 accumulators of BN columns
constexpr int kGroupCols = 32;               // activation rows per epilogue warp
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpEpi0 = 2;
// barriers: full[kStages], empty[kStages], tfull[kTmemBufs], tempty[kTmemBufs], drain; then the TMEM address
constexpr int kBarFull = 0, kBarEmpty = kStages, kBarTFull = 2 * kStages, kBarTEmpty = 2 * kStages + kTmemBufs,
              kBarDrain = 2 * kStages + 2 * kTmemBufs, kNumBars = kBarDrain + 1;

// The layout of one CTA for BN activation rows per tile: BN = 128 runs one CTA per SM with 16 epilogue warps;
// BN = 64 (small matrices: more tiles to spread over the SMs) runs two CTAs per SM with 8 epilogue warps each.
template <int BN>
struct GCfg {
  static constexpr int kGroups = BN / kGroupCols;     // column groups of the epilogue
  static constexpr int kEpiWarps = 4 * kGroups;        // each TMEM lane quarter x each column group
  static constexpr int kThreads = 32 * (kWarpEpi0 + kEpiWarps);
  static constexpr int kCtasPerSm = 128 / BN;
  static constexpr uint32_t kTmemCols = kTmemBufs * BN;
  static constexpr uint32_t kABytes = kBM * 128, kBBytes = BN * 128;
  static constexpr uint32_t kDaBytes = kBlocksPerStage * BN * 4, kDwBytes = kBlocksPerStage * kBM * 4;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes + kDaBytes + kDwBytes;
  static_assert(kStageBytes % 1024 == 0, "stages must keep the 1024-byte alignment of the swizzled tiles");
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
  static constexpr uint32_t kSmemBytes = kOffTmemSlot + 16;
};

// Instruction descriptor for kind::i8: signed 8-bit A and B, s32 accumulator, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_i8(int m, int n) {
  return (2u << 4)                                  // D format: s32
         | (1u << 7) | (1u << 10)                   // A, B: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// D(tmem) = A(smem desc) * B(smem desc), kind::i8 (no accumulation: every block gets a fresh buffer).
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u)
      : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread i of the warp gets columns [col, col+32) of its TMEM lane.
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

// Packed pairs of floats (f32x2: two independent IEEE round-to-nearest operations per instruction).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t a) { return __uint_as_float(static_cast<uint32_t>(a)); }
__device__ __forceinline__ float f2_hi(uint64_t a) { return __uint_as_float(static_cast<uint32_t>(a >> 32)); }

// Two int32 dots as exact floats: for |s| < 2^22 the float with bits 0x4B400000 + s is 1.5 * 2^23 + s exactly,
// and subtracting 1.5 * 2^23 (exact, Sterbenz) leaves s. A block dot is at most 32 * 128 * 127 in magnitude.
__device__ __forceinline__ uint64_t exact_float2(uint32_t s0, uint32_t s1) {
  constexpr uint32_t kMagicBits = 0x4B400000u;
  constexpr float kMagic = 12582912.0f;
  const uint64_t biased = (static_cast<uint64_t>(kMagicBits + s1) << 32) | (kMagicBits + s0);
  return f2_add(biased, f2(-kMagic, -kMagic));
}

struct QGemmMaps {
  CUtensorMap wv[kMaxMulti];  // weight values, int8 [rows][ne0], box 128 x 128, 128-byte swizzle
  CUtensorMap wd[kMaxMulti];  // weight scales, fp32 [blocks][rows], box 4 x 128
  CUtensorMap av;             // activation values, int8 [n][ne0], box 128 x BN, 128-byte swizzle
  CUtensorMap ad;             // activation scales, fp32 [blocks][n], box 4 x BN
};
struct QGemmArgs {
  float* y[kMaxMulti];
  int32_t rows[kMaxMulti];
  int32_t tiles_end[kMaxMulti];  // cumulative tile counts per weight
  int count, n, nb, n_tt, n_tiles;
  int* err;
};

struct Tile {
  int j, row0, tok0;
};
template <int BN>
__device__ __forceinline__ Tile tile_of(const QGemmArgs& a, int t) {
  int j = 0, begin = 0;
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < a.count && t >= a.tiles_end[i - 1]) {
      j = i;
      begin = a.tiles_end[i - 1];
    }
  const int local = t - begin;
  return {j, (local / a.n_tt) * kBM, (local % a.n_tt) * BN};
}
template <typename T>
__device__ __forceinline__ T pick(const T (&v)[kMaxMulti], int j) {
  T r = v[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (j == i) r = v[i];
  return r;
}

template <int T, int BN>
__global__ void __launch_bounds__(GCfg<BN>::kThreads, GCfg<BN>::kCtasPerSm)
    qgemm_kernel(const __grid_constant__ QGemmMaps maps, const QGemmArgs a) {
  using C = GCfg<BN>;
  constexpr int kEpiWarps = C::kEpiWarps;
  constexpr uint32_t kABytes = C::kABytes, kBBytes = C::kBBytes, kDaBytes = C::kDaBytes, kStageBytes = C::kStageBytes;
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
      mbar_init(&bars[kBarFull + s], 1);
      mbar_init(&bars[kBarEmpty + s], 1 + kEpiWarps);  // the MMA commit and every epilogue warp
    }
    for (int b = 0; b < kTmemBufs; ++b) {
      mbar_init(&bars[kBarTFull + b], 1);
      mbar_init(&bars[kBarTEmpty + b], kEpiWarps);
    }
    mbar_init(&bars[kBarDrain], 1);
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
  const int n_kc = (a.nb + kBlocksPerStage - 1) / kBlocksPerStage;

  if (warp == kWarpTma) {
    // ================= producer: per stage, 4 blocks of the tile's weight rows and activation rows + both scales
    if (lane == 0) {
      prefetch_tensormap(&maps.av);
      prefetch_tensormap(&maps.ad);
      int kt = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
        const Tile tl = tile_of<BN>(a, t);
        const CUtensorMap* wv = &maps.wv[0];
        const CUtensorMap* wd = &maps.wd[0];
#pragma unroll
        for (int i = 1; i < kMaxMulti; ++i)
          if (tl.j == i) wv = &maps.wv[i], wd = &maps.wd[i];
        for (int kc = 0; kc < n_kc; ++kc, ++kt) {
          const int s = kt % kStages;
          if (kt >= kStages && !mbar_wait(&bars[kBarEmpty + s], ((kt / kStages) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars[kBarFull + s], kStageBytes);
          tma_load_2d(st, wv, kc * 128, tl.row0, &bars[kBarFull + s]);
          tma_load_2d(st + kABytes, &maps.av, kc * 128, tl.tok0, &bars[kBarFull + s]);
          tma_load_2d(st + kABytes + kBBytes, &maps.ad, tl.tok0, kc * kBlocksPerStage, &bars[kBarFull + s]);
          tma_load_2d(st + kABytes + kBBytes + kDaBytes, wd, tl.row0, kc * kBlocksPerStage, &bars[kBarFull + s]);
        }
      }
      // copies still in flight (an early exit only): let them land before the CTA ends
      for (int k = std::max(0, kt - kStages); k < kt; ++k)
        mbar_wait(&bars[kBarFull + k % kStages], (k / kStages) & 1, a.err);
    }
  } else if (warp == kWarpMma) {
    // ================= MMA issuer: one kind::i8 MMA per block into the next TMEM buffer of the ring
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_i8(kBM, BN);
      int kt = 0, kb = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
        for (int kc = 0; kc < n_kc && ok; ++kc, ++kt) {
          const int s = kt % kStages;
          if (!mbar_wait(&bars[kBarFull + s], (kt / kStages) & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * kStageBytes), b_addr = a_addr + kABytes;
          for (int i = 0; i < kBlocksPerStage && kc * kBlocksPerStage + i < a.nb; ++i, ++kb) {
            const int buf = kb % kTmemBufs;
            if (kb >= kTmemBufs && !mbar_wait(&bars[kBarTEmpty + buf], ((kb / kTmemBufs) & 1) ^ 1, a.err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            tc_mma_i8(tmem + buf * BN, make_sdesc(a_addr + i * 32, 16, 1024, 2),
                      make_sdesc(b_addr + i * 32, 16, 1024, 2), idesc);
            tc_commit(&bars[kBarTFull + buf]);
          }
          tc_commit(&bars[kBarEmpty + s]);
        }
      }
      // every MMA issued has completed before TMEM is released
      tc_commit(&bars[kBarDrain]);
      mbar_wait(&bars[kBarDrain], 0, a.err);
    }
  } else {
    // ================= epilogue: per block, this warp's 32 weight rows x 32 activation rows of int32 dots ->
    // the block's float terms, added to the running sums in block order
    const int e = warp - kWarpEpi0, quarter = warp & 3, group = e / 4;
    const int r_in = quarter * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
    int kt = 0, kb = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
      const Tile tl = tile_of<BN>(a, t);
      float sum[kGroupCols];
#pragma unroll
      for (int c = 0; c < kGroupCols; ++c) sum[c] = 0.f;
      for (int kc = 0; kc < n_kc && ok; ++kc, ++kt) {
        const int s = kt % kStages;
        if (!warp_wait_all(&bars[kBarFull + s], (kt / kStages) & 1, a.err)) {
          ok = false;
          break;
        }
        const float* da_s = reinterpret_cast<const float*>(smem + s * kStageBytes + kABytes + kBBytes);
        const float* dw_s = da_s + kBlocksPerStage * BN;
        for (int i = 0; i < kBlocksPerStage && kc * kBlocksPerStage + i < a.nb; ++i, ++kb) {
          const int buf = kb % kTmemBufs;
          if (!warp_wait_all(&bars[kBarTFull + buf], (kb / kTmemBufs) & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t raw[kGroupCols];
          tmem_ld32(tmem + t_lane + buf * BN + group * kGroupCols, raw);
          tc_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kBarTEmpty + buf]);
          const float dw = dw_s[i * kBM + r_in];
          const uint64_t dw2 = f2(dw, dw);
          const float4* da4 = reinterpret_cast<const float4*>(da_s + i * BN + group * kGroupCols);
#pragma unroll
          for (int c4 = 0; c4 < kGroupCols / 4; ++c4) {
            const float4 d = da4[c4];
            const uint64_t da01 = f2(d.x, d.y), da23 = f2(d.z, d.w);
            const uint64_t s01 = exact_float2(raw[4 * c4], raw[4 * c4 + 1]);
            const uint64_t s23 = exact_float2(raw[4 * c4 + 2], raw[4 * c4 + 3]);
            // the first product packed (its consumer is a multiply), the last product and the add as the
            // scalar _rn intrinsics, which are never merged into a fused multiply-add
            uint64_t a01, b01, a23, b23;
            if constexpr (T == NBL_Q4_0) {  // sumi * d_w * d_a
              a01 = f2_mul(s01, dw2), b01 = da01, a23 = f2_mul(s23, dw2), b23 = da23;
            } else {  // sumi * (d_w * d_a); Q5_0's (d_w * d_a) * sumi is the same product
              a01 = s01, b01 = f2_mul(dw2, da01), a23 = s23, b23 = f2_mul(dw2, da23);
            }
            sum[4 * c4] = __fadd_rn(sum[4 * c4], __fmul_rn(f2_lo(a01), f2_lo(b01)));
            sum[4 * c4 + 1] = __fadd_rn(sum[4 * c4 + 1], __fmul_rn(f2_hi(a01), f2_hi(b01)));
            sum[4 * c4 + 2] = __fadd_rn(sum[4 * c4 + 2], __fmul_rn(f2_lo(a23), f2_lo(b23)));
            sum[4 * c4 + 3] = __fadd_rn(sum[4 * c4 + 3], __fmul_rn(f2_hi(a23), f2_hi(b23)));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarEmpty + s]);
      }
      if (!ok) break;
      const int rows = pick(a.rows, tl.j);
      float* y = pick(a.y, tl.j);
      const int r = tl.row0 + r_in;
      if (r < rows) {
#pragma unroll
        for (int c = 0; c < kGroupCols; ++c) {
          const int tok = tl.tok0 + group * kGroupCols + c;
          if (tok < a.n) y[static_cast<int64_t>(tok) * rows + r] = sum[c];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Activation rows quantized for the GEMM: values [n][ne0], scales transposed [blocks][n_pad] (one warp per block).
__global__ void quantize_act_kernel(const float* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ d,
                                    int64_t n, int64_t ne0, int64_t n_pad) {
  const int lane = threadIdx.x & 31;
  const int64_t nb = ne0 / 32;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x / 32);
  for (int64_t blk = int64_t(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); blk < n * nb; blk += warps) {
    const int64_t t = blk / nb, k = blk - t * nb;
    const float dd = quantize_block(x[t * ne0 + k * 32 + lane], &q[t * ne0 + k * 32 + lane]);
    if (lane == 0) d[k * n_pad + t] = dd;
  }
}

// A Q4_0 / Q5_0 weight's values as int8 [rows][ne0] (value - 8 / value - 16), one thread per block.
template <int T>
__global__ void unpack_values_kernel(const QWeightView w, int8_t* __restrict__ out, int64_t rows, int64_t nb) {
  const int64_t total = rows * nb;
  for (int64_t wb = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; wb < total; wb += int64_t(gridDim.x) * blockDim.x) {
    int lo[4], hi[4];
    unpack_nibbles(*reinterpret_cast<const uint4*>(w.qs + wb * 16), lo, hi);
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (T == NBL_Q4_0) {
        v[i] = __vsub4(lo[i], 0x08080808u);
        v[4 + i] = __vsub4(hi[i], 0x08080808u);
      } else {
        const uint32_t qh = w.qh[wb];
        v[i] = __vsub4(lo[i] | high_bits4(qh, 4 * i), 0x10101010u);
        v[4 + i] = __vsub4(hi[i] | high_bits4(qh, 16 + 4 * i), 0x10101010u);
      }
    }
    uint4* o = reinterpret_cast<uint4*>(out + wb * 32);
    o[0] = make_uint4(v[0], v[1], v[2], v[3]);
    o[1] = make_uint4(v[4], v[5], v[6], v[7]);
  }
}

// fp16 scale bits [rows][blocks] -> fp32 [blocks][rows_pad].
__global__ void scales_t_kernel(const uint16_t* __restrict__ d, float* __restrict__ out, int64_t rows, int64_t nb,
                                int64_t rows_pad) {
  const int64_t total = rows * nb;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t k = i / rows, r = i - k * rows;
    out[k * rows_pad + r] = __half2float(__ushort_as_half(d[r * nb + k]));
  }
}

int64_t pad4(int64_t v) { return (v + 3) / 4 * 4; }

void encode_values(CUtensorMap* m, const void* base, int64_t ne0, int64_t rows, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(ne0), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ne0)};
  const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box);
}
void encode_scales(CUtensorMap* m, const float* base, int64_t rows, int64_t nb, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(nb)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pad4(rows) * 4)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_rows), kBlocksPerStage};
  encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
              CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int T, int BN>
void launch_t(cudaStream_t st, const QGemmMaps& maps, const QGemmArgs& a, int grid) {
  using C = GCfg<BN>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(qgemm_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes),
               "quant gemm smem attribute");
    configured.fetch_or(bit);
  }
  qgemm_kernel<T, BN><<<grid, C::kThreads, C::kSmemBytes, st>>>(maps, a);
}

template <int BN>
void launch_bn(cudaStream_t st, int32_t dtype, const QGemmMaps& maps, const QGemmArgs& a, int grid) {
  switch (dtype) {
    case NBL_Q4_0: launch_t<NBL_Q4_0, BN>(st, maps, a, grid); break;
    case NBL_Q5_0: launch_t<NBL_Q5_0, BN>(st, maps, a, grid); break;
    default: launch_t<NBL_Q8_0, BN>(st, maps, a, grid); break;
  }
}

}  // namespace

void prepare_qgemm(cudaStream_t st, Weight& w, int num_sms) {
  if (w.qg) return;
  auto* g = new QGemmOperand();
  const int64_t nb = w.ne0 / 32;
  try {
    if (w.dtype == NBL_Q8_0) {
      g->vals = reinterpret_cast<const int8_t*>(w.q.qs);
    } else {
      check_cuda(cudaMalloc(&g->owned, static_cast<size_t>(w.ne1 * w.ne0)), "quant gemm values");
      const int64_t blocks = std::min<int64_t>((w.ne1 * nb + 255) / 256, int64_t(num_sms) * 16);
      if (w.dtype == NBL_Q4_0) unpack_values_kernel<NBL_Q4_0><<<blocks, 256, 0, st>>>(w.q, g->owned, w.ne1, nb);
      else unpack_values_kernel<NBL_Q5_0><<<blocks, 256, 0, st>>>(w.q, g->owned, w.ne1, nb);
      check_cuda(cudaGetLastError(), "quant gemm unpack");
      g->vals = g->owned;
    }
    check_cuda(cudaMalloc(&g->scales_t, static_cast<size_t>(nb * pad4(w.ne1)) * sizeof(float)), "quant gemm scales");
    const int64_t blocks = std::min<int64_t>((w.ne1 * nb + 255) / 256, int64_t(num_sms) * 16);
    scales_t_kernel<<<blocks, 256, 0, st>>>(w.q.d, g->scales_t, w.ne1, nb, pad4(w.ne1));
    check_cuda(cudaGetLastError(), "quant gemm scales");
    encode_values(&g->vmap, g->vals, w.ne0, w.ne1, kBM);
    encode_scales(&g->smap, g->scales_t, w.ne1, nb, kBM);
  } catch (...) {
    release_qgemm(g);
    throw;
  }
  w.qg = g;
}

void release_qgemm(QGemmOperand* g) {
  if (!g) return;
  if (g->owned) cudaFree(g->owned);
  if (g->scales_t) cudaFree(g->scales_t);
  delete g;
}

size_t qgemm_act_bytes(int64_t n, int64_t ne0) {
  const size_t vals = (static_cast<size_t>(n * ne0) + 255) / 256 * 256;
  return vals + static_cast<size_t>(ne0 / 32 * pad4(n)) * sizeof(float);
}

void launch_qgemm(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x, int64_t n,
                  void* act, int num_sms, int* err) {
  const int64_t ne0 = ws[0]->ne0, nb = ne0 / 32;
  int8_t* aq = static_cast<int8_t*>(act);
  float* ad = reinterpret_cast<float*>(static_cast<uint8_t*>(act) + (static_cast<size_t>(n * ne0) + 255) / 256 * 256);
  const int64_t qblocks = std::min<int64_t>((n * nb + 7) / 8, int64_t(num_sms) * 16);
  quantize_act_kernel<<<qblocks, 256, 0, st>>>(x, aq, ad, n, ne0, pad4(n));
  check_cuda(cudaGetLastError(), "quant gemm activations");
  QGemmMaps maps;
  QGemmArgs a{};
  a.count = count;
  a.n = static_cast<int>(n);
  a.nb = static_cast<int>(nb);
  a.err = err;
  // 128 activation rows per tile, or 64 (two CTAs per SM) when 128 would leave fewer than two tiles per SM
  int64_t row_tiles = 0;
  for (int i = 0; i < count; ++i) row_tiles += (ws[i]->ne1 + kBM - 1) / kBM;
  const int bn = row_tiles * ((n + 127) / 128) < 2 * int64_t(num_sms) ? 64 : 128;
  a.n_tt = static_cast<int>((n + bn - 1) / bn);
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    maps.wv[i] = ws[i]->qg->vmap;
    maps.wd[i] = ws[i]->qg->smap;
    a.y[i] = ys[i];
    a.rows[i] = static_cast<int32_t>(ws[i]->ne1);
    tiles += static_cast<int>((ws[i]->ne1 + kBM - 1) / kBM) * a.n_tt;
    a.tiles_end[i] = tiles;
  }
  for (int i = count; i < kMaxMulti; ++i) {
    maps.wv[i] = maps.wv[0];
    maps.wd[i] = maps.wd[0];
    a.y[i] = nullptr;
    a.rows[i] = 0;
    a.tiles_end[i] = tiles;
  }
  a.n_tiles = tiles;
  encode_values(&maps.av, aq, ne0, n, bn);
  encode_scales(&maps.ad, ad, n, nb, bn);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, int64_t(num_sms) * (128 / bn)));
  if (bn == 64) launch_bn<64>(st, ws[0]->dtype, maps, a, grid);
  else launch_bn<128>(st, ws[0]->dtype, maps, a, grid);
  check_cuda(cudaGetLastError(), "quant gemm launch");
}

}  // namespace nbl
