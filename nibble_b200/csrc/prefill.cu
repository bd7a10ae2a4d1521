// Causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMEM), reading K/V from the paged pool.
//
// Replaces Backend::attention for n > 1 (src/backend/backend.h:66-69; the reference's scalar loop is
// src/backend/cpu/ref_ops.cpp:188-214): query row t of an item has position kv_pos0 + t and attends keys
// 0..kv_pos0+t; query head h reads KV head h / G.
//
// One CTA = one 128-row query tile of one head. Six warps, specialised:
//   warp 0      TMA producer: the Q tile once (3-D map over q), then K/V tiles of 128 keys (8 pages, one
//               16x64 box each for K and V) through a 3-stage shared-memory ring; 128-byte swizzle.
//   warp 1      MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=128, K=64), then O += P V into TMEM
//               (M=128, N=64, K=128) with V used as an MN-major operand straight from the TMA tile. Completion
//               is signalled with tcgen05.commit on mbarriers.
//   warps 2-5   softmax: thread i owns query row i = TMEM lane i. It loads its S row from TMEM, applies the
//               causal mask, keeps the online max/sum in fp32 (log2 domain), writes P as bf16/fp16 into a
//               swizzled shared tile (the A operand of the PV MMA), rescales its O row in TMEM when the max
//               moves, and finally normalises O and stores the output row.
// S_{j+1} = Q K_{j+1}^T is issued as soon as the softmax has read S_j, so it overlaps the exponentials of
// tile j; PV_j overlaps the exponentials of tile j+1.
// CTAs of one (item, KV head) are numbered consecutively, so the G heads x query tiles that read the same K/V
// run together and the K/V tiles come from L2 after the first read.
//
// Every mbarrier wait is bounded (nbl_device.cuh): a lost completion ends the CTA with kErrTimeout set.
#include <algorithm>
#include <atomic>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

constexpr int kD = 64;
constexpr int kBM = 128;                 // query rows per CTA
constexpr int kBN = 128;                 // keys per tile
constexpr int kPage = 16;
constexpr int kPagesPerTile = kBN / kPage;
constexpr int kStages = 3;
constexpr int kTileBytes = kBN * kD * 2;  // one K (or V) tile: 16 KB
constexpr int kQBytes = kBM * kD * 2;     // 16 KB
constexpr int kPBytes = kBM * kBN * 2;    // 32 KB (two 64-key swizzle atoms of [128 rows][128 B])
constexpr int kBoxBytes = kPage * kD * 2; // 2 KB
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kQBytes;
constexpr int kOffP = kOffKV + kStages * 2 * kTileBytes;
constexpr int kOffBar = kOffP + kPBytes;
constexpr int kSmemBytes = 1024 + kOffBar + 256;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;  // S: columns [0,128), O: [128,192)
constexpr uint32_t kColS = 0, kColO = 128;
// barrier slots
constexpr int kBarQ = 0, kBarFull = 1, kBarEmpty = 1 + kStages, kBarSFull = 1 + 2 * kStages,
              kBarSFree = kBarSFull + 1, kBarPFull = kBarSFull + 2, kBarODone = kBarSFull + 3;

struct PrefillArgs {
  const int32_t* q_start;
  const int32_t* q_len;
  const int32_t* kv_pos0;
  const int32_t* page_table;
  void* out;
  int* err;
  int64_t n_pages;
  int64_t n_q_rows;
  int32_t pt_stride;
  int out_f32;
  int n_heads, n_kv_heads, group, m_tiles;
  float scale_log2;
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 32 consecutive TMEM columns of this warp's lane quarter into registers, waiting for completion inside the
// same asm statement so no use of the registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld32_wait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

// Bounded wait executed by every lane of a warp; true only if all lanes saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, err));
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kvmap,
                   const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- which tile: CTAs of one (item, KV head) are consecutive; heavier (later) query tiles first
  const int per_group = a.m_tiles * a.group;
  const int grp = blockIdx.x / per_group;
  const int within = blockIdx.x % per_group;
  const int mt = a.m_tiles - 1 - within / a.group;
  const int g = within % a.group;
  const int item = grp / a.n_kv_heads, kvh = grp % a.n_kv_heads;
  const int h = kvh * a.group + g;
  const int qlen = a.q_len[item], pos0 = a.kv_pos0[item], qs = a.q_start[item];
  const int m0 = mt * kBM;
  if (qlen <= 0 || m0 >= qlen) return;
  const int64_t kv_len = int64_t(pos0) + qlen;
  if (pos0 < 0 || qs < 0 || int64_t(qs) + qlen > a.n_q_rows || kv_len > int64_t(a.pt_stride) * kPage) {
    if (threadIdx.x == 0) flag_error(a.err, kErrLength);
    return;
  }
  const int kv_end = static_cast<int>(std::min<int64_t>(kv_len, int64_t(pos0) + m0 + kBM));
  const int n_kv = (kv_end + kBN - 1) / kBN;
  const int n_item_pages = static_cast<int>((kv_len + kPage - 1) / kPage);
  const int32_t* pt_row = a.page_table + int64_t(item) * a.pt_stride;

  uint8_t* sQ = smem + kOffQ;
  uint8_t* sP = smem + kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 128);
  auto sK = [&](int s) { return smem + kOffKV + s * 2 * kTileBytes; };
  auto sV = [&](int s) { return smem + kOffKV + s * 2 * kTileBytes + kTileBytes; };

  if (threadIdx.x == 0) {
    mbar_init(&bars[kBarQ], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarFull + s], 1);
      mbar_init(&bars[kBarEmpty + s], 1);
    }
    mbar_init(&bars[kBarSFull], 1);
    mbar_init(&bars[kBarSFree], 128);
    mbar_init(&bars[kBarPFull], 128);
    mbar_init(&bars[kBarODone], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ================= TMA producer
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kvmap);
      mbar_arrive_expect_tx(&bars[kBarQ], kQBytes);
      tma_load_3d(sQ, &qmap, 0, h, qs + m0, &bars[kBarQ]);
    }
    for (int j = 0; j < n_kv; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !warp_wait(&bars[kBarEmpty + s], ((j / kStages) & 1) ^ 1, a.err)) break;
      const int pg = j * kPagesPerTile + lane;
      int32_t pid = -1;
      if (lane < kPagesPerTile && pg < n_item_pages) {
        pid = pt_row[pg];
        if (pid < 0 || pid >= a.n_pages) {
          flag_error(a.err, kErrPageId);
          pid = -1;
        }
      }
      const uint32_t present = __ballot_sync(0xffffffffu, pid >= 0) & 0xffu;
      if (present != 0xffu) {
        // Pages past the item's end (or rejected ids) are zero-filled so P*V sees finite data there.
        for (int p = 0; p < kPagesPerTile; ++p) {
          if ((present >> p) & 1u) continue;
          uint4* zk = reinterpret_cast<uint4*>(sK(s) + p * kBoxBytes);
          uint4* zv = reinterpret_cast<uint4*>(sV(s) + p * kBoxBytes);
          for (int idx = lane; idx < kBoxBytes / 16; idx += 32) zk[idx] = zv[idx] = uint4{};
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&bars[kBarFull + s], __popc(present) * 2u * kBoxBytes);
      __syncwarp();
      if (pid >= 0) {
        const int32_t yk = ((pid * 2 + 0) * a.n_kv_heads + kvh) * kPage;
        const int32_t yv = ((pid * 2 + 1) * a.n_kv_heads + kvh) * kPage;
        tma_load_2d(sK(s) + lane * kBoxBytes, &kvmap, 0, yk, &bars[kBarFull + s]);
        tma_load_2d(sV(s) + lane * kBoxBytes, &kvmap, 0, yv, &bars[kBarFull + s]);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, BF16, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, kD, BF16, false, true);
      const uint32_t tS = tmem + kColS, tO = tmem + kColO;
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = mbar_wait(&bars[kBarQ], 0, a.err);
      auto qk = [&](int j) {
        const int s = j % kStages;
        ok = ok && mbar_wait(&bars[kBarFull + s], (j / kStages) & 1, a.err);
        if (j > 0) ok = ok && mbar_wait(&bars[kBarSFree], (j - 1) & 1, a.err);
        if (!ok) return;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK(s));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          tc_mma_ss(tS, make_sdesc(q_addr + kk * 32, 16, 1024, 2), make_sdesc(k_addr + kk * 32, 16, 1024, 2), idesc_qk,
                    kk > 0 ? 1u : 0u);
        tc_commit(&bars[kBarSFull]);
      };
      auto pv = [&](int j) {
        const int s = j % kStages;
        ok = ok && mbar_wait(&bars[kBarPFull], j & 1, a.err);
        if (!ok) return;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV(s));
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          tc_mma_ss(tO, make_sdesc(p_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024, 2),
                    make_sdesc(v_addr + kk * 16 * 128, 0, 1024, 2), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&bars[kBarODone]);
        tc_commit(&bars[kBarEmpty + s]);
      };
      qk(0);
      for (int j = 1; j < n_kv; ++j) {
        qk(j);
        pv(j - 1);
      }
      pv(n_kv - 1);
    }
    __syncwarp();
  } else {
    // ================= softmax / correction / epilogue: thread = query row = TMEM lane
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int qpos = pos0 + m0 + r;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = warp_wait(&bars[kBarSFull], j & 1, a.err);
      if (!ok) break;
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t t[32];
        tmem_ld32_wait(t_lane + kColS + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(t[i]);
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarSFree]);
      const int kbase = j * kBN;
      if (kbase + kBN - 1 > qpos) {
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (kbase + c > qpos) s[c] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < kBN; ++c) mx = fmaxf(mx, s[c]);
      const float m_new = fmaxf(m_run, mx * a.scale_log2);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = fast_exp2(m_run - m_use);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        s[c] = fast_exp2(fmaf(s[c], a.scale_log2, -m_use));
        sum += s[c];
      }
      l_run = l_run * alpha + sum;
      m_run = m_new;
      if (j > 0) {
        ok = warp_wait(&bars[kBarODone], (j - 1) & 1, a.err);  // PV_{j-1} done: P tile free, O stable
        if (!ok) break;
        tc_fence_after();
      }
      // P row r -> swizzled K-major tile (keys 0-63 in the first atom column, 64-127 in the second)
#pragma unroll
      for (int at = 0; at < 2; ++at)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float* v = s + at * 64 + ch * 8;
          const uint4 w = make_uint4(pack2<BF16>(v[0], v[1]), pack2<BF16>(v[2], v[3]), pack2<BF16>(v[4], v[5]),
                                     pack2<BF16>(v[6], v[7]));
          *reinterpret_cast<uint4*>(sP + at * (kBM * 128) + swz128(r, ch)) = w;
        }
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t t[32];
          tmem_ld32_wait(t_lane + kColO + c * 32, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
          tmem_st16(t_lane + kColO + c * 32, *reinterpret_cast<uint32_t(*)[16]>(&t[0]));
          tmem_st16(t_lane + kColO + c * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&t[16]));
        }
        tc_wait_st();
      }
      fence_proxy_async_smem();  // P stores -> visible to the tensor core
      tc_fence_before();
      mbar_arrive(&bars[kBarPFull]);
    }
    // ---- epilogue
    if (ok) ok = warp_wait(&bars[kBarODone], (n_kv - 1) & 1, a.err);
    if (ok) {
      tc_fence_after();
      float o[kD];
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t t[32];
        tmem_ld32_wait(t_lane + kColO + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = __uint_as_float(t[i]);
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      if (m0 + r < qlen) {
        const int64_t orow = (int64_t(qs) + m0 + r) * a.n_heads + h;
        if (a.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow * kD);
#pragma unroll
          for (int i = 0; i < kD / 4; ++i)
            dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + orow * kD);
#pragma unroll
          for (int i = 0; i < kD / 8; ++i)
            dst[i] = make_uint4(pack2<BF16>(o[8 * i] * inv, o[8 * i + 1] * inv),
                                pack2<BF16>(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                                pack2<BF16>(o[8 * i + 4] * inv, o[8 * i + 5] * inv),
                                pack2<BF16>(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool BF16>
void launch_t(cudaStream_t st, const CUtensorMap& qmap, const CUtensorMap& kvmap, const PrefillArgs& a, int grid) {
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(prefill_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
               "prefill smem attribute");
    configured.fetch_or(bit);
  }
  prefill_kernel<BF16><<<grid, kThreads, kSmemBytes, st>>>(qmap, kvmap, a);
}

}  // namespace

void launch_prefill(cudaStream_t st, const nbl_kv* kv, const void* q, int64_t n_q_rows, const int32_t* q_start,
                    const int32_t* q_len, const int32_t* kv_pos0, const int32_t* page_table, int32_t pt_stride,
                    int n_items, int n_heads, int max_q_len, void* out, int out_dtype, int* err) {
  const auto& c = kv->cfg;
  const bool bf16 = c.dtype == NBL_BF16;
  if (n_q_rows * n_heads >= (int64_t(1) << 31)) fail(NBL_E_INVALID, "prefill: q has more than 2^31 head rows");
  CUtensorMap qmap;
  const cuuint64_t dims[3] = {kD, static_cast<cuuint64_t>(n_heads), static_cast<cuuint64_t>(n_q_rows)};
  const cuuint64_t strides[2] = {kD * 2, static_cast<cuuint64_t>(n_heads) * kD * 2};
  const cuuint32_t box[3] = {kD, 1, kBM};
  encode_tmap(&qmap, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
              const_cast<void*>(q), dims, strides, box);
  PrefillArgs a{};
  a.q_start = q_start;
  a.q_len = q_len;
  a.kv_pos0 = kv_pos0;
  a.page_table = page_table;
  a.out = out;
  a.err = err;
  a.n_pages = c.n_pages;
  a.n_q_rows = n_q_rows;
  a.pt_stride = pt_stride;
  a.out_f32 = out_dtype == NBL_F32;
  a.n_heads = n_heads;
  a.n_kv_heads = c.n_kv_heads;
  a.group = n_heads / c.n_kv_heads;
  a.m_tiles = (max_q_len + kBM - 1) / kBM;
  a.scale_log2 = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
  const int64_t grid = int64_t(n_items) * n_heads * a.m_tiles;
  if (grid > 0x7fffffff) fail(NBL_E_INVALID, "prefill: items * heads * query tiles exceeds the grid limit");
  if (bf16) launch_t<true>(st, qmap, kv->tmap, a, static_cast<int>(grid));
  else launch_t<false>(st, qmap, kv->tmap, a, static_cast<int>(grid));
  check_cuda(cudaGetLastError(), "prefill launch");
}

}  // namespace nbl
