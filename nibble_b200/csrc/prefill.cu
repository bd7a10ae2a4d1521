// Causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMEM), reading K/V from the paged pool.
//
// Replaces Backend::attention for n > 1 (src/backend/backend.h:66-69; the reference's scalar loop is
// src/backend/cpu/ref_ops.cpp:188-214): query row t of an item has position kv_pos0 + t and attends keys
// 0..kv_pos0+t; query head h reads KV head h / G.
//
// Persistent: two CTAs per SM walk the works -- a work is one 128-row query tile for two query heads of the same
// KV group (NH = 2; the heads share every K/V tile staged in shared memory, and an odd group leaves the last pair
// with one head) -- in rounds of gridDim.x consecutive works, CTA c taking work c of even rounds and
// gridDim.x - 1 - c of odd ones, so heavy and light query tiles even out and the works running at one time share
// their K/V in L2. Warps, specialised:
//   warps 0..7   softmax, one warpgroup per head: thread i of a warpgroup owns query row i = TMEM lane i (a warp
//                reaches the lane quarter warp % 4). Per K/V tile it loads its S row (64 fp32) from TMEM in one
//                instruction, masks causally, takes the row max with 3-input max instructions, and keeps a
//                reference max m_ref (log2 domain) that only moves when the tile max exceeds it by more than 2^8, so
//                the O accumulator in TMEM is rescaled rarely; p = 2^(s*scale - m_ref) via ex2.approx (one pair in eight on the FMA
//                pipe) with packed fp32x2 arguments, the row sum with packed adds; P is packed to bf16/fp16 pairs
//                and stored into the first 32 columns of its S region as the A operand of the PV MMA. After a
//                work's last tile it reads O out of TMEM (releasing it to the next work), normalises and stores.
//   warp 8       TMA producer: each work's Q tiles into one of two Q buffers (so the next work's Q loads while the
//                current one runs), then its K/V tiles of 64 keys (4 pages, one 16x64 box each for K and V)
//                through a 3-stage ring that runs on across works; 128-byte swizzle.
//   warp 9       MMA issuer (one thread): S_g = Q_g K_j^T (M=128, N=64, K=64, both operands K-major from shared
//                memory) and O_g += P_g V_j (M=128, N=64, K=64) with P read from TMEM and V used as an MN-major
//                operand straight from the TMA tile, issued per head as PV_g(j), S_g(j+1) so a head's next S never
//                waits for the other head's softmax. MMAs execute in issue order, so S_g(j+1) -- and the next
//                work's S_g(0) -- may overwrite the TMEM columns PV_g(j) read P_g from; a work's first PV, which
//                overwrites O_g, waits until the previous work's epilogue has read O_g.
// Sizing: 320 threads at <= 102 registers, 256 TMEM columns (per head 64 for S/P and 64 for O) and 112 KB of
// shared memory, so two CTAs share an SM: four independent softmax -> MMA -> softmax chains per SM hide each
// other's hand-offs, and per-SM exp throughput (16 ex2 per clock, about 1.6x the tensor time of a 128x64 tile at
// head_dim 64) sets the pace.
//
// Every mbarrier wait is bounded (nbl_device.cuh): a lost completion ends the CTA with kErrTimeout set.
#include <algorithm>
#include <atomic>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

constexpr int kD = 64;
constexpr int kBM = 128;                  // query rows per tile
constexpr int kPage = 16;
constexpr int kQBytes = kBM * kD * 2;     // one Q tile: 16 KB
constexpr int kBoxBytes = kPage * kD * 2; // 2 KB
constexpr float kRescaleThreshold = 8.0f;  // log2 units: p may reach 2^8 before the reference max moves

template <int NH, int BN>
struct Cfg {
  static constexpr int kBN = BN;                       // keys per K/V tile
  static constexpr int kPagesPerTile = BN / kPage;
  static constexpr int kTileBytes = BN * kD * 2;       // one K (or V) tile
  static constexpr int kStages = 3;                    // K/V ring depth
  static constexpr int kThreads = (4 * NH + 2) * 32;
  static constexpr int kWarpTma = 4 * NH, kWarpMma = 4 * NH + 1;
  static constexpr int kCtasPerSm = 2;
  static constexpr uint32_t kTmemCols = NH * (BN + kD) <= 128 ? 128 : (NH * (BN + kD) <= 256 ? 256 : 512);
  static constexpr int kOffQ = 0;                                  // 2 buffers x NH heads x 16 KB
  static constexpr int kOffKV = 2 * NH * kQBytes;
  static constexpr int kOffBar = kOffKV + kStages * 2 * kTileBytes;
  // barrier slots: Q buffers full/free, K/V ring full/empty, per head S full, P full, O done, O drained
  static constexpr int kBarQFull = 0, kBarQFree = 2, kBarFull = 4, kBarEmpty = 4 + kStages,
                       kBarSFull = 4 + 2 * kStages, kBarPFull = kBarSFull + NH, kBarODone = kBarPFull + NH,
                       kBarODrained = kBarODone + NH, kNumBars = kBarODrained + NH;
  static constexpr int kOffTmemSlot = kOffBar + ((kNumBars * 8 + 15) & ~15);
  static constexpr int kSmemBytes = kOffTmemSlot + 16;
  // TMEM columns of head g's S region (P aliases its first BN/2 columns) and O accumulator
  __host__ __device__ static constexpr uint32_t col_s(int g) { return g * BN; }
  __host__ __device__ static constexpr uint32_t col_o(int g) { return NH * BN + g * kD; }
};

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
  int n_heads, n_kv_heads, group, n_hgroups, m_tiles;
  int n_works;  // items x KV heads x head groups x query tiles
  float scale_log2;
};

// One unit of work: a 128-row query tile of up to NH heads of one KV group of one item. Works are numbered with
// the (item, KV head) pair slowest, then query tile (latest first), then head group, so the works a grid-stride
// of CTAs runs at one time share their K/V in L2.
struct Work {
  int kvh, n_g, head0, qlen, pos0, qs, m0, n_kv, n_item_pages;
  const int32_t* pt_row;
  bool valid;
};

// Work w (-1: none) with the per-item fields it reads.
struct WorkItem {
  int w;  // -1: none for this CTA in this round
  int qlen, pos0, qs;
};

__device__ __forceinline__ WorkItem item_fields(const PrefillArgs& a, int w) {
  WorkItem n{w, 0, 0, 0};
  if (w < 0) return n;
  const int item = w / (a.m_tiles * a.n_hgroups) / a.n_kv_heads;
  n.qlen = a.q_len[item];
  n.pos0 = a.kv_pos0[item];
  n.qs = a.q_start[item];
  return n;
}

template <int NH, int BN>
__device__ __forceinline__ Work decode_work(const PrefillArgs& a, const WorkItem& n) {
  Work k{};
  k.valid = false;
  if (n.w < 0) return k;
  const int w = n.w;
  const int per_group = a.m_tiles * a.n_hgroups;
  const int grp = w / per_group;
  const int within = w - grp * per_group;
  const int mt = a.m_tiles - 1 - within / a.n_hgroups;
  const int hg = within % a.n_hgroups;
  const int item = grp / a.n_kv_heads;
  k.kvh = grp - item * a.n_kv_heads;
  const int g0 = NH * hg;
  k.n_g = min(NH, a.group - g0);  // an odd group leaves the last pair with one head
  k.head0 = k.kvh * a.group + g0;
  k.qlen = n.qlen;
  k.pos0 = n.pos0;
  k.qs = n.qs;
  k.m0 = mt * kBM;
  k.valid = k.qlen > 0 && k.m0 < k.qlen;
  if (!k.valid) return k;
  const int64_t kv_len = int64_t(k.pos0) + k.qlen;
  if (k.pos0 < 0 || k.qs < 0 || int64_t(k.qs) + k.qlen > a.n_q_rows || kv_len > int64_t(a.pt_stride) * kPage) {
    flag_error(a.err, kErrLength);
    k.valid = false;
    return k;
  }
  const int kv_end = static_cast<int>(std::min<int64_t>(kv_len, int64_t(k.pos0) + k.m0 + kBM));
  k.n_kv = (kv_end + BN - 1) / BN;
  k.n_item_pages = static_cast<int>((kv_len + kPage - 1) / kPage);
  k.pt_row = a.page_table + int64_t(item) * a.pt_stride;
  return k;
}

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

// 64 consecutive TMEM columns, waiting inside the same asm statement.
__device__ __forceinline__ void tmem_ld64_wait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// 2^x for two arguments on the FMA and integer pipes instead of the SFU (16 ex2 per clock per SM, the softmax's
// bottleneck at head_dim 64). x = j + f with j = round(x) (adding 1.5 * 2^23 rounds to an integer held in the low
// mantissa bits) and f in [-0.5, 0.5]; 2^f is a degree-3 polynomial whose coefficients are this library's own
// minimax fit of relative error on that interval (7.5e-5 evaluated in fp32, well below the bf16 rounding P gets
// anyway); 2^j is added to the exponent field. Arguments are clamped to >= -125 so the exponent never
// underflows: a masked score (-inf) gives 2^-125 ~ 2e-38 instead of 0, which no sum or bf16 product notices.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kC0 = 0.9999280571937561f, kC1 = 0.6932609677314758f, kC2 = 0.2426111251115799f,
                  kC3 = 0.0551716685295105f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x = make_float2(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 j = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(make_float2(kC3, kC3), f, make_float2(kC2, kC2));
  p = __ffma2_rn(p, f, make_float2(kC1, kC1));
  p = __ffma2_rn(p, f, make_float2(kC0, kC0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}
// Score pairs 0, 8, 16, 24 of a row's 32 per tile take exp2_poly2, the rest ex2.approx. Measured on config 3:
// 1 pair in 8 is 1.3 % faster than none; 2 in 8 or more is slower (the per-tile chain is latency-bound, and the
// polynomial's extra instructions lengthen it).
__host__ __device__ constexpr bool poly_pair(int q) { return q % 8 == 0; }

// max(a, b, c) in one instruction (sm_100's three-input max: the row max over 64 scores takes 34 instructions
// instead of 63).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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
  return warp_wait_all(bar, parity, err);
}

template <bool BF16, int NH, int BN>
__global__ void __launch_bounds__(Cfg<NH, BN>::kThreads, Cfg<NH, BN>::kCtasPerSm)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kvmap,
                   const PrefillArgs a) {
  using C = Cfg<NH, BN>;
  constexpr int kBN = C::kBN, kPagesPerTile = C::kPagesPerTile, kTileBytes = C::kTileBytes;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (smem_u32(smem) & 1023u) {  // 128-byte-swizzled tiles need 1024-byte alignment; never expected to trip
    if (threadIdx.x == 0) flag_error(a.err, kErrSmemAlign);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);
  auto sQ = [&](int buf, int g) { return smem + C::kOffQ + (buf * NH + g) * kQBytes; };
  auto sK = [&](int s) { return smem + C::kOffKV + s * 2 * kTileBytes; };
  auto sV = [&](int s) { return smem + C::kOffKV + s * 2 * kTileBytes + kTileBytes; };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars[C::kBarQFull + b], 1);
      mbar_init(&bars[C::kBarQFree + b], 1);
    }
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars[C::kBarFull + s], 1);
      mbar_init(&bars[C::kBarEmpty + s], 1);
    }
    for (int g = 0; g < NH; ++g) {
      mbar_init(&bars[C::kBarSFull + g], 1);
      mbar_init(&bars[C::kBarPFull + g], 128);
      mbar_init(&bars[C::kBarODone + g], 1);
      mbar_init(&bars[C::kBarODrained + g], 128);
    }
    fence_barrier_init();
  }
  if (warp == C::kWarpMma) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Rounds of gridDim.x consecutive works; CTA c takes work c of even rounds and gridDim.x - 1 - c of odd ones
  // (a snake order: the heavy and light query tiles of a round even out over two rounds), -1 past the end.
  auto work_of = [](int w0, int n_works) {
    const int w = w0 + (((w0 / static_cast<int>(gridDim.x)) & 1) ? static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x)
                                                                  : static_cast<int>(blockIdx.x));
    return w < n_works ? w : -1;
  };
  // Every role walks the same works (in the order work_of gives) and skips the same invalid ones, so the
  // barrier phase counts below agree: lw = this CTA's valid works so far (Q buffer lw & 1, its use lw >> 1),
  // kt = K/V tiles so far (ring stage kt % kStages), and per head the tiles and works that head took part in.
  if (warp == C::kWarpTma) {
    // ================= TMA producer: Q of each work into the free Q buffer, then its K/V tiles into the ring
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kvmap);
    }
    int lw = 0, kt = 0;
    bool ok = true;
    for (int w0 = 0; w0 < a.n_works && ok; w0 += gridDim.x) {
      const Work wk = decode_work<NH, BN>(a, item_fields(a, work_of(w0, a.n_works)));
      if (!wk.valid) continue;
      const int qb = lw & 1, use = lw >> 1;
      if (use > 0 && !warp_wait(&bars[C::kBarQFree + qb], (use - 1) & 1, a.err)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[C::kBarQFull + qb], wk.n_g * kQBytes);
        for (int g = 0; g < wk.n_g; ++g)
          tma_load_3d(sQ(qb, g), &qmap, 0, wk.head0 + g, wk.qs + wk.m0, &bars[C::kBarQFull + qb]);
      }
      for (int j = 0; j < wk.n_kv; ++j, ++kt) {
        const int s = kt % C::kStages;
        if (kt >= C::kStages && !warp_wait(&bars[C::kBarEmpty + s], ((kt / C::kStages) & 1) ^ 1, a.err)) {
          ok = false;
          break;
        }
        const int pg = j * kPagesPerTile + lane;
        int32_t pid = -1;
        if (lane < kPagesPerTile && pg < wk.n_item_pages) {
          pid = wk.pt_row[pg];
          if (pid < 0 || pid >= a.n_pages) {
            flag_error(a.err, kErrPageId);
            pid = -1;
          }
        }
        constexpr uint32_t kAllPages = (1u << kPagesPerTile) - 1u;
        const uint32_t present = __ballot_sync(0xffffffffu, pid >= 0) & kAllPages;
        if (present != kAllPages) {
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
        if (lane == 0) mbar_arrive_expect_tx(&bars[C::kBarFull + s], __popc(present) * 2u * kBoxBytes);
        __syncwarp();
        if (pid >= 0) {
          const int32_t yk = ((pid * 2 + 0) * a.n_kv_heads + wk.kvh) * kPage;
          const int32_t yv = ((pid * 2 + 1) * a.n_kv_heads + wk.kvh) * kPage;
          tma_load_2d(sK(s) + lane * kBoxBytes, &kvmap, 0, yk, &bars[C::kBarFull + s]);
          tma_load_2d(sV(s) + lane * kBoxBytes, &kvmap, 0, yv, &bars[C::kBarFull + s]);
        }
      }
      ++lw;
    }
  } else if (warp == C::kWarpMma) {
    // ================= MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, BF16, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, kD, BF16, false, true);
      int lw = 0, kt = 0;
      int h_tiles[NH], h_works[NH];
#pragma unroll
      for (int g = 0; g < NH; ++g) h_tiles[g] = h_works[g] = 0;
      // S_g = Q_g K^T for head g from Q buffer qb and ring stage s (signals S_g full).
      auto qk = [&](int g, int qb, int s) {
        const uint32_t q_addr = smem_u32(sQ(qb, g)), k_addr = smem_u32(sK(s));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          tc_mma_ss(tmem + C::col_s(g), make_sdesc(q_addr + kk * 32, 16, 1024, 2),
                    make_sdesc(k_addr + kk * 32, 16, 1024, 2), idesc_qk, kk > 0 ? 1u : 0u);
        tc_commit(&bars[C::kBarSFull + g]);
      };
      auto kv_ready = [&](int t) -> bool {
        if (!mbar_wait(&bars[C::kBarFull + t % C::kStages], (t / C::kStages) & 1, a.err)) return false;
        tc_fence_after();
        return true;
      };
      bool ok = true;
      for (int w0 = 0; w0 < a.n_works && ok; w0 += gridDim.x) {
        const Work wk = decode_work<NH, BN>(a, item_fields(a, work_of(w0, a.n_works)));
        if (!wk.valid) continue;
        const int qb = lw & 1;
        ok = mbar_wait(&bars[C::kBarQFull + qb], (lw >> 1) & 1, a.err) && kv_ready(kt);
        if (!ok) break;
        // S_g(0) may overwrite the columns the previous work's last PV_g read P from: MMAs run in issue order.
        for (int g = 0; g < wk.n_g; ++g) qk(g, qb, kt % C::kStages);
        for (int j = 0; j < wk.n_kv && ok; ++j, ++kt) {
          const bool more = j + 1 < wk.n_kv;
          if (more) ok = kv_ready(kt + 1);
          for (int g = 0; g < wk.n_g && ok; ++g) {
            // O_g += P_g V_j once head g's softmax has written P_g; the work's first PV overwrites O_g, so it
            // also waits for the previous work's epilogue to have read O_g out.
            if (j == 0 && h_works[g] > 0) ok = mbar_wait(&bars[C::kBarODrained + g], (h_works[g] - 1) & 1, a.err);
            if (ok) ok = mbar_wait(&bars[C::kBarPFull + g], h_tiles[g] & 1, a.err);
            if (!ok) break;
            ++h_tiles[g];
            tc_fence_after();
            const uint32_t v_addr = smem_u32(sV(kt % C::kStages));
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk)
              tc_mma_ts(tmem + C::col_o(g), tmem + C::col_s(g) + kk * 8,
                        make_sdesc(v_addr + kk * 16 * 128, 0, 1024, 2), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
            if (more) qk(g, qb, (kt + 1) % C::kStages);
          }
          tc_commit(&bars[C::kBarEmpty + kt % C::kStages]);  // K and V of this stage fully consumed
        }
        if (!ok) break;
        tc_commit(&bars[C::kBarQFree + qb]);  // every QK of this work has read its Q tiles
        for (int g = 0; g < wk.n_g; ++g) {
          tc_commit(&bars[C::kBarODone + g]);
          ++h_works[g];
        }
        ++lw;
      }
    }
    __syncwarp();
  } else {
    // ================= softmax / correction / epilogue of head g: thread = query row = TMEM lane
    const int g = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + C::col_s(g) + lane_off, tO = tmem + C::col_o(g) + lane_off;
    const float scale = a.scale_log2;
    const float2 scale2 = make_float2(scale, scale);
    int h_tiles = 0, h_works = 0;
    bool ok = true;
    for (int w0 = 0; w0 < a.n_works && ok; w0 += gridDim.x) {
      const Work wk = decode_work<NH, BN>(a, item_fields(a, work_of(w0, a.n_works)));
      if (!wk.valid || g >= wk.n_g) continue;
      const int qpos = wk.pos0 + wk.m0 + r;
      float m_ref = -INFINITY, l_run = 0.f;
      for (int j = 0; j < wk.n_kv; ++j, ++h_tiles) {
        ok = warp_wait(&bars[C::kBarSFull + g], h_tiles & 1, a.err);
        if (!ok) break;
        tc_fence_after();
        uint32_t t[kBN];
        static_assert(kBN == 64, "one 64-column TMEM load per S row");
        tmem_ld64_wait(tS, t);
        const int kbase = j * kBN;
        if (kbase + kBN - 1 > qpos) {  // the tile holds keys past this row's position
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (kbase + c > qpos) t[c] = __float_as_uint(-INFINITY);
        }
        // four chains of 3-input maxima over 16 columns each (c = i, i+4, ..., i+60)
        float mx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          mx[i] = fmax3(__uint_as_float(t[i]), __uint_as_float(t[i + 4]), __uint_as_float(t[i + 8]));
#pragma unroll
          for (int c = 12; c < 60; c += 8)
            mx[i] = fmax3(mx[i], __uint_as_float(t[c + i]), __uint_as_float(t[c + 4 + i]));
          mx[i] = fmaxf(mx[i], __uint_as_float(t[60 + i]));
        }
        const float m_tile = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * scale;
        const bool need = m_tile > m_ref + kRescaleThreshold;  // false for m_tile = -inf
        const float m_new = need ? m_tile : m_ref;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = need ? fast_exp2(m_ref - m_use) : 1.f;  // m_ref = -inf gives 0
        const float2 neg_m2 = make_float2(-m_use, -m_use);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        // p = 2^(s*scale - m), packed in place: pair c/2 goes to t[c/2] (already consumed)
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(t[c]), __uint_as_float(t[c + 1])), scale2, neg_m2);
          const float2 e = poly_pair(c >> 1) ? exp2_poly2(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
          acc[(c >> 1) & 3] = __fadd2_rn(acc[(c >> 1) & 3], e);
          t[c >> 1] = pack2<BF16>(e.x, e.y);
        }
        const float2 sum2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
        l_run = l_run * alpha + (sum2.x + sum2.y);
        m_ref = m_new;
        // P into the first BN/2 columns of this head's S region (the PV MMA's A operand)
        tmem_st32(tS, *reinterpret_cast<uint32_t(*)[32]>(&t[0]));
        // S_g(j) completing implies PV_g(j-1) completed (MMAs execute in order), so O_g is stable here.
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32_wait(tO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[C::kBarPFull + g]);
      }
      if (!ok) break;
      // ---- epilogue: O_g out of TMEM (then the next work's first PV may overwrite it), normalise, store
      ok = warp_wait(&bars[C::kBarODone + g], h_works & 1, a.err);
      if (!ok) break;
      ++h_works;
      tc_fence_after();
      uint32_t o[kD];
      tmem_ld32_wait(tO, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32_wait(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tc_fence_before();
      mbar_arrive(&bars[C::kBarODrained + g]);
      if (wk.m0 + r < wk.qlen) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        const int64_t orow = (int64_t(wk.qs) + wk.m0 + r) * a.n_heads + wk.head0 + g;
        if (a.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow * kD);
#pragma unroll
          for (int i = 0; i < kD / 4; ++i)
            dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                 __uint_as_float(o[4 * i + 2]) * inv, __uint_as_float(o[4 * i + 3]) * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + orow * kD);
#pragma unroll
          for (int i = 0; i < kD / 8; ++i)
            dst[i] = make_uint4(pack2<BF16>(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                                pack2<BF16>(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                                pack2<BF16>(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                                pack2<BF16>(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <bool BF16, int NH, int BN>
void launch_t(cudaStream_t st, const CUtensorMap& qmap, const CUtensorMap& kvmap, const PrefillArgs& a, int grid) {
  using C = Cfg<NH, BN>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(prefill_kernel<BF16, NH, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::kSmemBytes),
               "prefill smem attribute");
    configured.fetch_or(bit);
  }
  prefill_kernel<BF16, NH, BN><<<grid, C::kThreads, C::kSmemBytes, st>>>(qmap, kvmap, a);
}

}  // namespace

void launch_prefill(cudaStream_t st, const nbl_kv* kv, const void* q, int64_t n_q_rows, const int32_t* q_start,
                    const int32_t* q_len, const int32_t* kv_pos0, const int32_t* page_table, int32_t pt_stride,
                    int n_items, int n_heads, int max_q_len, void* out, int out_dtype, int* err) {
  constexpr int NH = 2, BN = 64;  // heads per CTA, keys per K/V tile (see the file comment)
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
  a.n_hgroups = (a.group + NH - 1) / NH;
  a.m_tiles = (max_q_len + kBM - 1) / kBM;
  a.scale_log2 = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
  const int64_t works = int64_t(n_items) * c.n_kv_heads * a.n_hgroups * a.m_tiles;
  if (works > 0x7fffffff) fail(NBL_E_INVALID, "prefill: items * heads * query tiles exceeds 2^31 works");
  a.n_works = static_cast<int>(works);
  // persistent: Cfg::kCtasPerSm CTAs per SM walk the works with a grid stride
  static const int sms = [] {
    int dev = 0, n = 148;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "SM count");
    return n;
  }();
  const int grid = static_cast<int>(std::min<int64_t>(works, int64_t(sms) * Cfg<NH, BN>::kCtasPerSm));
  if (bf16) launch_t<true, NH, BN>(st, qmap, kv->tmap, a, grid);
  else launch_t<false, NH, BN>(st, qmap, kv->tmap, a, grid);
  check_cuda(cudaGetLastError(), "prefill launch");
}

}  // namespace nbl
