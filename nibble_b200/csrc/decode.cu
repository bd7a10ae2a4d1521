// Split-K flash-decode over the paged fp16 K/V pool, plus the log-sum-exp merge of partial results.
//
// Replaces Backend::attention with n = 1 (src/backend/backend.h:66-69), which the reference runs once per layer
// per generated token (src/model/transformer.cpp:201, src/nibble.cpp:212) as a scalar/AVX2 loop over the whole
// fp32 cache (src/backend/cpu/ref_ops.cpp:188-214, src/backend/cpu/simd/ops.cpp:104-139).
//
// Work decomposition. One CTA per (row, KV head, split): a row is one (sequence, layer) query, the CTA serves
// all G = n_heads / n_kv_heads query heads of its KV head, so each K/V byte is read from HBM once. A split is a
// contiguous range of pages. Inside the CTA the 4 warps take the split's 2-page chunks round-robin; each warp
// owns a private 3-stage ring in shared memory filled by TMA (one 16x64 box per page for K and for V, 128-byte
// swizzle) and keeps its own online-softmax state, so the main loop has no CTA-wide barrier. The warps' states
// are merged through shared memory at the end; splits are merged by the last split of each (row, KV head) to
// finish (an arrival counter per pair), or by lse_merge_kernel when the caller has no counters.
//
// Page ids are read ahead: the first three chunks' ids by six lanes at once, before q is loaded, so a CTA's first
// K/V loads issue after one page-table latency; in the loop, the ids of the chunk a stage takes next are read at
// the top of the iteration and used at its end.
//
// Arithmetic. Scores S^T[token][head] = K * Q^T and O^T[dim][head] = V^T * P^T run on the tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation). K and V are fp16 in the pool, so they are exact
// operands; q (pre-scaled by log2(e)/sqrt(64)) and p are split into fp16 hi + lo parts (x = hi + lo to ~2^-22
// relative) and both halves are accumulated, which keeps the result within ~1e-6 of fp32 arithmetic. The
// softmax runs in the log2 domain with exp2f.
#include <algorithm>
#include <atomic>

#include "nbl_device.cuh"
#include "nbl_internal.h"

namespace nbl {
namespace {

constexpr int kD = 64;              // head_dim
constexpr int kPage = 16;           // tokens per page
constexpr int kWarps = 4;           // warps per CTA
constexpr int kStages = 3;          // ring depth per warp
constexpr int kChunkPages = 2;      // pages per stage
constexpr int kChunkTok = kChunkPages * kPage;               // 32 tokens
constexpr int kBoxBytes = kPage * kD * 2;                    // one page of K (or V) for one KV head: 2 KB
constexpr int kStageBytes = 2 * kChunkPages * kBoxBytes;     // K pages then V pages: 8 KB
constexpr int kRingBytes = kWarps * kStages * kStageBytes;   // 96 KB
constexpr int kPBytes = 2 * kChunkTok * 8 * 2;               // P^T hi and lo, [32 tokens][8 heads] fp16: 1 KB
constexpr int kSmemBytes = 1024 /*alignment slack*/ + kRingBytes + kWarps * kPBytes + kWarps * kStages * 8;
constexpr int kCtasPerSm = 2;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The cross-rank exchange fused into the decode (world > 0): a (row, KV head)'s final (O, lse) is stored straight
// into slot `rank` of the current epoch's half of every rank's receive buffer ([2][world][part] floats, part =
// rows * heads * 64 outputs followed by rows * heads lse, the layout nbl_lse_exchange_peers uses), over NVLink for
// the other ranks; the grid's last finalising CTA then raises this rank's flag word on every rank. sync: [0] the
// last epoch this rank pushed, [1] finalised (row, KV head) pairs of the current launch (0 between launches).
struct PeerOut {
  float* recv[kMaxPeers];
  uint32_t* flags[kMaxPeers];
  uint32_t* sync;
  int world, rank;  // world 0: no exchange, results go to out / lse
  int64_t part;
};

struct DecodeArgs {
  const float* q;
  const int32_t* page_table;
  const int32_t* seq_lens;
  float* out;
  float* lse;
  float* part_o;    // [n_splits, n_rows, n_heads, 64] when n_splits > 1
  float* part_lse;  // [n_splits, n_rows, n_heads]
  unsigned* counts; // [n_rows * n_kv_heads] arrival counters, all 0 between launches; NULL: lse_merge_kernel merges
  int* err;
  int64_t n_pages;
  int32_t pt_stride;
  int n_rows, n_heads, n_kv_heads;
  int n_splits, pages_per_split;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  PeerOut px;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) { return fmaxf(a, fmaxf(b, c)); }

template <int G>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
    decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x % a.n_splits;
  const int rest = blockIdx.x / a.n_splits;
  const int kvh = rest % a.n_kv_heads;
  const int row = rest / a.n_kv_heads;

  uint8_t* ring = smem + warp * kStages * kStageBytes;
  uint8_t* pbuf = smem + kRingBytes + warp * kPBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRingBytes + kWarps * kPBytes) + warp * kStages;

  // ---- this split's page range
  int len = a.seq_lens[row];
  const int max_len = a.pt_stride * kPage;
  if (len < 0 || len > max_len) {
    if (threadIdx.x == 0) flag_error(a.err, kErrLength);
    len = len < 0 ? 0 : max_len;
  }
  const int row_pages = (len + kPage - 1) / kPage;
  const int p_begin = split * a.pages_per_split;
  const int p_end = min(row_pages, p_begin + a.pages_per_split);
  const int n_chunks = p_end > p_begin ? (p_end - p_begin + kChunkPages - 1) / kChunkPages : 0;
  const int my_n = n_chunks > warp ? (n_chunks - warp + kWarps - 1) / kWarps : 0;
  const int32_t* pt_row = a.page_table + int64_t(row) * a.pt_stride;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmap);
  }
  __syncwarp();

  const uint64_t policy = policy_evict_first();
  static_assert(kChunkPages == 2, "a chunk's page ids travel as two lanes' values");
  // Page id of page j of this warp's chunk i, read by one lane; -1 past the split (never loaded).
  auto chunk_pid = [&](int i, int j) -> int32_t {
    const int pg = p_begin + (warp + kWarps * i) * kChunkPages + j;
    return i < my_n && pg < p_end ? pt_row[pg] : -1;
  };
  // loaded: bit 2 * stage + j set when page j of the chunk in ring stage `stage` was loaded (identical in every
  // lane; tokens of pages not loaded are masked).
  uint32_t loaded = 0;
  // Loads chunk i of this warp into ring stage `stage` given its page ids (all lanes call it; lane 0 issues).
  // Pages whose id is out of range are not loaded and flag the error word.
  auto issue = [&](int i, int stage, int32_t pid0, int32_t pid1) {
    const int pg0 = p_begin + (warp + kWarps * i) * kChunkPages;
    const int npg = min(kChunkPages, p_end - pg0);
    const bool ok0 = pid0 >= 0 && pid0 < a.n_pages;
    const bool ok1 = npg > 1 && pid1 >= 0 && pid1 < a.n_pages;
    loaded = (loaded & ~(3u << (2 * stage))) | ((ok0 ? 1u : 0u) << (2 * stage)) | ((ok1 ? 2u : 0u) << (2 * stage));
    if (lane != 0) return;
    if (!ok0 || (npg > 1 && !ok1)) flag_error(a.err, kErrPageId);
    uint8_t* st = ring + stage * kStageBytes;
    mbar_arrive_expect_tx(&bars[stage], (int(ok0) + int(ok1)) * 2u * kBoxBytes);
    if (ok0) {
      tma_load_2d_hint(st, &tmap, 0, ((pid0 * 2 + 0) * a.n_kv_heads + kvh) * kPage, &bars[stage], policy);
      tma_load_2d_hint(st + kChunkPages * kBoxBytes, &tmap, 0, ((pid0 * 2 + 1) * a.n_kv_heads + kvh) * kPage,
                       &bars[stage], policy);
    }
    if (ok1) {
      tma_load_2d_hint(st + kBoxBytes, &tmap, 0, ((pid1 * 2 + 0) * a.n_kv_heads + kvh) * kPage, &bars[stage], policy);
      tma_load_2d_hint(st + (kChunkPages + 1) * kBoxBytes, &tmap, 0, ((pid1 * 2 + 1) * a.n_kv_heads + kvh) * kPage,
                       &bars[stage], policy);
    }
  };
  // The first kStages chunks: lane 2c + j reads page j of chunk c, so all their loads issue after one page-table
  // latency, before q is read (q's load latency overlaps theirs).
  {
    const int32_t pf = lane < 2 * kStages ? chunk_pid(lane >> 1, lane & 1) : -1;
    for (int i = 0; i < min(kStages, my_n); ++i)
      issue(i, i, __shfl_sync(0xffffffffu, pf, 2 * i), __shfl_sync(0xffffffffu, pf, 2 * i + 1));
  }

  // ---- Q^T as the B operand of S^T = K Q^T: lane holds head n = lane/4, dims 16ks + 2(lane%4) + {0,1} (+8)
  uint32_t qh[4][2], ql[4][2];
  {
    const int n = lane >> 2;
    const float* qrow = a.q + (int64_t(row) * a.n_heads + int64_t(kvh) * G + (n < G ? n : 0)) * kD;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int d = 16 * ks + 2 * (lane & 3) + 8 * hf;
        const float x0 = n < G ? qrow[d] * a.scale_log2 : 0.f;
        const float x1 = n < G ? qrow[d + 1] * a.scale_log2 : 0.f;
        const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
        qh[ks][hf] = pack_half2(h0, h1);
        ql[ks][hf] = pack_half2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
      }
  }

  float o[4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int c = 0; c < 4; ++c) o[mt][c] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // heads 2(lane%4) and 2(lane%4)+1
  int done = 0;  // chunks whose loads have completed

  for (int i = 0; i < my_n; ++i) {
    const int stage = i % kStages;
    const bool ok = warp_wait_all(&bars[stage], (i / kStages) & 1, a.err);
    if (!ok) break;
    done = i + 1;
    const int pg0 = p_begin + (warp + kWarps * i) * kChunkPages;
    const int npg = min(kChunkPages, p_end - pg0);
    const int tok0 = pg0 * kPage;
    // page ids of the chunk this stage takes next, read now and used at the end of the iteration
    const int32_t nxt = lane < kChunkPages ? chunk_pid(i + kStages, lane) : -1;
    // valid-token mask: inside the sequence, on a loaded page
    uint32_t vmask = 0;
    for (int j = 0; j < npg; ++j) {
      if (!((loaded >> (2 * stage + j)) & 1u)) continue;
      const int nv = min(kPage, len - (tok0 + j * kPage));
      if (nv > 0) vmask |= (nv >= 32 ? 0xffffffffu : ((1u << nv) - 1u)) << (j * kPage);
    }
    uint8_t* kst = ring + stage * kStageBytes;
    uint8_t* vst = kst + kChunkPages * kBoxBytes;
    if (vmask != 0xffffffffu) {
      // Zero the V rows of masked tokens: p = 0 there, and 0 * (stale non-finite data) would poison O.
      for (int idx = lane; idx < kChunkTok * 8; idx += 32)
        if (!((vmask >> (idx >> 3)) & 1u)) *reinterpret_cast<uint4*>(vst + (idx >> 3) * 128 + (idx & 7) * 16) = uint4{};
      __syncwarp();
    }
    const uint32_t kaddr = smem_u32(kst), vaddr = smem_u32(vst);

    // ---- S^T[32 tokens][8 heads] = K Q^T (two 16-token m-tiles)
    float s[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int c = 0; c < 4; ++c) s[mt][c] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int mi = lane >> 3;
        const int tok = 16 * mt + (lane & 7) + 8 * (mi & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kaddr + swz128(tok, 2 * ks + (mi >> 1)), a0, a1, a2, a3);
        mma_f16_16816(s[mt], a0, a1, a2, a3, qh[ks][0], qh[ks][1]);
        mma_f16_16816(s[mt], a0, a1, a2, a3, ql[ks][0], ql[ks][1]);
      }
    }
    // lane's tokens: 16mt + lane/4 (c0, c1) and +8 (c2, c3); heads 2(lane%4) (c0, c2) and +1 (c1, c3)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int ta = 16 * mt + (lane >> 2);
      if (!((vmask >> ta) & 1u)) s[mt][0] = s[mt][1] = -INFINITY;
      if (!((vmask >> (ta + 8)) & 1u)) s[mt][2] = s[mt][3] = -INFINITY;
    }
    float mx0 = fmaxf(fmax3(s[0][0], s[0][2], s[1][0]), s[1][2]);
    float mx1 = fmaxf(fmax3(s[0][1], s[0][3], s[1][1]), s[1][3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m_run[0] - mu0), al1 = exp2f(m_run[1] - mu1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      s[mt][0] = exp2f(s[mt][0] - mu0);
      s[mt][1] = exp2f(s[mt][1] - mu1);
      s[mt][2] = exp2f(s[mt][2] - mu0);
      s[mt][3] = exp2f(s[mt][3] - mu1);
      ps0 += s[mt][0] + s[mt][2];
      ps1 += s[mt][1] + s[mt][3];
    }
    l_run[0] = l_run[0] * al0 + ps0;
    l_run[1] = l_run[1] * al1 + ps1;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      o[mt][0] *= al0;
      o[mt][1] *= al1;
      o[mt][2] *= al0;
      o[mt][3] *= al1;
    }
    // ---- P^T [token][head] as fp16 hi and lo
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int tok = 16 * mt + (lane >> 2) + 8 * hf;
        const float p0 = s[mt][2 * hf], p1 = s[mt][2 * hf + 1];
        const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
        const uint32_t off = tok * 16 + (lane & 3) * 4;
        *reinterpret_cast<uint32_t*>(pbuf + off) = pack_half2(h0, h1);
        *reinterpret_cast<uint32_t*>(pbuf + kPBytes / 2 + off) =
            pack_half2(__float2half_rn(p0 - __half2float(h0)), __float2half_rn(p1 - __half2float(h1)));
      }
    __syncwarp();
    // ---- O^T[64 dims][8 heads] += V^T P^T
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t bh0, bh1, bl0, bl1;
      {
        const int mi = lane >> 3;
        const int tok = 16 * ks + 8 * (mi & 1) + (lane & 7);
        ldsm_x4_t(smem_u32(pbuf + (mi >> 1) * (kPBytes / 2) + tok * 16), bh0, bh1, bl0, bl1);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int mi = lane >> 3;
        const int tok = 16 * ks + (lane & 7) + 8 * (mi >> 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vaddr + swz128(tok, 2 * mt + (mi & 1)), a0, a1, a2, a3);
        mma_f16_16816(o[mt], a0, a1, a2, a3, bh0, bh1);
        mma_f16_16816(o[mt], a0, a1, a2, a3, bl0, bl1);
      }
    }
    __syncwarp();
    if (i + kStages < my_n) {
      const int32_t p0 = __shfl_sync(0xffffffffu, nxt, 0), p1 = __shfl_sync(0xffffffffu, nxt, 1);
      if (lane == 0) fence_proxy_async_smem();  // order this warp's generic smem accesses before the next async write
      issue(i + kStages, stage, p0, p1);
    }
  }
  // After a timed-out wait, drain the loads still in flight (chunks done .. done+kStages-1; bounded) before the
  // ring is reused.
  if (done < my_n)
    for (int i = done; i < min(my_n, done + kStages); ++i) mbar_wait(&bars[i % kStages], (i / kStages) & 1, a.err);

  // ---- per-warp totals, then merge the 4 warps through shared memory
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
    l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
  }
  __syncthreads();  // every warp is past its ring: reuse it for the merge
  float* mrg = reinterpret_cast<float*>(smem);
  float* w_m = mrg + warp * (16 + kD * 8);
  float* w_l = w_m + 8;
  float* w_o = w_m + 16;  // [64 dims][8 heads]
  if (lane < 4) {
    w_m[2 * lane] = m_run[0];
    w_m[2 * lane + 1] = m_run[1];
    w_l[2 * lane] = l_run[0];
    w_l[2 * lane + 1] = l_run[1];
  }
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int dim = 16 * mt + (lane >> 2) + 8 * (c >> 1);
      const int head = 2 * (lane & 3) + (c & 1);
      w_o[dim * 8 + head] = o[mt][c];
    }
  __syncthreads();
  // A finished (row, head) output: to out / lse, or with the exchange fused in, into every rank's receive buffer.
  // The epoch is read before this CTA is counted below, so before the last CTA advances it.
  const uint32_t epoch = a.px.world > 0 ? a.px.sync[0] + 1u : 0u;
  auto finish = [&](int64_t r, int d, float val, float lse_nat) {
    if (a.px.world == 0) {
      a.out[r * kD + d] = val;
      if (d == 0 && a.lse) a.lse[r] = lse_nat;
      return;
    }
    const int64_t slot = (int64_t(epoch & 1u) * a.px.world + a.px.rank) * a.px.part;
    const int64_t n_out = int64_t(a.n_rows) * a.n_heads * kD;
    for (int p = 0; p < a.px.world; ++p) {
      a.px.recv[p][slot + r * kD + d] = val;
      if (d == 0) a.px.recv[p][slot + n_out + r] = lse_nat;
    }
  };
  for (int idx = threadIdx.x; idx < G * kD; idx += kWarps * 32) {
    const int g = idx / kD, d = idx % kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, mrg[w * (16 + kD * 8) + g]);
    float L = 0.f, O = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* wb = mrg + w * (16 + kD * 8);
        const float sc = exp2f(wb[g] - mx);  // 0 for warps that saw no token
        L += sc * wb[8 + g];
        O += sc * wb[16 + d * 8 + g];
      }
    }
    const int head = kvh * G + g;
    const float val = L > 0.f ? O / L : 0.f;
    const float lse_nat = L > 0.f ? (mx + __log2f(L)) * kLn2 : -INFINITY;
    if (a.n_splits == 1) {
      finish(int64_t(row) * a.n_heads + head, d, val, lse_nat);
    } else {
      const int64_t prow = (int64_t(split) * a.n_rows + row) * a.n_heads + head;
      a.part_o[prow * kD + d] = val;
      if (d == 0) a.part_lse[prow] = lse_nat;
    }
  }
  if (a.n_splits > 1) {
    if (a.counts == nullptr) return;  // lse_merge_kernel merges the splits
    // The last split of this (row, KV head) to finish merges all splits' partials (as lse_merge_kernel does), so no
    // second launch waits for the whole grid. The arrival counter wraps back to 0 on the last arrival (atomicInc),
    // ready for the next launch; every CTA reaches this point, whatever happened in its main loop.
    __shared__ int last;
    __threadfence();  // this CTA's partials are visible device-wide before its arrival is counted
    __syncthreads();
    if (threadIdx.x == 0) last = atomicInc(&a.counts[rest], static_cast<unsigned>(a.n_splits - 1)) ==
                                 static_cast<unsigned>(a.n_splits - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < G * kD; idx += kWarps * 32) {
      const int g = idx / kD, d = idx % kD;
      const int64_t r = int64_t(row) * a.n_heads + kvh * G + g;
      const int64_t lse_stride = int64_t(a.n_rows) * a.n_heads;
      float mx = -INFINITY;
      for (int p = 0; p < a.n_splits; ++p) mx = fmaxf(mx, __ldcg(a.part_lse + p * lse_stride + r));
      float W = 0.f, O = 0.f;
      if (mx != -INFINITY) {
        for (int p = 0; p < a.n_splits; ++p) {
          const float w = expf(__ldcg(a.part_lse + p * lse_stride + r) - mx);
          W += w;
          if (w > 0.f) O += w * __ldcg(a.part_o + (p * lse_stride + r) * kD + d);
        }
      }
      finish(r, d, W > 0.f ? O / W : 0.f, W > 0.f ? mx + logf(W) : -INFINITY);
    }
  }
  if (a.px.world == 0) return;
  // This CTA finalised its (row, KV head): count it; the grid's last one publishes the epoch to every rank once
  // every finalising CTA's peer stores are fenced at system scope.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned units = static_cast<unsigned>(a.n_rows) * static_cast<unsigned>(a.n_kv_heads);
    if (atomicAdd(&a.px.sync[1], 1u) == units - 1u) {
      __threadfence_system();
      a.px.sync[0] = epoch;
      a.px.sync[1] = 0u;
      for (int p = 0; p < a.px.world; ++p) st_release_sys(a.px.flags[p] + a.px.rank, epoch);
    }
  }
}

// One CTA per group of rows; a thread per head dimension. part_o [n_parts, rows, D], part_lse [n_parts, rows].
// Part p's outputs start at part_o + p * o_stride ([rows, head_dim]) and its lse at part_lse + p * lse_stride.
__device__ __forceinline__ void lse_merge_rows(const float* __restrict__ part_o, int64_t o_stride,
                                               const float* __restrict__ part_lse, int64_t lse_stride, int n_parts,
                                               int64_t rows, int head_dim, float* __restrict__ out,
                                               float* __restrict__ lse);
__global__ void lse_merge_kernel(const float* __restrict__ part_o, int64_t o_stride, const float* __restrict__ part_lse,
                                 int64_t lse_stride, int n_parts, int64_t rows, int head_dim, float* __restrict__ out,
                                 float* __restrict__ lse) {
  lse_merge_rows(part_o, o_stride, part_lse, lse_stride, n_parts, rows, head_dim, out, lse);
}

// ---- the long-context exchange over peer memory (nbl_lse_exchange_peers)
// Every rank's receive buffer holds [2 (epoch parity)][world][part] floats, a part being one rank's packed
// [rows * D outputs | rows lse]; every rank's flag words hold [world] epochs. Rank r's push writes its part into
// slot r of the epoch's half of every rank's buffer, then -- once every CTA's stores are fenced -- stores the epoch
// into word r of every rank's flags (release, system scope). A rank merges after it has seen the epoch (acquire)
// in all words. Two halves suffice: a rank pushes epoch e + 1 only after its own merge of e, which needed every
// rank's push of e, so no rank can overwrite a half another rank may still be reading.
struct PeerBufs {
  float* recv[kMaxPeers];
  uint32_t* flags[kMaxPeers];
};

// sync[0] = this rank's last pushed epoch, sync[1] = CTAs done with the current push (back to 0 after it).
// VEC: part % 4 == 0 and 16-byte-aligned buffers, so every store over NVLink is 16 bytes.
template <bool VEC>
__global__ void peer_push_kernel(const float* __restrict__ send, int64_t part, PeerBufs px, int world, int rank,
                                 uint32_t* sync) {
  const uint32_t e = sync[0] + 1u;  // read by every CTA before the last one (which waits for all) updates it
  const int64_t off = (int64_t(e & 1u) * world + rank) * part;
  if constexpr (VEC) {
    const int64_t n4 = part / 4;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(send)[i];
      for (int p = 0; p < world; ++p) reinterpret_cast<float4*>(px.recv[p] + off)[i] = v;
    }
  } else {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < part; i += int64_t(gridDim.x) * blockDim.x) {
      const float v = send[i];
      for (int p = 0; p < world; ++p) px.recv[p][off + i] = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&sync[1], 1u);
    if (prev == gridDim.x - 1) {  // the last CTA: every part store of this rank is fenced
      __threadfence_system();
      sync[0] = e;
      sync[1] = 0u;
      for (int p = 0; p < world; ++p) st_release_sys(px.flags[p] + rank, e);
    }
  }
}

// Waits (bounded by kWaitLimitNs of %globaltimer; on timeout flags kErrTimeout and writes nothing) until every
// rank's epoch has arrived in this rank's flags, then merges the world parts of that epoch.
__global__ void peer_merge_kernel(const float* __restrict__ recv, const uint32_t* flags, const uint32_t* sync,
                                  int world, int64_t part, int64_t rows, int head_dim, float* __restrict__ out,
                                  float* __restrict__ lse, int* err) {
  __shared__ int ok;
  const uint32_t e = sync[0];
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    // relaxed polls; one acquire load per flag once it shows the epoch orders the data reads after it
    for (int q = 0; q < world && ok; ++q) {
      while (static_cast<int32_t>(*reinterpret_cast<const volatile uint32_t*>(flags + q) - e) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs || (*reinterpret_cast<volatile int*>(err) & kErrTimeout)) {
          flag_error(err, kErrTimeout);
          ok = 0;
          break;
        }
      }
      if (ok) (void)ld_acquire_sys(flags + q);
    }
  }
  __syncthreads();
  if (!ok) return;
  const float* base = recv + int64_t(e & 1u) * world * part;
  lse_merge_rows(base, part, base + rows * head_dim, part, world, rows, head_dim, out, lse);
}

__device__ __forceinline__ void lse_merge_rows(const float* __restrict__ part_o, int64_t o_stride,
                                               const float* __restrict__ part_lse, int64_t lse_stride, int n_parts,
                                               int64_t rows, int head_dim, float* __restrict__ out,
                                               float* __restrict__ lse) {
  const int d = threadIdx.x;
  for (int64_t r = blockIdx.x * int64_t(blockDim.y) + threadIdx.y; r < rows; r += int64_t(gridDim.x) * blockDim.y) {
    float mx = -INFINITY;
    for (int p = 0; p < n_parts; ++p) mx = fmaxf(mx, part_lse[p * lse_stride + r]);
    float W = 0.f, O = 0.f;
    if (mx != -INFINITY) {
      for (int p = 0; p < n_parts; ++p) {
        const float w = expf(part_lse[p * lse_stride + r] - mx);
        W += w;
        if (d < head_dim && w > 0.f) O += w * part_o[p * o_stride + r * head_dim + d];
      }
    }
    if (d < head_dim) out[r * head_dim + d] = W > 0.f ? O / W : 0.f;
    if (d == 0 && lse) lse[r] = W > 0.f ? mx + logf(W) : -INFINITY;
  }
}

template <int G>
void launch_g(cudaStream_t st, const CUtensorMap& tmap, const DecodeArgs& a, int grid) {
  static std::atomic<uint64_t> configured{0};  // one bit per device: the attribute is per device context
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(configured.load() & bit)) {
    check_cuda(cudaFuncSetAttribute(decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
               "decode smem attribute");
    configured.fetch_or(bit);
  }
  decode_kernel<G><<<grid, kWarps * 32, kSmemBytes, st>>>(tmap, a);
}

}  // namespace

void preload_decode() {
  // Setting the shared-memory attribute needs each kernel's function handle, which loads the module (CUDA loads
  // modules lazily on first use); the merge kernel is loaded the same way.
  auto set = [](const void* fn) {
    check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes),
               "decode smem attribute");
  };
  set(reinterpret_cast<const void*>(decode_kernel<1>));
  set(reinterpret_cast<const void*>(decode_kernel<2>));
  set(reinterpret_cast<const void*>(decode_kernel<3>));
  set(reinterpret_cast<const void*>(decode_kernel<4>));
  set(reinterpret_cast<const void*>(decode_kernel<5>));
  set(reinterpret_cast<const void*>(decode_kernel<6>));
  set(reinterpret_cast<const void*>(decode_kernel<7>));
  set(reinterpret_cast<const void*>(decode_kernel<8>));
  cudaFuncAttributes attr;
  check_cuda(cudaFuncGetAttributes(&attr, lse_merge_kernel), "lse_merge attributes");
}

DecodePlan plan_decode(int n_rows, int n_kv_heads, int group, int n_heads, int max_seq_len, int page_size,
                       int num_sms, int requested_splits) {
  (void)group;
  DecodePlan p;
  const int max_pages = std::max(1, (max_seq_len + page_size - 1) / page_size);
  const int64_t units = int64_t(n_rows) * n_kv_heads;
  const int64_t slots = int64_t(num_sms) * kCtasPerSm;
  int ns = 1;
  if (requested_splits > 0) {
    ns = requested_splits;
  } else if (units * 5 < slots * 4) {
    // Fewer units than ~0.8 of a wave of CTAs. Measured on config-2 and config-4 slices: splitting a row costs
    // 10-15 % (each CTA's start and end, the merge), while CTAs that all run in one wave keep HBM busy; so the
    // largest split count whose CTAs still fit one wave, with at least 8 pages per split (16 rows x 8 KV heads
    // at 16k-64k tokens: 2 splits, 8-15 % faster than 4 or 9).
    const int ns_max = std::max(1, max_pages / 8);
    ns = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ns_max, slots / units)));
    if ((max_pages + ns - 1) / ns > 3072) {
      // Very long rows (131k tokens on 128 units: 2 splits leave 4097 pages per CTA): at least two waves,
      // preferring a count whose CTA total fills the last wave (>= 92 % of slots busy on average).
      const int ns_min = static_cast<int>(std::min<int64_t>(ns_max, (2 * slots + units - 1) / units));
      int best = ns_min;
      double best_eff = 0.0;
      for (int c = ns_min; c <= std::min(ns_max, ns_min * 4); ++c) {
        const int64_t ctas = units * c;
        const double eff = double(ctas) / double(((ctas + slots - 1) / slots) * slots);
        if (eff > best_eff + 1e-9) {
          best_eff = eff;
          best = c;
        }
        if (eff >= 0.92) break;
      }
      ns = best;
    }
  }
  // Otherwise one split: at 256-2048 units of 4097-token rows one split measured faster than 2, 3 or 4 at every
  // size, although a part-empty last wave is left.
  ns = std::min(ns, max_pages);
  int pps = (max_pages + ns - 1) / ns;
  pps = (pps + kChunkPages - 1) / kChunkPages * kChunkPages;  // splits start on a chunk boundary
  ns = (max_pages + pps - 1) / pps;
  p.n_splits = ns;
  p.pages_per_split = pps;
  p.scratch_bytes = ns > 1 ? size_t(ns) * n_rows * n_heads * (kD + 1) * sizeof(float) : 0;
  return p;
}

namespace {

DecodeArgs decode_args(const nbl_kv* kv, const float* q, const int32_t* page_table, int32_t pt_stride,
                       const int32_t* seq_lens, int n_rows, int n_heads, float* out, float* lse, const DecodePlan& plan,
                       void* scratch, int* err, unsigned* counts) {
  const auto& c = kv->cfg;
  DecodeArgs a{};
  a.q = q;
  a.page_table = page_table;
  a.seq_lens = seq_lens;
  a.out = out;
  a.lse = lse;
  a.err = err;
  a.n_pages = c.n_pages;
  a.pt_stride = pt_stride;
  a.n_rows = n_rows;
  a.n_heads = n_heads;
  a.n_kv_heads = c.n_kv_heads;
  a.n_splits = plan.n_splits;
  a.pages_per_split = plan.pages_per_split;
  a.scale_log2 = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
  if (plan.n_splits > 1) {
    a.part_o = static_cast<float*>(scratch);
    a.part_lse = a.part_o + size_t(plan.n_splits) * n_rows * n_heads * kD;
    a.counts = counts;
  }
  return a;
}

void launch_decode_kernel(cudaStream_t st, const nbl_kv* kv, const DecodeArgs& a) {
  const int group = a.n_heads / a.n_kv_heads;
  const int64_t grid = int64_t(a.n_rows) * a.n_kv_heads * a.n_splits;
  if (grid > 0x7fffffff) fail(NBL_E_INVALID, "decode: rows * kv_heads * splits exceeds the grid limit");
  switch (group) {
    case 1: launch_g<1>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 2: launch_g<2>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 3: launch_g<3>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 4: launch_g<4>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 5: launch_g<5>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 6: launch_g<6>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 7: launch_g<7>(st, kv->tmap, a, static_cast<int>(grid)); break;
    case 8: launch_g<8>(st, kv->tmap, a, static_cast<int>(grid)); break;
    default: fail(NBL_E_UNSUPPORTED, "decode: n_heads / n_kv_heads must be 1..8");
  }
  check_cuda(cudaGetLastError(), "decode launch");
}

void launch_peer_merge(cudaStream_t st, const float* recv, const uint32_t* flags, const uint32_t* sync, int world,
                       int64_t part, int64_t rows, int head_dim, float* out, float* lse, int* err, int num_sms) {
  const int tx = head_dim <= 32 ? 32 : (head_dim <= 64 ? 64 : (head_dim <= 128 ? 128 : 256));
  const int ty = std::max(1, 256 / tx);
  const int64_t blocks = std::min<int64_t>((rows + ty - 1) / ty, int64_t(num_sms) * 4);
  peer_merge_kernel<<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), dim3(tx, ty), 0, st>>>(
      recv, flags, sync, world, part, rows, head_dim, out, lse, err);
  check_cuda(cudaGetLastError(), "peer merge launch");
}

}  // namespace

void launch_decode(cudaStream_t st, const nbl_kv* kv, const float* q, const int32_t* page_table, int32_t pt_stride,
                   const int32_t* seq_lens, int n_rows, int n_heads, float* out, float* lse, const DecodePlan& plan,
                   void* scratch, int* err, unsigned* counts) {
  const DecodeArgs a = decode_args(kv, q, page_table, pt_stride, seq_lens, n_rows, n_heads, out, lse, plan, scratch,
                                   err, counts);
  launch_decode_kernel(st, kv, a);
  if (plan.n_splits > 1 && counts == nullptr)
    launch_lse_merge(st, a.part_o, a.part_lse, plan.n_splits, int64_t(n_rows) * n_heads, kD, out, lse);
}

void launch_decode_peers(cudaStream_t st, const nbl_kv* kv, const float* q, const int32_t* page_table,
                         int32_t pt_stride, const int32_t* seq_lens, int n_rows, int n_heads, const DecodePlan& plan,
                         void* scratch, unsigned* counts, int world, int rank, float* const* recv,
                         uint32_t* const* flags, uint32_t* sync, float* out, float* lse, int* err, int num_sms) {
  if (plan.n_splits > 1 && counts == nullptr) fail(NBL_E_INVALID, "decode_peers: split counters are required");
  DecodeArgs a = decode_args(kv, q, page_table, pt_stride, seq_lens, n_rows, n_heads, nullptr, nullptr, plan, scratch,
                             err, counts);
  a.px.world = world;
  a.px.rank = rank;
  a.px.sync = sync;
  a.px.part = int64_t(n_rows) * n_heads * (kD + 1);
  for (int p = 0; p < world; ++p) {
    a.px.recv[p] = recv[p];
    a.px.flags[p] = flags[p];
  }
  launch_decode_kernel(st, kv, a);
  launch_peer_merge(st, recv[rank], flags[rank], sync, world, a.px.part, int64_t(n_rows) * n_heads, kD, out, lse, err,
                    num_sms);
}

void launch_lse_exchange_peers(cudaStream_t st, const float* send, int64_t rows, int head_dim, int world, int rank,
                               float* const* recv, uint32_t* const* flags, uint32_t* sync, float* out, float* lse,
                               int* err, int num_sms) {
  PeerBufs px{};
  for (int p = 0; p < world; ++p) {
    px.recv[p] = recv[p];
    px.flags[p] = flags[p];
  }
  const int64_t part = rows * (int64_t(head_dim) + 1);
  bool vec = part % 4 == 0 && (reinterpret_cast<uintptr_t>(send) & 15u) == 0;
  for (int p = 0; p < world; ++p) vec = vec && (reinterpret_cast<uintptr_t>(recv[p]) & 15u) == 0;
  const int64_t items = vec ? part / 4 : part;
  const int push_grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, num_sms)));
  if (vec) peer_push_kernel<true><<<push_grid, 256, 0, st>>>(send, part, px, world, rank, sync);
  else peer_push_kernel<false><<<push_grid, 256, 0, st>>>(send, part, px, world, rank, sync);
  check_cuda(cudaGetLastError(), "peer push launch");
  launch_peer_merge(st, recv[rank], flags[rank], sync, world, part, rows, head_dim, out, lse, err, num_sms);
}

void launch_lse_merge(cudaStream_t st, const float* part_o, const float* part_lse, int n_parts, int64_t rows,
                      int head_dim, float* out, float* lse, int64_t o_stride, int64_t lse_stride) {
  if (o_stride < 0) o_stride = rows * head_dim;
  if (lse_stride < 0) lse_stride = rows;
  const int tx = head_dim <= 32 ? 32 : (head_dim <= 64 ? 64 : (head_dim <= 128 ? 128 : 256));
  const int ty = std::max(1, 256 / tx);
  const int64_t blocks = std::min<int64_t>((rows + ty - 1) / ty, 65535 * 16);
  lse_merge_kernel<<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), dim3(tx, ty), 0, st>>>(
      part_o, o_stride, part_lse, lse_stride, n_parts, rows, head_dim, out, lse);
  check_cuda(cudaGetLastError(), "lse_merge launch");
}

}  // namespace nbl
