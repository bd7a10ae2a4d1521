// The model's non-attention Backend ops on the GPU: embedding lookup, weight matmul, RMSNorm, residual add and
// the SwiGLU gate (src/backend/backend.h:54-70; the reference kernels are src/backend/cpu/ref_ops.cpp:80-98
// (embed), :109-136 (matmul_rows), :138-148 (rmsnorm), :151-153 (add), :217-222 (silu_mul)).
//
// Weights (F32 or F16, [ne1 rows][ne0]) live on the device as uploaded by nbl_weight_create. Decode-sized
// matmuls (n <= kGemvMaxRows activation rows) stream the weight once with 16-byte loads and keep all n rows'
// accumulators in registers: HBM-bound on the weight bytes. Larger n goes to the tensor-core GEMM (f32_gemm.cu), or,
// for a row width TMA cannot tile, to this file's fp32 CUDA-core GEMM (results within fp32 rounding of the CPU's).

#include <algorithm>

#include "model_ops.h"
#include "nbl_device.cuh"
#include "qkv_epilogue.cuh"

namespace nbl {
namespace {

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---------------------------------------------------------------- embed
// out[t][k] = table[ids[t]][k] widened to fp32. ids were range-checked on the host.
template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int32_t* __restrict__ ids, float* __restrict__ out,
                             int64_t ne0) {
  const int64_t t = blockIdx.y;
  const T* row = table + static_cast<int64_t>(ids[t]) * ne0;
  float* o = out + t * ne0;
  for (int64_t k = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; k < ne0; k += int64_t(gridDim.x) * blockDim.x) {
    if constexpr (sizeof(T) == 4) o[k] = row[k];
    else o[k] = __half2float(row[k]);
  }
}

// ---------------------------------------------------------------- matmul, decode-sized n (GEMV)
// y_j[t][r] = sum_k x[t][k] * w_j[r][k] for t < NT over up to kMaxMulti weights sharing x (Backend::matmul_multi:
// the Q/K/V and gate/up projections) in one launch: their rows are numbered consecutively. A fixed grid (a few CTAs
// per SM) of warps walks the rows with a grid stride; a row is cut into groups of 32 x kUnroll 16-byte chunks
// (lane l takes chunks l, l + 32, ...), and the next (row, group)'s chunks are loaded before the current one is
// used, so every warp keeps two groups (8 KB) of weight in flight and never waits on a CTA launch. x (NT rows)
// is read through the read-only cache: every warp reads the same few KB.
constexpr int kGemvThreads = 128;
constexpr int kGemvCtasPerSm = 4;  // at most; 128 threads at 128 registers: the register file holds exactly 4 CTAs
constexpr int kUnroll = 8;

template <int U, typename T>
__device__ __forceinline__ void gemv_load(uint4 (&raw)[U], const T* wr, int64_t base, int lane, int64_t n_chunks) {
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t c = base + lane + 32 * u;
    raw[u] = c < n_chunks ? __ldg(reinterpret_cast<const uint4*>(wr) + c) : make_uint4(0, 0, 0, 0);
  }
}

// Weight j of global row r (rows numbered consecutively over the batch): its row pointer, output column base and
// row count. A static scan, so the parameter block is never indexed dynamically.
template <typename T>
__device__ __forceinline__ void gemv_row(const GemvBatch& b, int64_t r, int64_t ne0, const T*& wr, float*& ybase,
                                         int64_t& local, int64_t& rows_j) {
  int64_t begin = 0;
  wr = static_cast<const T*>(b.w[0]);
  ybase = b.y[0];
  rows_j = b.row_end[0];
  bool found = r < b.row_end[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < b.count && !found && r < b.row_end[i]) {
      found = true;
      wr = static_cast<const T*>(b.w[i]);
      ybase = b.y[i];
      begin = b.row_end[i - 1];
      rows_j = b.row_end[i] - b.row_end[i - 1];
    }
  local = r - begin;
  wr += local * ne0;
}

// XREG (one activation row whose width fits one group, n_chunks <= 32 * kUnroll): each lane holds its slice of x --
// the kVec elements of each of its chunks, at most 64 floats -- in registers, so only the weights pass through L1
// (with x read through L1 as well, a 16-byte weight chunk costs 48 bytes of L1 traffic, and L1, not DRAM, limits
// the large matrices).
//
// EPI: the fused Q/K/V projection (launch_gemv_qkv). A warp takes pairs of rows instead of rows (qkv_row) and, when
// a pair's second row is done, lanes 0..NT-1 run the epilogue of one activation row each.
template <typename T, int NT, bool XREG, bool EPI = false>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvBatch b, const float* __restrict__ x,
                                                            int64_t ne0, const QkvEpilogue e) {
  static_assert(!XREG || NT == 1, "x in registers holds one activation row");
  constexpr int kVec = 16 / sizeof(T);  // weight elements per 16-byte load
  constexpr int kGroup = 32 * kUnroll;  // chunks per (row, group) item
  const int lane = threadIdx.x & 31;
  // Let the next kernel in the stream launch now: a dependent GEMV starts streaming its own weights while this one
  // finishes (it reads this one's output only after its griddepcontrol.wait).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  int64_t total = b.row_end[0];
#pragma unroll
  for (int i = 1; i < kMaxMulti; ++i)
    if (i < b.count) total = b.row_end[i];
  const int64_t n_warps = int64_t(gridDim.x) * (kGemvThreads / 32);
  const int64_t n_chunks = ne0 / kVec;
  const int64_t groups = (n_chunks + kGroup - 1) / kGroup;
  const int64_t warp_id = int64_t(blockIdx.x) * (kGemvThreads / 32) + (threadIdx.x >> 5);
  // r: the warp's current (virtual) row. Plain: rows warp_id, warp_id + n_warps, ...; EPI: pairs warp_id,
  // warp_id + n_warps, ..., each as its two virtual rows 2u, 2u + 1.
  int64_t r = EPI ? 2 * warp_id : warp_id;
  auto next_row = [&](int64_t v) -> int64_t { return EPI ? ((v & 1) ? v - 1 + 2 * n_warps : v + 1) : v + n_warps; };
  int region = 0, head = 0, pair = 0;
  auto phys = [&](int64_t v) -> int64_t { return EPI ? qkv_row(v, e, region, head, pair) : v; };
  int64_t g = 0;
  const T* wr = nullptr;
  float* ybase = nullptr;
  int64_t local = 0, rows_j = 0;
  uint4 raw[kUnroll];
  if (r < total) {
    gemv_row<T>(b, phys(r), ne0, wr, ybase, local, rows_j);
    gemv_load<kUnroll>(raw, wr, 0, lane, n_chunks);  // independent of the previous kernel: before the wait
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x (the previous kernel's output) is visible after this
  float xr[XREG ? kUnroll : 1][XREG ? kVec : 1];
  if constexpr (XREG) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t c = lane + 32 * u;
#pragma unroll
      for (int v = 0; v < kVec; v += 4) {
        const float4 xv = c < n_chunks ? ldg4(x + c * kVec + v) : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[u][v] = xv.x, xr[u][v + 1] = xv.y, xr[u][v + 2] = xv.z, xr[u][v + 3] = xv.w;
      }
    }
  }
  float acc[NT];
  float first = 0.f;  // EPI: lane t's sum of activation row t for the pair's first member
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  while (r < total) {
    const int64_t r_cur = r;
    uint4 cur[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) cur[u] = raw[u];
    const int64_t base = g * kGroup;
    // the next item of this warp: the row's next group, or the first group of its next row
    float* y_cur = ybase;
    const int64_t local_cur = local, rows_cur = rows_j;
    const bool row_done = g + 1 == groups;
    int64_t r2 = r, g2 = g + 1;
    if (row_done) {
      r2 = next_row(r);
      g2 = 0;
    }
    int region_cur = region, head_cur = head, pair_cur = pair;
    if (r2 < total) {
      if (row_done) gemv_row<T>(b, phys(r2), ne0, wr, ybase, local, rows_j);
      gemv_load<kUnroll>(raw, wr, g2 * kGroup, lane, n_chunks);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t c = base + lane + 32 * u;
      if (c < n_chunks) {
        float wv[kVec];
        if constexpr (sizeof(T) == 4) {
          wv[0] = __uint_as_float(cur[u].x);
          wv[1] = __uint_as_float(cur[u].y);
          wv[2] = __uint_as_float(cur[u].z);
          wv[3] = __uint_as_float(cur[u].w);
        } else {
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&cur[u].x));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&cur[u].y));
          const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&cur[u].z));
          const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&cur[u].w));
          wv[0] = f0.x, wv[1] = f0.y, wv[2] = f1.x, wv[3] = f1.y, wv[4] = f2.x, wv[5] = f2.y, wv[6] = f3.x, wv[7] = f3.y;
        }
        if constexpr (XREG) {
#pragma unroll
          for (int v = 0; v < kVec; ++v) acc[0] = fmaf(xr[u][v], wv[v], acc[0]);
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float* xt = x + t * ne0 + c * kVec;
#pragma unroll
            for (int v = 0; v < kVec; v += 4) {
              const float4 xv = ldg4(xt + v);
              acc[t] = fmaf(xv.x, wv[v], acc[t]);
              acc[t] = fmaf(xv.y, wv[v + 1], acc[t]);
              acc[t] = fmaf(xv.z, wv[v + 2], acc[t]);
              acc[t] = fmaf(xv.w, wv[v + 3], acc[t]);
            }
          }
        }
      }
    }
    if (row_done) {
      if constexpr (!EPI) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float s = acc[t];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) y_cur[t * rows_cur + local_cur] = s;
          acc[t] = 0.f;
        }
      } else {
        (void)y_cur;
        (void)local_cur;
        (void)rows_cur;
        float s_t = 0.f;  // lane t keeps activation row t's sum
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float s = acc[t];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == t) s_t = s;
          acc[t] = 0.f;
        }
        if ((r_cur & 1) == 0) {
          first = s_t;  // the pair's first member; lanes >= NT hold nothing
        } else if (lane < NT) {
          qkv_store(e, region_cur, head_cur, pair_cur, lane, first, s_t);
        }
      }
    }
    r = r2;
    g = g2;
  }
}

// Any ne0 (no alignment assumptions): one warp per output row and activation row, scalar loads.
template <typename T>
__global__ void gemv_scalar_kernel(const T* __restrict__ w, const float* __restrict__ x, float* __restrict__ y,
                                   int64_t ne0, int64_t ne1, int64_t n) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = int64_t(blockIdx.x) * (blockDim.x / 32) + warp;
  const int64_t t = blockIdx.y;
  if (r >= ne1 || t >= n) return;
  const T* wr = w + r * ne0;
  const float* xt = x + t * ne0;
  float s = 0.f;
  for (int64_t k = lane; k < ne0; k += 32) {
    float wk;
    if constexpr (sizeof(T) == 4) wk = wr[k];
    else wk = __half2float(wr[k]);
    s = fmaf(xt[k], wk, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) y[t * ne1 + r] = s;
}

// ---------------------------------------------------------------- rmsnorm
// One CTA per row: sum of squares in double, scale = 1 / sqrt(ss / d + eps) in double, y = x * scale * w rounded
// once to float -- the reference's arithmetic (ref_ops.cpp:138-148); only the order of the double sum differs.
constexpr int kNormThreads = 256;

// rmsnorm, add and silu_mul are launched with programmatic stream serialization (pdl_launch): one of them may be
// scheduled while the kernel before it in the stream still runs -- the GEMVs allow that from their first
// instruction -- and waits here, before touching memory, until that kernel has finished and its writes are
// visible. A decode step is a chain of ~10 short dependent launches per layer, so hiding their launch latency
// behind the GEMVs is worth 17-26 % of whole-model decode throughput. These kernels never signal their own
// dependents early: whatever follows them starts only once they have finished (measured: letting the small
// kernels release their successors at their start made the batched-decoder and flat-route model checks fail).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
void pdl_launch(cudaStream_t st, void (*kernel)(KArgs...), dim3 grid, dim3 block, const char* what, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), what);
}

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               float* __restrict__ y, int64_t d, float eps) {
  pdl_wait();
  __shared__ double part[kNormThreads / 32];
  const float* xt = x + int64_t(blockIdx.x) * d;
  float* yt = y + int64_t(blockIdx.x) * d;
  double ss = 0.0;
  for (int64_t i = threadIdx.x; i < d; i += kNormThreads) ss += static_cast<double>(xt[i]) * xt[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += part[i];
  const double scale = 1.0 / sqrt(tot / static_cast<double>(d) + static_cast<double>(eps));
  for (int64_t i = threadIdx.x; i < d; i += kNormThreads)
    yt[i] = static_cast<float>(static_cast<double>(xt[i]) * scale * static_cast<double>(w[i]));
}

// ---------------------------------------------------------------- elementwise
// vec: both pointers 16-byte aligned (float4 body, scalar tail); otherwise all scalar.
__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t count, bool vec) {
  pdl_wait();
  const int64_t n4 = vec ? count / 4 : 0;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(x)[i];
    const float4 b = ldg4(y + 4 * i);
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    reinterpret_cast<float4*>(x)[i] = a;
  }
  for (int64_t i = 4 * n4 + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count;
       i += int64_t(gridDim.x) * blockDim.x)
    x[i] += y[i];
}

// gate = g / (1 + e^-g) * up in float, like ref_ops.cpp:217-222 (expf here, std::exp there: both within an ulp
// or two of e^-g).
__device__ __forceinline__ float silu_mul1(float g, float u) { return g / (1.0f + expf(-g)) * u; }

__global__ void silu_mul_kernel(float* __restrict__ gate, const float* __restrict__ up, int64_t count, bool vec) {
  pdl_wait();
  const int64_t n4 = vec ? count / 4 : 0;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 g = reinterpret_cast<float4*>(gate)[i];
    const float4 u = ldg4(up + 4 * i);
    g.x = silu_mul1(g.x, u.x);
    g.y = silu_mul1(g.y, u.y);
    g.z = silu_mul1(g.z, u.z);
    g.w = silu_mul1(g.w, u.w);
    reinterpret_cast<float4*>(gate)[i] = g;
  }
  for (int64_t i = 4 * n4 + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count;
       i += int64_t(gridDim.x) * blockDim.x)
    gate[i] = silu_mul1(gate[i], up[i]);
}

bool aligned16(const void* a, const void* b) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u) == 0;
}

int elementwise_grid(int64_t count, int num_sms) {
  const int64_t want = (count / 4 + 255) / 256;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(num_sms) * 8)));
}

// Launched with programmatic stream serialization: the kernel may start while the previous one in the stream is
// still running, and orders itself behind it with griddepcontrol.wait before reading x.
template <typename T, int NT, bool XREG = false, bool EPI = false>
void gemv_t(cudaStream_t st, const GemvBatch& b, const float* x, int64_t ne0, int num_sms,
            const QkvEpilogue& e = QkvEpilogue{}) {
  // resident CTAs per SM for this instantiation (its register count decides: 3 or 4)
  static const int per_sm = [] {
    int n = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kernel<T, NT, XREG, EPI>, kGemvThreads, 0),
               "gemv occupancy");
    return std::max(1, std::min(n, kGemvCtasPerSm));
  }();
  const int64_t warps_per_cta = kGemvThreads / 32;
  const int64_t items = EPI ? b.row_end[b.count - 1] / 2 : b.row_end[b.count - 1];  // pairs for EPI
  const int64_t grid = std::min<int64_t>((items + warps_per_cta - 1) / warps_per_cta, int64_t(num_sms) * per_sm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kGemvThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, gemv_kernel<T, NT, XREG, EPI>, b, x, ne0, e), "gemv launch");
}

template <typename T, bool EPI = false>
void gemv_dispatch(cudaStream_t st, const GemvBatch& b, const float* x, int64_t ne0, int64_t n, int sms,
                   const QkvEpilogue& e = QkvEpilogue{}) {
  constexpr int64_t kVec = 16 / sizeof(T);
  if (n == 1 && ne0 / kVec <= 32 * kUnroll) return gemv_t<T, 1, true, EPI>(st, b, x, ne0, sms, e);
  switch (n) {
    case 1: return gemv_t<T, 1, false, EPI>(st, b, x, ne0, sms, e);
    case 2: return gemv_t<T, 2, false, EPI>(st, b, x, ne0, sms, e);
    case 3: return gemv_t<T, 3, false, EPI>(st, b, x, ne0, sms, e);
    case 4: return gemv_t<T, 4, false, EPI>(st, b, x, ne0, sms, e);
    case 5: return gemv_t<T, 5, false, EPI>(st, b, x, ne0, sms, e);
    case 6: return gemv_t<T, 6, false, EPI>(st, b, x, ne0, sms, e);
    case 7: return gemv_t<T, 7, false, EPI>(st, b, x, ne0, sms, e);
    default: return gemv_t<T, 8, false, EPI>(st, b, x, ne0, sms, e);
  }
}

}  // namespace

void launch_embed(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out, int num_sms) {
  const int64_t per_row = std::max<int64_t>(1, std::min<int64_t>((table.ne0 + 255) / 256, 64));
  const dim3 grid(static_cast<unsigned>(per_row), static_cast<unsigned>(n));
  (void)num_sms;
  if (table.dtype == NBL_F32)
    embed_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(table.dev), ids, out, table.ne0);
  else
    embed_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(table.dev), ids, out, table.ne0);
}

// y[n][ne1] = x[n][ne0] . W[ne1][ne0]^T in fp32 on the CUDA cores, for float weights whose row width the tensor-core
// GEMM cannot tile with TMA (ne0 not a multiple of 8 for F16, of 4 for F32: no model nibble loads has such a width,
// so this is a correctness path, not a fast one). 64 x 64 output tiles; each of 256 threads accumulates a 4 x 4 block
// with fused multiply-adds over k in order, so every output is one fp32 sum of the reference's products (within
// the fp32 summation bound of the reference's own loop, ref_ops.cpp:109-136). K is staged through shared memory
// 16 columns at a time; any shape and any 4-byte-aligned pointers.
constexpr int kSgTile = 64;

template <typename T>
__global__ void __launch_bounds__(256) sgemm_nt_kernel(const T* __restrict__ w, const float* __restrict__ x,
                                                       float* __restrict__ y, int64_t ne0, int64_t ne1, int64_t n) {
  constexpr int kK = 16;
  __shared__ float xs[kK][kSgTile + 4];  // [k][activation row]
  __shared__ float ws[kK][kSgTile + 4];  // [k][weight row]
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row0 = int64_t(blockIdx.y) * kSgTile, col0 = int64_t(blockIdx.x) * kSgTile;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int64_t k0 = 0; k0 < ne0; k0 += kK) {
    for (int i = threadIdx.x; i < kSgTile * kK; i += 256) {
      const int r = i / kK, k = i % kK;
      const int64_t gk = k0 + k;
      xs[k][r] = row0 + r < n && gk < ne0 ? x[(row0 + r) * ne0 + gk] : 0.f;
      ws[k][r] = col0 + r < ne1 && gk < ne0 ? static_cast<float>(w[(col0 + r) * ne0 + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[k][ty * 4 + i];
        b[i] = ws[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty * 4 + i;
    if (r >= n) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = col0 + tx * 4 + j;
      if (c < ne1) y[r * ne1 + c] = acc[i][j];
    }
  }
}

bool gemv_vector_ok(const Weight& w, const float* x) {
  const int vec = w.dtype == NBL_F32 ? 4 : 8;
  return w.ne0 % vec == 0 && (reinterpret_cast<uintptr_t>(w.dev) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
}

void launch_gemv_multi(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x,
                       int64_t n, int num_sms) {
  const Weight& w0 = *ws[0];
  bool vec = true;
  for (int i = 0; i < count; ++i) vec = vec && gemv_vector_ok(*ws[i], x) && ws[i]->dtype == w0.dtype;
  if (!vec) {
    for (int i = 0; i < count; ++i) {
      const Weight& w = *ws[i];
      const dim3 grid(static_cast<unsigned>((w.ne1 + 7) / 8), static_cast<unsigned>(n));
      if (w.dtype == NBL_F32)
        gemv_scalar_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w.dev), x, ys[i], w.ne0, w.ne1, n);
      else
        gemv_scalar_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w.dev), x, ys[i], w.ne0, w.ne1, n);
    }
    return;
  }
  for (int64_t t0 = 0; t0 < n; t0 += kGemvMaxRows) {
    const int64_t nt = std::min<int64_t>(kGemvMaxRows, n - t0);
    GemvBatch b{};
    b.count = count;
    int64_t rows = 0;
    for (int i = 0; i < count; ++i) {
      b.w[i] = ws[i]->dev;
      b.y[i] = ys[i] + t0 * ws[i]->ne1;
      rows += ws[i]->ne1;
      b.row_end[i] = rows;
    }
    if (w0.dtype == NBL_F32) gemv_dispatch<float>(st, b, x + t0 * w0.ne0, w0.ne0, nt, num_sms);
    else gemv_dispatch<__half>(st, b, x + t0 * w0.ne0, w0.ne0, nt, num_sms);
  }
}

bool gemv_qkv_ok(const Weight* const* ws, const float* x, int64_t n, int64_t n_heads, int64_t n_kv_heads) {
  const Weight &wq = *ws[0], &wk = *ws[1], &wv = *ws[2];
  return n >= 1 && n <= kGemvMaxRows && wq.dtype == wk.dtype && wq.dtype == wv.dtype &&
         (wq.dtype == NBL_F32 || wq.dtype == NBL_F16) && wq.ne0 == wk.ne0 && wq.ne0 == wv.ne0 &&
         wq.ne1 == n_heads * 64 && wk.ne1 == n_kv_heads * 64 && wv.ne1 == wk.ne1 && n_heads > 0 && n_kv_heads > 0 &&
         gemv_vector_ok(wq, x) && gemv_vector_ok(wk, x) && gemv_vector_ok(wv, x);
}

bool launch_gemv_qkv(cudaStream_t st, const Weight* const* ws, const float* x, int64_t n, const QkvEpilogue& e,
                     int num_sms) {
  const Weight& wq = *ws[0];
  if (!gemv_qkv_ok(ws, x, n, e.n_heads, e.n_kv_heads)) return false;
  GemvBatch b{};
  b.count = 3;
  int64_t rows = 0;
  for (int i = 0; i < 3; ++i) {
    b.w[i] = ws[i]->dev;
    b.y[i] = nullptr;  // the epilogue stores instead
    rows += ws[i]->ne1;
    b.row_end[i] = rows;
  }
  if (wq.dtype == NBL_F32) gemv_dispatch<float, true>(st, b, x, wq.ne0, n, num_sms, e);
  else gemv_dispatch<__half, true>(st, b, x, wq.ne0, n, num_sms, e);
  return true;
}

void launch_gemv(cudaStream_t st, const Weight& w, const float* x, float* y, int64_t n, int num_sms) {
  const Weight* ws[1] = {&w};
  float* ys[1] = {y};
  launch_gemv_multi(st, ws, ys, 1, x, n, num_sms);
}

void launch_gemm_fallback(cudaStream_t st, const Weight& w, const float* x, float* y, int64_t n) {
  const dim3 grid(static_cast<unsigned>((w.ne1 + kSgTile - 1) / kSgTile), static_cast<unsigned>((n + kSgTile - 1) / kSgTile));
  if (grid.y > 65535u) fail(NBL_E_INVALID, "matmul: too many activation rows for the fallback GEMM");
  if (w.dtype == NBL_F32)
    sgemm_nt_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w.dev), x, y, w.ne0, w.ne1, n);
  else
    sgemm_nt_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w.dev), x, y, w.ne0, w.ne1, n);
  check_cuda(cudaGetLastError(), "fallback GEMM launch");
}

void launch_rmsnorm(cudaStream_t st, const float* x, const float* w, float* y, int64_t n, int64_t d, float eps) {
  pdl_launch(st, rmsnorm_kernel, dim3(static_cast<unsigned>(n)), dim3(kNormThreads), "rmsnorm launch", x, w, y, d, eps);
}

void launch_add(cudaStream_t st, float* x, const float* y, int64_t count, int num_sms) {
  pdl_launch(st, add_kernel, dim3(elementwise_grid(count, num_sms)), dim3(256), "add launch", x, y, count,
             aligned16(x, y));
}

void launch_silu_mul(cudaStream_t st, float* gate, const float* up, int64_t count, int num_sms) {
  pdl_launch(st, silu_mul_kernel, dim3(elementwise_grid(count, num_sms)), dim3(256), "silu_mul launch", gate, up,
             count, aligned16(gate, up));
}

}  // namespace nbl
