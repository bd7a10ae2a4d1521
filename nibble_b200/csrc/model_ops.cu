// The model's non-attention Backend ops on the GPU: embedding lookup, weight matmul, RMSNorm, residual add and
// the SwiGLU gate (src/backend/backend.h:54-70; the reference kernels are src/backend/cpu/ref_ops.cpp:80-98
// (embed), :109-136 (matmul_rows), :138-148 (rmsnorm), :151-153 (add), :217-222 (silu_mul)).
//
// Weights (F32 or F16, [ne1 rows][ne0]) live on the device as uploaded by nbl_weight_create. Decode-sized
// matmuls (n <= kGemvMaxRows activation rows) stream the weight once with 16-byte loads and keep all n rows'
// accumulators in registers: HBM-bound on the weight bytes. Larger n goes to cuBLAS SGEMM on an fp32 copy of
// the weight (plain fp32 arithmetic, no TF32, so results stay within fp32 rounding of the CPU's).
#include <cublas_v2.h>

#include <algorithm>

#include "model_ops.h"
#include "nbl_device.cuh"

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
// y[t][r] = sum_k x[t][k] * w[r][k] for t < NT. One warp per kRowsPerWarp weight rows; lane l reads 16-byte
// chunks l, l+32, ... of each row (kVec elements), so a warp streams whole 512-byte segments. x (NT rows) is
// read through the read-only cache: every warp of every CTA reads the same few KB.
constexpr int kGemvThreads = 256;
constexpr int kRowsPerWarp = 2;

template <typename T, int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const T* __restrict__ w, const float* __restrict__ x,
                                                            float* __restrict__ y, int64_t ne0, int64_t ne1) {
  constexpr int kVec = 16 / sizeof(T);  // weight elements per 16-byte load
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t(blockIdx.x) * (kGemvThreads / 32) + warp) * kRowsPerWarp;
  if (r0 >= ne1) return;
  float acc[kRowsPerWarp][NT];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[i][t] = 0.f;
  const int64_t n_chunks = ne0 / kVec;
#pragma unroll 2
  for (int64_t c = lane; c < n_chunks; c += 32) {
    float wv[kRowsPerWarp][kVec];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int64_t r = min(r0 + i, ne1 - 1);  // a missing last row re-reads a valid one; its sum is dropped
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(w + r * ne0) + c);
      if constexpr (sizeof(T) == 4) {
        wv[i][0] = __uint_as_float(raw.x);
        wv[i][1] = __uint_as_float(raw.y);
        wv[i][2] = __uint_as_float(raw.z);
        wv[i][3] = __uint_as_float(raw.w);
      } else {
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
          wv[i][2 * j] = f.x;
          wv[i][2 * j + 1] = f.y;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float* xt = x + t * ne0 + c * kVec;
#pragma unroll
      for (int v = 0; v < kVec; v += 4) {
        const float4 xv = ldg4(xt + v);
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
          acc[i][t] = fmaf(xv.x, wv[i][v], acc[i][t]);
          acc[i][t] = fmaf(xv.y, wv[i][v + 1], acc[i][t]);
          acc[i][t] = fmaf(xv.z, wv[i][v + 2], acc[i][t]);
          acc[i][t] = fmaf(xv.w, wv[i][v + 3], acc[i][t]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float s = acc[i][t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      acc[i][t] = s;
    }
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i)
      if (r0 + i < ne1)
#pragma unroll
        for (int t = 0; t < NT; ++t) y[t * ne1 + r0 + i] = acc[i][t];
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

__global__ void widen_f16_kernel(const __half* __restrict__ src, float* __restrict__ dst, int64_t count) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __half2float(src[i]);
}

// ---------------------------------------------------------------- rmsnorm
// One CTA per row: sum of squares in double, scale = 1 / sqrt(ss / d + eps) in double, y = x * scale * w rounded
// once to float -- the reference's arithmetic (ref_ops.cpp:138-148); only the order of the double sum differs.
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               float* __restrict__ y, int64_t d, float eps) {
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

template <typename T, int NT>
void gemv_t(cudaStream_t st, const void* w, const float* x, float* y, int64_t ne0, int64_t ne1) {
  const int64_t rows_per_cta = (kGemvThreads / 32) * kRowsPerWarp;
  const int64_t grid = (ne1 + rows_per_cta - 1) / rows_per_cta;
  gemv_kernel<T, NT><<<static_cast<unsigned>(grid), kGemvThreads, 0, st>>>(static_cast<const T*>(w), x, y, ne0, ne1);
}

template <typename T>
void gemv_dispatch(cudaStream_t st, const void* w, const float* x, float* y, int64_t ne0, int64_t ne1, int64_t n) {
  switch (n) {
    case 1: return gemv_t<T, 1>(st, w, x, y, ne0, ne1);
    case 2: return gemv_t<T, 2>(st, w, x, y, ne0, ne1);
    case 3: return gemv_t<T, 3>(st, w, x, y, ne0, ne1);
    case 4: return gemv_t<T, 4>(st, w, x, y, ne0, ne1);
    case 5: return gemv_t<T, 5>(st, w, x, y, ne0, ne1);
    case 6: return gemv_t<T, 6>(st, w, x, y, ne0, ne1);
    case 7: return gemv_t<T, 7>(st, w, x, y, ne0, ne1);
    default: return gemv_t<T, 8>(st, w, x, y, ne0, ne1);
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

void launch_widen_f16(cudaStream_t st, const void* src, float* dst, int64_t count, int num_sms) {
  widen_f16_kernel<<<elementwise_grid(count, num_sms), 256, 0, st>>>(static_cast<const __half*>(src), dst, count);
}

bool gemv_vector_ok(const Weight& w, const float* x) {
  const int vec = w.dtype == NBL_F32 ? 4 : 8;
  return w.ne0 % vec == 0 && (reinterpret_cast<uintptr_t>(w.dev) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
}

void launch_gemv(cudaStream_t st, const Weight& w, const float* x, float* y, int64_t n) {
  if (gemv_vector_ok(w, x)) {
    for (int64_t t0 = 0; t0 < n; t0 += kGemvMaxRows) {
      const int64_t nt = std::min<int64_t>(kGemvMaxRows, n - t0);
      if (w.dtype == NBL_F32) gemv_dispatch<float>(st, w.dev, x + t0 * w.ne0, y + t0 * w.ne1, w.ne0, w.ne1, nt);
      else gemv_dispatch<__half>(st, w.dev, x + t0 * w.ne0, y + t0 * w.ne1, w.ne0, w.ne1, nt);
    }
  } else {
    const dim3 grid(static_cast<unsigned>((w.ne1 + 7) / 8), static_cast<unsigned>(n));
    if (w.dtype == NBL_F32)
      gemv_scalar_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(w.dev), x, y, w.ne0, w.ne1, n);
    else
      gemv_scalar_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(w.dev), x, y, w.ne0, w.ne1, n);
  }
}

void gemm_f32(cublasHandle_t h, cudaStream_t st, const float* w_f32, const float* x, float* y, int64_t ne0, int64_t ne1,
              int64_t n) {
  // Row-major y[n][ne1] = x[n][ne0] . W^T is column-major Y^T (ne1 x n) = W (as ne0 x ne1, transposed) . X^T.
  const float one = 1.f, zero = 0.f;
  if (cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS) fail(NBL_E_CUDA, "cublasSetStream failed");
  const cublasStatus_t s =
      cublasSgemm(h, CUBLAS_OP_T, CUBLAS_OP_N, static_cast<int>(ne1), static_cast<int>(n), static_cast<int>(ne0), &one,
                  w_f32, static_cast<int>(ne0), x, static_cast<int>(ne0), &zero, y, static_cast<int>(ne1));
  if (s != CUBLAS_STATUS_SUCCESS) fail(NBL_E_CUDA, "cublasSgemm failed (status " + std::to_string(int(s)) + ")");
}

void launch_rmsnorm(cudaStream_t st, const float* x, const float* w, float* y, int64_t n, int64_t d, float eps) {
  rmsnorm_kernel<<<static_cast<unsigned>(n), kNormThreads, 0, st>>>(x, w, y, d, eps);
}

void launch_add(cudaStream_t st, float* x, const float* y, int64_t count, int num_sms) {
  add_kernel<<<elementwise_grid(count, num_sms), 256, 0, st>>>(x, y, count, aligned16(x, y));
}

void launch_silu_mul(cudaStream_t st, float* gate, const float* up, int64_t count, int num_sms) {
  silu_mul_kernel<<<elementwise_grid(count, num_sms), 256, 0, st>>>(gate, up, count, aligned16(gate, up));
}

}  // namespace nbl
