// extern "C" shim over nibble's own attention-path code, compiled together with the reference sources
// (oracle/Makefile) into oracle/_ref/libnibble_ref.so.
//
// TEST INFRASTRUCTURE ONLY: tests use it to pin the C oracle (nbl_oracle.c) against the reference itself, the
// golden-fixture generator uses it, and bench.py's CPU-baseline / reference arm times CpuBackend::attention
// through it. The product library never loads it.
//
// Wrapped entry points:
//   nibble::cpu::attention_heads   src/backend/cpu/ref_ops.cpp:188   (scalar oracle)
//   nibble::cpu::rope              src/backend/cpu/ref_ops.cpp:166
//   nibble::cpu::softmax_inplace   src/backend/cpu/ref_ops.cpp:66
//   nibble::cpu::CpuBackend        src/backend/cpu/cpu_backend.cpp:20 (ctor), :272 (attention) on a ThreadPool
//   nibble::simd::select           src/backend/cpu/simd/dispatch.cpp:123 (the kernel tier the backend runs)
//   nibble::fp16_to_fp32 / fp32_to_fp16   src/fp16.h:18, :46
//   nibble::cpu::embed / matmul_rows / rmsnorm / add / silu_mul   src/backend/cpu/ref_ops.cpp:80, :109, :138, :151,
//                                  :217 (the model's other ops, scalar), and the same ops through CpuBackend
#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <span>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "backend/cpu/ref_ops.h"
#include "backend/cpu/simd/dispatch.h"
#include "fp16.h"
#include "quant.h"
#include "thread_pool.h"

namespace {
thread_local char g_err[512];
void set_err(const char* m) {
  std::strncpy(g_err, m, sizeof g_err - 1);
  g_err[sizeof g_err - 1] = 0;
}
// A thread pool plus the CPU backend that runs on it (the pair Model::Impl builds, src/nibble.cpp:79-81).
struct RefBackend {
  nibble::ThreadPool pool;
  nibble::cpu::CpuBackend be;
  explicit RefBackend(int threads) : pool(threads), be(pool) {}
};
}  // namespace

extern "C" {

const char* nref_last_error() { return g_err; }

void nref_attention_scalar(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                           int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float* scratch) {
  nibble::cpu::attention_heads(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, 0, n_heads, scratch);
}

void nref_rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, float freq_base, int neox,
               const float* freq_factors) {
  const nibble::RopeParams p{freq_base, neox != 0, freq_factors};
  nibble::cpu::rope(x, n, n_heads, head_dim, pos0, p);
}

void nref_softmax(float* x, int64_t n) { nibble::cpu::softmax_inplace(x, n); }

float nref_fp16_to_fp32(uint16_t h) { return nibble::fp16_to_fp32(h); }
uint16_t nref_fp32_to_fp16(float f) { return nibble::fp32_to_fp16(f); }
// Bulk forms: results never pass through a host-language float, so NaN payloads arrive unchanged.
void nref_fp16_to_fp32_n(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = nibble::fp16_to_fp32(src[i]);
}
void nref_fp32_to_fp16_n(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = nibble::fp32_to_fp16(src[i]);
}

// Name of the SIMD tier CpuBackend selects on this CPU ("scalar" when none).
const char* nref_kernels_name() {
  try {
    const nibble::simd::Kernels* k = nibble::simd::select();
    return k ? k->name : "scalar";
  } catch (const std::exception& e) {
    set_err(e.what());
    return nullptr;
  }
}

// Creates a ThreadPool of `threads` (caller included) and a CpuBackend on it; nullptr on failure.
void* nref_backend_create(int threads) {
  try {
    return new RefBackend(threads);
  } catch (const std::exception& e) {
    set_err(e.what());
    return nullptr;
  }
}

void nref_backend_destroy(void* h) { delete static_cast<RefBackend*>(h); }

int nref_backend_threads(void* h) { return static_cast<RefBackend*>(h)->pool.size(); }

// Backend::reserve(ReserveParams{n_ctx, n_heads, max_rows, max_width}); 0 on success.
int nref_backend_reserve(void* h, int64_t n_ctx, int64_t n_heads, int64_t max_rows, int64_t max_width) {
  try {
    static_cast<RefBackend*>(h)->be.reserve({n_ctx, n_heads, max_rows, max_width});
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

// CpuBackend::attention on host buffers (the CPU backend's memory is host memory).
int nref_backend_attention(void* h, const float* q, const float* k, const float* v, float* out, int64_t n,
                           int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
  try {
    static_cast<RefBackend*>(h)->be.attention(q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

// CpuBackend::rope (scalar cpu::rope behind the backend's dispatch).
int nref_backend_rope(void* h, float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, float freq_base,
                      int neox, const float* freq_factors) {
  try {
    const nibble::RopeParams p{freq_base, neox != 0, freq_factors};
    static_cast<RefBackend*>(h)->be.rope(x, n, n_heads, head_dim, pos0, p);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

// ---- the model's other ops (dtype 0 = F32, 1 = F16) ----
namespace {
// dtype: 0 = F32, 1 = F16, otherwise a quantized type's DType id (2 Q4_0, 6 Q5_0, 8 Q8_0, ...).
nibble::Tensor tensor_of(const void* data, int dtype, int64_t ne0, int64_t ne1) {
  nibble::Tensor t;
  t.type = static_cast<nibble::DType>(dtype);
  t.n_dims = ne1 > 1 ? 2 : 1;
  t.ne = {ne0, ne1, 1, 1};
  t.data = data;
  return t;
}
}  // namespace

int nref_embed(const void* table, int dtype, int64_t ne0, int64_t n_rows, const int32_t* ids, int64_t n, float* out) {
  try {
    nibble::cpu::embed(tensor_of(table, dtype, ne0, n_rows), std::span<const int32_t>(ids, static_cast<size_t>(n)), out);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

int nref_matmul(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n) {
  try {
    nibble::cpu::matmul_rows(tensor_of(w, dtype, ne0, ne1), x, y, n, 0, ne1, nullptr);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

// nibble::quantize_row_q8_0 (src/quant.cpp:250) into 34-byte blocks.
void nref_quantize_q8_0(const float* x, void* blocks, int64_t n) {
  nibble::quantize_row_q8_0(x, static_cast<nibble::BlockQ8_0*>(blocks), n);
}

// nibble::dequantize_row (src/quant.cpp:158) for any supported dtype id.
int nref_dequantize_row(int dtype, const void* src, float* dst, int64_t n) {
  try {
    nibble::dequantize_row(static_cast<nibble::DType>(dtype), src, dst, n);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

// nibble::quantize_row_q8_1 (src/quant.cpp:260) into 36-byte blocks and nibble::quantize_row_q8_K (:276) into
// 292-byte blocks.
void nref_quantize_q8_1(const float* x, void* blocks, int64_t n) {
  nibble::quantize_row_q8_1(x, static_cast<nibble::BlockQ8_1*>(blocks), n);
}
void nref_quantize_q8_K(const float* x, void* blocks, int64_t n) {
  nibble::quantize_row_q8_K(x, static_cast<nibble::BlockQ8_K*>(blocks), n);
}

// nibble::cpu::matmul_rows with a quantized weight: x quantized row by row to the weight type's activation blocks
// (Q8_0 by quantize_rows_q8_0; Q8_1 and Q8_K by quantize_row_q8_1 / quantize_row_q8_K, as CpuBackend::matmul_multi
// does at src/backend/cpu/cpu_backend.cpp:165-207), then the scalar block dots.
int nref_matmul_q(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n) {
  try {
    const auto act = nibble::act_type(static_cast<nibble::DType>(dtype));
    std::vector<nibble::BlockQ8_0> xq;
    std::vector<nibble::BlockQ8_1> xq1;
    std::vector<nibble::BlockQ8_K> xqk;
    nibble::QuantActs acts;
    if (act == nibble::ActType::Q8_0) {
      xq.resize(static_cast<size_t>(n * (ne0 / 32)));
      nibble::cpu::quantize_rows_q8_0(x, xq.data(), n, ne0);
      acts.q8_0 = xq.data();
    } else if (act == nibble::ActType::Q8_1) {
      xq1.resize(static_cast<size_t>(n * (ne0 / 32)));
      for (int64_t t = 0; t < n; ++t) nibble::quantize_row_q8_1(x + t * ne0, xq1.data() + t * (ne0 / 32), ne0);
      acts.q8_1 = xq1.data();
    } else {
      xqk.resize(static_cast<size_t>(n * (ne0 / 256)));
      for (int64_t t = 0; t < n; ++t) nibble::quantize_row_q8_K(x + t * ne0, xqk.data() + t * (ne0 / 256), ne0);
      acts.q8_K = xqk.data();
    }
    nibble::cpu::matmul_rows(tensor_of(w, dtype, ne0, ne1), x, y, n, 0, ne1, &acts);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

void nref_rmsnorm(const float* x, const float* weight, float* y, int64_t n, int64_t d, float eps) {
  nibble::cpu::rmsnorm(x, tensor_of(weight, 0, d, 1), y, n, eps);
}

void nref_add(float* x, const float* y, int64_t count) { nibble::cpu::add(x, y, count); }

void nref_silu_mul(float* gate, const float* up, int64_t count) { nibble::cpu::silu_mul(gate, up, count); }

// The same ops through CpuBackend (its SIMD tier where the build has one).
int nref_backend_matmul(void* h, const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y,
                        int64_t n) {
  try {
    static_cast<RefBackend*>(h)->be.matmul(tensor_of(w, dtype, ne0, ne1), x, y, n);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

int nref_backend_rmsnorm(void* h, const float* x, const float* weight, float* y, int64_t n, int64_t d, float eps) {
  try {
    static_cast<RefBackend*>(h)->be.rmsnorm(x, tensor_of(weight, 0, d, 1), y, n, eps);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

int nref_backend_silu_mul(void* h, float* gate, const float* up, int64_t count) {
  try {
    static_cast<RefBackend*>(h)->be.silu_mul(gate, up, count);
    return 0;
  } catch (const std::exception& e) {
    set_err(e.what());
    return 1;
  }
}

}  // extern "C"
