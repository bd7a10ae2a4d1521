#pragma once
// The operator interface nibble's Transformer is written against, restated for this build so a CUDA backend
// can be compiled beside it. Names, argument meaning and error behaviour follow the reference:
//   DType / Tensor          src/tensor.h:21-31, :53-66   (ggml type ids; non-owning row-major view)
//   RopeParams              src/backend/backend.h:16-20
//   ReserveParams           src/backend/backend.h:24-26
//   Backend                 src/backend/backend.h:36-71
//   Error                   include/nibble/error.h:8-13  (input/resource faults; self-contained what())
// A nibble tree that links this backend uses its own copies of these declarations; they must stay
// layout- and signature-identical, which is why this header keeps them alike.
#include <array>
#include <cstdint>
#include <span>
#include <stdexcept>

namespace nibble {

class Error : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

enum class DType : uint32_t { F32 = 0, F16 = 1, Q4_0 = 2, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

struct Tensor {
  DType type = DType::F32;
  int n_dims = 0;
  std::array<int64_t, 4> ne{1, 1, 1, 1};
  const void* data = nullptr;
  int64_t rows() const { return ne[1] * ne[2] * ne[3]; }
};

struct RopeParams {
  float freq_base;
  bool neox;
  const float* freq_factors;  // nullptr or head_dim/2 floats (host)
};

struct ReserveParams {
  int64_t n_ctx, n_heads, max_rows, max_width;
};

class Backend {
 public:
  virtual ~Backend() = default;
  virtual bool supports(DType weight_type) const = 0;
  virtual void reserve(const ReserveParams&) = 0;
  virtual float* alloc(int64_t n_floats) = 0;
  virtual void free(float* p) = 0;
  virtual void read(float* host_dst, const float* src, int64_t n) = 0;
  virtual void embed(const Tensor& table, std::span<const int32_t> ids, float* out) = 0;
  virtual void matmul(const Tensor& w, const float* x, float* y, int64_t n) = 0;
  virtual void matmul_multi(std::span<const Tensor* const> ws, const float* x, std::span<float* const> ys, int64_t n) {
    for (size_t i = 0; i < ws.size(); ++i) matmul(*ws[i], x, ys[i], n);
  }
  virtual void rmsnorm(const float* x, const Tensor& weight, float* y, int64_t n, float eps) = 0;
  virtual void add(float* x, const float* y, int64_t count) = 0;
  virtual void add_bias(float* x, const Tensor& bias, int64_t n) = 0;
  virtual void rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, const RopeParams&) = 0;
  virtual void copy(float* dst, const float* src, int64_t count) = 0;
  virtual void attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                         int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) = 0;
  virtual void silu_mul(float* gate, const float* up, int64_t count) = 0;
};

}  // namespace nibble
