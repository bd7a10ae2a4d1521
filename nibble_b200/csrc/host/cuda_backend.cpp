// CudaBackend: nibble::Backend over the C ABI (see cuda_backend.h).
#include "cuda_backend.h"

#include <string>
#include <vector>

namespace nibble::cuda {

void check(int status) {
  if (status == NBL_OK) return;
  const size_t n = nbl_last_error(nullptr, 0);
  std::string msg(n, '\0');
  nbl_last_error(msg.data(), n + 1);
  throw Error("cuda backend: " + msg);
}

CudaBackend::CudaBackend(int device, bool paged_kv) {
  check(nbl_ctx_create(device, &ctx_));
  if (paged_kv) {
    const int st = nbl_ctx_set_paged_kv(ctx_, 1);
    if (st != NBL_OK) {
      nbl_ctx_destroy(ctx_);
      check(st);
    }
  }
}

CudaBackend::~CudaBackend() { nbl_ctx_destroy(ctx_); }  // releases the uploaded weights too

void CudaBackend::reserve(const ReserveParams& rp) {
  check(nbl_reserve(ctx_, rp.n_ctx, rp.n_heads, rp.max_rows, rp.max_width));
}

float* CudaBackend::alloc(int64_t n_floats) {
  float* p = nullptr;
  check(nbl_alloc(ctx_, n_floats, &p));
  return p;
}

void CudaBackend::free(float* p) { check(nbl_free(ctx_, p)); }

void CudaBackend::read(float* host_dst, const float* src, int64_t n) { check(nbl_read(ctx_, host_dst, src, n)); }

void CudaBackend::write(float* dst, const float* host_src, int64_t n) { check(nbl_write(ctx_, dst, host_src, n)); }

void CudaBackend::synchronize() { check(nbl_ctx_check(ctx_)); }

const nbl_weight* CudaBackend::device_weight(const Tensor& t) {
  auto it = weights_.find(t.data);
  if (it != weights_.end()) return it->second;
  if (!t.data) throw Error("cuda backend: weight tensor has no data");
  int32_t dt;
  switch (t.type) {
    case DType::F32: dt = NBL_F32; break;
    case DType::F16: dt = NBL_F16; break;
    case DType::Q4_0: dt = NBL_Q4_0; break;
    case DType::Q5_0: dt = NBL_Q5_0; break;
    case DType::Q8_0: dt = NBL_Q8_0; break;
    case DType::Q5_1: dt = NBL_Q5_1; break;
    case DType::Q4_K: dt = NBL_Q4_K; break;
    case DType::Q5_K: dt = NBL_Q5_K; break;
    case DType::Q6_K: dt = NBL_Q6_K; break;
    default: throw Error("cuda backend: unsupported weight dtype");
  }
  nbl_weight* w = nullptr;
  check(nbl_weight_create(ctx_, t.data, dt, t.ne[0], t.rows(), &w));
  weights_.emplace(t.data, w);
  return w;
}

// Backend::embed (src/backend/backend.h:54-55): ids stay host memory, as in the reference's span.
void CudaBackend::embed(const Tensor& table, std::span<const int32_t> ids, float* out) {
  check(nbl_embed(ctx_, device_weight(table), ids.data(), static_cast<int64_t>(ids.size()), out));
}

void CudaBackend::matmul(const Tensor& w, const float* x, float* y, int64_t n) {
  check(nbl_matmul(ctx_, device_weight(w), x, y, n));
}

void CudaBackend::matmul_multi(std::span<const Tensor* const> ws, const float* x, std::span<float* const> ys,
                               int64_t n) {
  if (ws.size() != ys.size()) throw Error("matmul_multi: weights and outputs differ in count");
  std::vector<const nbl_weight*> dw(ws.size());
  for (size_t i = 0; i < ws.size(); ++i) {
    if (ws[i]->ne[0] != ws[0]->ne[0]) return Backend::matmul_multi(ws, x, ys, n);  // one matmul per weight
    dw[i] = device_weight(*ws[i]);
  }
  check(nbl_matmul_multi(ctx_, dw.data(), static_cast<int32_t>(dw.size()), x, ys.data(), n));
}

void CudaBackend::rmsnorm(const float* x, const Tensor& weight, float* y, int64_t n, float eps) {
  if (weight.type != DType::F32) throw Error("rmsnorm: weight must be an F32 tensor");
  check(nbl_rmsnorm(ctx_, x, device_weight(weight), y, n, eps));
}

void CudaBackend::add(float* x, const float* y, int64_t count) { check(nbl_add(ctx_, x, y, count)); }

void CudaBackend::copy(float* dst, const float* src, int64_t count) { check(nbl_copy(ctx_, dst, src, count)); }

void CudaBackend::silu_mul(float* gate, const float* up, int64_t count) { check(nbl_silu_mul(ctx_, gate, up, count)); }

// Each of n rows += bias (F32 vector of width bias.ne[0]) -- CpuBackend::add_bias, cpu_backend.cpp:247-252.
void CudaBackend::add_bias(float* x, const Tensor& bias, int64_t n) {
  if (bias.type != DType::F32 || !bias.data) throw Error("add_bias: bias must be an F32 tensor");
  const void* b = nullptr;
  check(nbl_weight_data(device_weight(bias), &b, nullptr, nullptr, nullptr));
  check(nbl_add_bias(ctx_, x, static_cast<const float*>(b), bias.ne[0], n));
}

void CudaBackend::rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, const RopeParams& p) {
  const nbl_rope_params rp{p.freq_base, p.neox ? 1 : 0, p.freq_factors};
  check(nbl_rope(ctx_, x, n, n_heads, head_dim, pos0, &rp));
}

void CudaBackend::attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                            int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
  check(nbl_attention(ctx_, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim));
}

}  // namespace nibble::cuda
