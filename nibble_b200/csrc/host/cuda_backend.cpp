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

CudaBackend::CudaBackend(int device) { check(nbl_ctx_create(device, &ctx_)); }

CudaBackend::~CudaBackend() { nbl_ctx_destroy(ctx_); }

void CudaBackend::unsupported(const char* op) {
  throw Error(std::string("cuda backend: ") + op +
              " is not implemented on the GPU in this build (attention path only: reserve, alloc, free, read, "
              "add_bias, rope, attention)");
}

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

const float* CudaBackend::device_weight(const Tensor& t, int64_t n_floats) {
  auto it = weights_.find(t.data);
  if (it != weights_.end()) return it->second;
  float* d = alloc(n_floats);
  write(d, static_cast<const float*>(t.data), n_floats);
  weights_.emplace(t.data, d);
  return d;
}

// Each of n rows += bias (F32 vector of width bias.ne[0]) -- CpuBackend::add_bias, cpu_backend.cpp:247-252.
void CudaBackend::add_bias(float* x, const Tensor& bias, int64_t n) {
  if (bias.type != DType::F32 || !bias.data) throw Error("add_bias: bias must be an F32 tensor");
  const int64_t width = bias.ne[0];
  check(nbl_add_bias(ctx_, x, device_weight(bias, width), width, n));
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
