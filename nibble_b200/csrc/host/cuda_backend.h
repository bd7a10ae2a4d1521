#pragma once
// nibble::cuda::CudaBackend -- the Backend implementation nibble's Transformer can be handed instead of
// CpuBackend (the single wiring point is src/nibble.cpp:69,81 in the reference). It sits above the C ABI
// (include/nibble_cuda.h) and keeps the reference's contracts:
//   * activations are opaque device pointers from alloc() (zeroed), released by free() or the destructor
//     (CpuBackend::~CpuBackend, src/backend/cpu/cpu_backend.cpp:70-72);
//   * input/resource faults throw nibble::Error with the C layer's message (include/nibble/error.h);
//   * after reserve(), attention/rope within the reserved sizes allocate nothing.
// Weights arrive as host Tensor views (the mmap'd GGUF); the ones this backend consumes (biases) are uploaded
// once and cached by host address.
//
// Coverage: the attention path -- reserve, alloc, free, read, add_bias, rope, attention -- runs on the GPU. The
// weight GEMMs and the remaining elementwise ops (embed, matmul, rmsnorm, add, copy, silu_mul) are not part of
// this backend yet: supports() reports no weight type, so a model refuses to load on it instead of silently
// running anything on the CPU, and those ops throw nibble::Error.
//
// The paged fp16/bf16 fast path (fused append, split-K decode, tcgen05 prefill) is reached through handle()
// and the nbl_* functions, with check() turning their statuses into nibble::Error.
#include <unordered_map>

#include "../../../include/nibble_cuda.h"
#include "backend.h"

namespace nibble::cuda {

// Throws nibble::Error carrying nbl_last_error() when status != NBL_OK.
void check(int status);

class CudaBackend final : public Backend {
 public:
  explicit CudaBackend(int device = 0);
  ~CudaBackend() override;
  CudaBackend(const CudaBackend&) = delete;
  CudaBackend& operator=(const CudaBackend&) = delete;

  bool supports(DType) const override { return false; }
  void reserve(const ReserveParams& rp) override;
  float* alloc(int64_t n_floats) override;
  void free(float* p) override;
  void read(float* host_dst, const float* src, int64_t n) override;
  void add_bias(float* x, const Tensor& bias, int64_t n) override;
  void rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, const RopeParams& p) override;
  void attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0, int64_t n_heads,
                 int64_t n_kv_heads, int64_t head_dim) override;

  void embed(const Tensor&, std::span<const int32_t>, float*) override { unsupported("embed"); }
  void matmul(const Tensor&, const float*, float*, int64_t) override { unsupported("matmul"); }
  void rmsnorm(const float*, const Tensor&, float*, int64_t, float) override { unsupported("rmsnorm"); }
  void add(float*, const float*, int64_t) override { unsupported("add"); }
  void copy(float*, const float*, int64_t) override { unsupported("copy"); }
  void silu_mul(float*, const float*, int64_t) override { unsupported("silu_mul"); }

  // Host -> device upload into a block from alloc() (tests and callers that stage inputs).
  void write(float* dst, const float* host_src, int64_t n);
  // Waits for queued work; throws Error if a kernel flagged an out-of-range device-side index.
  void synchronize();
  nbl_ctx* handle() const { return ctx_; }

 private:
  [[noreturn]] static void unsupported(const char* op);
  const float* device_weight(const Tensor& t, int64_t n_floats);

  nbl_ctx* ctx_ = nullptr;
  std::unordered_map<const void*, float*> weights_;  // host weight address -> uploaded copy
};

}  // namespace nibble::cuda
