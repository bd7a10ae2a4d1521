#pragma once
// nibble::cuda::CudaBackend -- the Backend implementation nibble's Transformer can be handed instead of
// CpuBackend (the single wiring point is src/nibble.cpp:69,81 in the reference). It sits above the C ABI
// (include/nibble_cuda.h) and keeps the reference's contracts:
//   * activations are opaque device pointers from alloc() (zeroed), released by free() or the destructor
//     (CpuBackend::~CpuBackend, src/backend/cpu/cpu_backend.cpp:70-72);
//   * input/resource faults throw nibble::Error with the C layer's message (include/nibble/error.h);
//   * after reserve(), attention/rope within the reserved sizes allocate nothing.
// Weights arrive as host Tensor views (the mmap'd GGUF); each is uploaded once, on first use, and cached by host
// address (nbl_weight_create), so the first forward pass after construction allocates the model's device weights
// and later ones allocate nothing.
//
// Coverage: every Backend op runs on the GPU for every weight type the reference supports (F32, F16, Q4_0, Q5_0,
// Q8_0, Q5_1, Q4_K, Q5_K, Q6_K) -- embed, matmul (float: weight-streaming GEMV for up to 8 rows, tensor-core GEMM
// above; quantized: bit-identical to the CPU's block dots), rmsnorm, add, add_bias, rope, copy, attention, silu_mul --
// so nibble's Transformer (src/model/transformer.cpp) runs on it unchanged.
//
// Attention (the default, paged_kv = true): the Transformer's per-layer K/V blocks become fp16 pages the first time
// attention() sees them (head_dim 64), and the calls it makes per layer -- matmul_multi into the cache rows, add_bias,
// rope(q), rope(kc), attention (transformer.cpp:171-202) -- run as the matmul, ONE fused bias + RoPE + fp16 append
// launch and the split-K decode kernel (up to 8 query rows) or the tcgen05 prefill kernel (longer chunks); see
// nbl_ctx_set_paged_kv. Other head sizes keep the flat fp32 cache and the fp32 CUDA-core attention kernels.
// The same kernels over many sequences' pages are reached through handle() and the nbl_* functions (BatchedDecoder),
// with check() turning their statuses into nibble::Error.
#include <unordered_map>

#include "../../../include/nibble_cuda.h"
#ifdef NBL_WITH_NIBBLE_TREE
// Built inside a nibble tree (src/ and include/ on the include path): implement nibble's own interface header.
#include "backend/backend.h"
#include "nibble/error.h"
#else
#include "backend.h"  // this repository's restatement of src/backend/backend.h (identical declarations)
#endif

namespace nibble::cuda {

// Throws nibble::Error carrying nbl_last_error() when status != NBL_OK.
void check(int status);

class CudaBackend final : public Backend {
 public:
  // paged_kv: K/V blocks handed to attention() with head_dim 64 are kept as fp16 pages and served by the
  // split-K decode / tcgen05 prefill kernels with the bias + RoPE + append fused (nbl_ctx_set_paged_kv); false keeps
  // the reference's flat fp32 cache and the fp32 CUDA-core attention.
  explicit CudaBackend(int device = 0, bool paged_kv = true);
  ~CudaBackend() override;
  CudaBackend(const CudaBackend&) = delete;
  CudaBackend& operator=(const CudaBackend&) = delete;

  bool supports(DType t) const override {
    return t == DType::F32 || t == DType::F16 || t == DType::Q4_0 || t == DType::Q5_0 || t == DType::Q8_0 ||
           t == DType::Q5_1 || t == DType::Q4_K || t == DType::Q5_K || t == DType::Q6_K;
  }
  void reserve(const ReserveParams& rp) override;
  float* alloc(int64_t n_floats) override;
  void free(float* p) override;
  void read(float* host_dst, const float* src, int64_t n) override;
  void add_bias(float* x, const Tensor& bias, int64_t n) override;
  void rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, const RopeParams& p) override;
  void attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0, int64_t n_heads,
                 int64_t n_kv_heads, int64_t head_dim) override;

  void embed(const Tensor& table, std::span<const int32_t> ids, float* out) override;
  void matmul(const Tensor& w, const float* x, float* y, int64_t n) override;
  // One launch for the weights sharing x at decode sizes (the reference's contract: equal to separate calls).
  void matmul_multi(std::span<const Tensor* const> ws, const float* x, std::span<float* const> ys, int64_t n) override;
  void rmsnorm(const float* x, const Tensor& weight, float* y, int64_t n, float eps) override;
  void add(float* x, const float* y, int64_t count) override;
  void copy(float* dst, const float* src, int64_t count) override;
  void silu_mul(float* gate, const float* up, int64_t count) override;

  // Host -> device upload into a block from alloc() (tests and callers that stage inputs).
  void write(float* dst, const float* host_src, int64_t n);
  // Waits for queued work; throws Error if a kernel flagged an out-of-range device-side index.
  void synchronize();
  nbl_ctx* handle() const { return ctx_; }
  // The device copy of a weight Tensor (uploaded on first use, cached by host address); shared with code that runs
  // the same model through the nbl_* calls directly (BatchedDecoder).
  const nbl_weight* device_weight(const Tensor& t);

 private:

  nbl_ctx* ctx_ = nullptr;
  std::unordered_map<const void*, nbl_weight*> weights_;  // host weight address -> uploaded tensor
};

}  // namespace nibble::cuda
