// nibble's own Transformer (src/model/transformer.cpp, compiled unchanged from the reference tree into
// oracle/_ref/libnibble_ref.so) run on the same small random model over nibble's CpuBackend and over this
// repository's CudaBackend, in both of its K/V modes. The logits of a chunked prefill and of single-token decode
// steps must agree, and in the paged mode every layer's attention output is checked on its own.
//
// This is the drop-in check of the backend as a whole: the model code, its op order, its pointer arithmetic into
// the KV cache (K/V projected straight into cache rows, transformer.cpp:171-180) and its buffer sizes are the
// reference's; only the Backend object differs. Built by oracle/Makefile (target model-check) where the
// reference tree is present; tests/test_gpu_transformer.py runs it on a GPU.
//
// Backends compared with CpuBackend:
//   * flat  -- CudaBackend(0, false): the reference's fp32 K/V blocks and the fp32 CUDA-core attention kernels.
//   * paged -- CudaBackend(0, true), the default: K/V blocks held as fp16 pages, the bias + RoPE + append fused into
//     one launch, the split-K decode kernel for chunks of up to 8 rows and the tcgen05 prefill kernel above.
//   * paged, checked -- the same behind CheckingBackend, which after every attention() reads back the roped
//     queries, the cache (fp16 values) and the output, and holds the output against nibble's own scalar
//     cpu::attention_heads (src/backend/cpu/ref_ops.cpp:188-214) on those same inputs: decode rows (fp32
//     accumulate) to a max relative error of 1e-4 per (row, head), prefill chunks (fp16 operands on the tensor
//     cores) to max abs error 2e-2 and cosine >= 0.9999 per head. Reading the cache turns the pages back into flat
//     rows and the next attention() converts them again, which must not change a single bit: its logits are
//     required to equal the unchecked paged run's exactly.
//
// Models: "qwen2"-style (Q/K/V biases, NeoX rope, theta 1e6, 4 heads of 64, 2 KV heads) with F16, Q4_0, Q5_0, Q6_K
// and Q5_1 weights; "llama"-style (no biases, interleaved rope with per-pair frequency factors, theta 5e5) with 4
// heads of 64 (F32, F16) and 8 heads of 32 (Q8_0, Q4_K, Q5_K; head_dim 32 stays on the flat path in both modes).
// The prompt is longer than max_batch, so prefill runs in chunks (GEMM-sized and GEMV-sized) before the decode
// steps.
//
// Logit tolerance, per logit vector, max |gpu - cpu| / max |cpu|, and the same argmax:
//   flat: 1e-4 for float weights (the reference's own model-level bound against a naive fp64 forward,
//         tests/test_model.cpp:110-151), 2e-2 for quantized weights (their matmuls re-quantize their inputs, see run());
//   paged: 2e-3 for float weights -- K/V rounded to fp16 (2^-11 relative) and the prefill chunks' queries and softmax
//          weights fed to the tensor cores in fp16; quantized weights 3e-2.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "backend/cpu/ref_ops.h"
#include "cuda_backend.h"
#include "fp16.h"
#include "random_model.h"
#include "thread_pool.h"

using namespace nibble;

namespace {

int failures = 0;

// A Backend that forwards every op to a CudaBackend and checks each head_dim-64 attention() against nibble's
// scalar attention on the inputs the GPU used.
class CheckingBackend final : public Backend {
 public:
  explicit CheckingBackend(cuda::CudaBackend& be) : be_(be) {}
  bool supports(DType t) const override { return be_.supports(t); }
  void reserve(const ReserveParams& rp) override { be_.reserve(rp); }
  float* alloc(int64_t n) override { return be_.alloc(n); }
  void free(float* p) override { be_.free(p); }
  void read(float* dst, const float* src, int64_t n) override { be_.read(dst, src, n); }
  void embed(const Tensor& t, std::span<const int32_t> ids, float* out) override { be_.embed(t, ids, out); }
  void matmul(const Tensor& w, const float* x, float* y, int64_t n) override { be_.matmul(w, x, y, n); }
  void matmul_multi(std::span<const Tensor* const> ws, const float* x, std::span<float* const> ys,
                    int64_t n) override {
    be_.matmul_multi(ws, x, ys, n);
  }
  void rmsnorm(const float* x, const Tensor& w, float* y, int64_t n, float eps) override { be_.rmsnorm(x, w, y, n, eps); }
  void add(float* x, const float* y, int64_t c) override { be_.add(x, y, c); }
  void add_bias(float* x, const Tensor& b, int64_t n) override { be_.add_bias(x, b, n); }
  void rope(float* x, int64_t n, int64_t h, int64_t d, int64_t pos0, const RopeParams& p) override {
    be_.rope(x, n, h, d, pos0, p);
  }
  void copy(float* dst, const float* src, int64_t c) override { be_.copy(dst, src, c); }
  void silu_mul(float* g, const float* u, int64_t c) override { be_.silu_mul(g, u, c); }

  void attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0, int64_t H,
                 int64_t KVH, int64_t D) override {
    be_.attention(q, k, v, out, n, pos0, H, KVH, D);
    if (D != 64) return;
    const int64_t len = pos0 + n;
    std::vector<float> o(static_cast<size_t>(n * H * D)), qq(o.size()), ref(o.size());
    std::vector<float> kk(static_cast<size_t>(len * KVH * D)), vv(kk.size()), scratch(static_cast<size_t>(len));
    be_.read(o.data(), out, n * H * D);
    be_.read(qq.data(), q, n * H * D);  // applies the recorded bias/rope of q: the roped queries
    be_.read(kk.data(), k, len * KVH * D);  // the cache as the kernels saw it (fp16 values)
    be_.read(vv.data(), v, len * KVH * D);
    const bool prefill = n > 8;
    if (prefill)
      for (float& x : qq) x = fp16_to_fp32(fp32_to_fp16(x));  // the prefill kernel's queries are fp16
    cpu::attention_heads(qq.data(), kk.data(), vv.data(), ref.data(), n, pos0, H, KVH, D, 0, H, scratch.data());
    ++checked_;
    for (int64_t h = 0; h < H; ++h) {
      double dot = 0, ng = 0, nr = 0, abs_err = 0;
      for (int64_t t = 0; t < n; ++t) {
        double mx = 0, err = 0;
        for (int64_t d = 0; d < D; ++d) {
          const size_t i = static_cast<size_t>((t * H + h) * D + d);
          mx = std::max(mx, std::fabs(static_cast<double>(ref[i])));
          err = std::max(err, std::fabs(static_cast<double>(o[i]) - ref[i]));
          if (!std::isfinite(o[i])) err = INFINITY;
          dot += static_cast<double>(o[i]) * ref[i];
          ng += static_cast<double>(o[i]) * o[i];
          nr += static_cast<double>(ref[i]) * ref[i];
        }
        abs_err = std::max(abs_err, err);
        if (!prefill) worst_rel_ = std::max(worst_rel_, err / std::max(mx, 1e-30));
      }
      if (prefill) {
        worst_abs_ = std::max(worst_abs_, abs_err);
        worst_cos_ = std::min(worst_cos_, dot / std::max(std::sqrt(ng * nr), 1e-300));
      }
    }
    if (prefill) ++prefill_calls_;
    else ++decode_calls_;
  }

  // Prints the worst errors seen and counts a failure if any exceeds its tolerance.
  void report(const std::string& tag) const {
    const bool ok = worst_rel_ <= 1e-4 && worst_abs_ <= 2e-2 && worst_cos_ >= 0.9999 && checked_ > 0;
    std::printf("%-34s %d decode calls: max rel err/head %.2e; %d prefill calls: max abs %.2e, min cos %.6f  %s\n",
                (tag + " per-layer attention").c_str(), decode_calls_, worst_rel_, prefill_calls_, worst_abs_,
                worst_cos_, ok ? "ok" : "FAIL");
    if (!ok) ++failures;
  }

 private:
  cuda::CudaBackend& be_;
  int checked_ = 0, decode_calls_ = 0, prefill_calls_ = 0;
  double worst_rel_ = 0, worst_abs_ = 0, worst_cos_ = 1;
};

void compare(const char* what, const std::vector<float>& gpu, const std::vector<float>& cpu, double tol) {
  double mx = 0, err = 0;
  size_t am_g = 0, am_c = 0;
  for (size_t i = 0; i < cpu.size(); ++i) {
    mx = std::max(mx, static_cast<double>(std::fabs(cpu[i])));
    err = std::max(err, static_cast<double>(std::fabs(gpu[i] - cpu[i])));
    if (!std::isfinite(gpu[i])) err = INFINITY;
    if (gpu[i] > gpu[am_g]) am_g = i;
    if (cpu[i] > cpu[am_c]) am_c = i;
  }
  const double rel = err / mx;
  const bool ok = rel <= tol && am_g == am_c;
  std::printf("%-34s max|gpu-cpu|/max|cpu| = %.3e  argmax %zu/%zu  %s\n", what, rel, am_g, am_c, ok ? "ok" : "FAIL");
  if (!ok) ++failures;
}

void same_bits(const char* what, const std::vector<float>& a, const std::vector<float>& b) {
  const bool ok = std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
  std::printf("%-34s %s\n", what, ok ? "identical bits ok" : "bits differ FAIL");
  if (!ok) ++failures;
}

const char* type_name(DType t) {
  switch (t) {
    case DType::F32: return "F32";
    case DType::F16: return "F16";
    case DType::Q4_0: return "Q4_0";
    case DType::Q5_0: return "Q5_0";
    case DType::Q8_0: return "Q8_0";
    case DType::Q5_1: return "Q5_1";
    case DType::Q4_K: return "Q4_K";
    case DType::Q5_K: return "Q5_K";
    case DType::Q6_K: return "Q6_K";
    default: return "?";
  }
}

void run(bool qwen, DType wtype, int64_t n_heads) {
  // Float weights: 1e-4 flat. Quantized weights: the matmuls are bit-identical to the CPU's, but each one
  // re-quantizes its input to 8 bits, and a one-ulp difference in the float ops before it (rmsnorm, attention, silu)
  // can move an activation across a rounding boundary by one quantum (1/127 of its block's largest value), so the
  // logits are held to 2e-2 and the same argmax. The paged mode adds the fp16 rounding of the cache (and of the
  // prefill chunks' queries and softmax weights).
  const bool quant = !(wtype == DType::F32 || wtype == DType::F16);
  const double tol_flat = quant ? 2e-2 : 1e-4, tol_paged = quant ? 3e-2 : 2e-3;
  nbl_test::Model m;
  nbl_test::build(m, {qwen, wtype, 2, 256, 512, n_heads, 2, 3000},
                  (qwen ? 11 : 22) + static_cast<int>(wtype) + static_cast<int>(n_heads));
  const int64_t n_ctx = 256, max_batch = 32;
  ThreadPool pool(4);
  cpu::CpuBackend cpu_be(pool);
  cuda::CudaBackend flat_be(0, false), paged_be(0, true), chk_inner(0, true);
  CheckingBackend chk_be(chk_inner);
  if (!flat_be.supports(wtype)) {
    std::printf("CudaBackend does not support the weight type\n");
    ++failures;
    return;
  }
  model::Transformer t_cpu(m.c, m.w, cpu_be, n_ctx, max_batch);
  model::Transformer t_flat(m.c, m.w, flat_be, n_ctx, max_batch);
  model::Transformer t_paged(m.c, m.w, paged_be, n_ctx, max_batch);
  model::Transformer t_chk(m.c, m.w, chk_be, n_ctx, max_batch);
  std::mt19937_64 rng(qwen ? 5 : 6);
  std::vector<int32_t> prompt(70);
  for (auto& id : prompt) id = static_cast<int32_t>(rng() % static_cast<uint64_t>(m.c.n_vocab));
  const size_t V = static_cast<size_t>(m.c.n_vocab);
  std::vector<float> lc(V), lf(V), lp(V), lk(V);
  const std::string tag = std::string(qwen ? "qwen2/" : "llama/") + type_name(wtype) + "/hd" +
                          std::to_string(m.c.head_dim);
  auto step = [&](std::span<const int32_t> toks, int64_t pos, const std::string& what) {
    t_cpu.forward(toks, pos, lc.data());
    t_flat.forward(toks, pos, lf.data());
    t_paged.forward(toks, pos, lp.data());
    t_chk.forward(toks, pos, lk.data());
    compare((tag + " flat  " + what).c_str(), lf, lc, tol_flat);
    compare((tag + " paged " + what).c_str(), lp, lc, tol_paged);
    same_bits((tag + " paged checked " + what).c_str(), lk, lp);
  };
  step(prompt, 0, "prefill 70");  // chunks of 32, 32 and 6 rows
  // decode: feed the CPU's argmax back in, 5 steps, plus one 3-token continuation
  int64_t pos = static_cast<int64_t>(prompt.size());
  for (int s = 0; s < 5; ++s) {
    size_t am = 0;
    for (size_t i = 1; i < V; ++i)
      if (lc[i] > lc[am]) am = i;
    const int32_t tok = static_cast<int32_t>(am);
    step(std::span<const int32_t>(&tok, 1), pos, "decode " + std::to_string(s));
    ++pos;
  }
  const int32_t more[3] = {1, 2, 2999};
  step(std::span<const int32_t>(more, 3), pos, "continue 3");
  pos += 3;
  // a 20-token chunk after the continuation: a prefill chunk over a cached prefix
  std::vector<int32_t> chunk(20);
  for (auto& id : chunk) id = static_cast<int32_t>(rng() % static_cast<uint64_t>(m.c.n_vocab));
  step(chunk, pos, "chunk 20 at " + std::to_string(pos));
  if (m.c.head_dim == 64) chk_be.report(tag);
  // an out-of-range token id is an Error on both backends, with the reference's message
  const int32_t bad = static_cast<int32_t>(m.c.n_vocab);
  std::string e_cpu, e_gpu;
  try {
    t_cpu.forward(std::span<const int32_t>(&bad, 1), pos, lc.data());
  } catch (const Error& e) {
    e_cpu = e.what();
  }
  try {
    t_paged.forward(std::span<const int32_t>(&bad, 1), pos, lp.data());
  } catch (const Error& e) {
    e_gpu = e.what();
  }
  const bool same = !e_cpu.empty() && e_gpu.find(e_cpu) != std::string::npos;
  std::printf("%-34s cpu \"%s\" / gpu \"%s\"  %s\n", (tag + " bad token id").c_str(), e_cpu.c_str(), e_gpu.c_str(),
              same ? "ok" : "FAIL");
  if (!same) ++failures;
}

}  // namespace

int main() {
  try {
    run(true, DType::F16, 4);
    run(false, DType::F32, 4);
    run(false, DType::F16, 4);
    run(true, DType::Q4_0, 4);
    run(false, DType::Q8_0, 8);
    run(true, DType::Q5_0, 4);
    run(false, DType::Q4_K, 8);
    run(true, DType::Q6_K, 4);
    run(false, DType::Q5_K, 8);
    run(true, DType::Q5_1, 4);
  } catch (const std::exception& e) {
    std::printf("exception: %s\n", e.what());
    return 2;
  }
  if (failures) {
    std::printf("%d check(s) failed\n", failures);
    return 1;
  }
  std::printf("all passed\n");
  return 0;
}
