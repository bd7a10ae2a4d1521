// nibble's own Transformer (src/model/transformer.cpp, compiled unchanged from the reference tree into
// oracle/_ref/libnibble_ref.so) run twice on the same small random model: over nibble's CpuBackend and over this
// repository's CudaBackend. The logits of a chunked prefill and of single-token decode steps must agree.
//
// This is the drop-in check of the backend as a whole: the model code, its op order, its pointer arithmetic into
// the KV cache (K/V projected straight into cache rows, transformer.cpp:171-180) and its buffer sizes are the
// reference's; only the Backend object differs. Built by oracle/Makefile (target model-check) where the
// reference tree is present; tests/test_gpu_transformer.py runs it on a GPU.
//
// Model variants: "qwen2"-style (Q/K/V biases, NeoX rope, theta 1e6) with F16, Q4_0, Q5_0, Q6_K and Q5_1 weights,
// and "llama"-style (no biases, interleaved rope with per-pair frequency factors, theta 5e5) with F32, Q8_0, Q4_K
// and Q5_K weights.
// The prompt is longer than max_batch, so prefill runs in chunks (SGEMM-sized and GEMV-sized) before the decode
// steps.
//
// Tolerance: per logit vector, max |gpu - cpu| <= 1e-4 * max |cpu| for float weights (the reference's own
// model-level bound against a naive fp64 forward, tests/test_model.cpp:110-151), 2e-2 for quantized weights (whose
// matmuls re-quantize their inputs, see run()), and the same argmax.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "cuda_backend.h"
#include "random_model.h"
#include "thread_pool.h"

using namespace nibble;

namespace {

int failures = 0;
double tol = 1e-4;  // set per model by run()

void compare(const char* what, const std::vector<float>& gpu, const std::vector<float>& cpu) {
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

void run(bool qwen, DType wtype) {
  // Float weights: 1e-4. Quantized weights: the matmuls are bit-identical to the CPU's, but each one re-quantizes
  // its input to 8 bits, and a one-ulp difference in the float ops before it (rmsnorm, attention, silu) can move
  // an activation across a rounding boundary by one quantum (1/127 of its block's largest value), so the logits
  // are held to 2e-2 and the same argmax.
  tol = wtype == DType::F32 || wtype == DType::F16 ? 1e-4 : 2e-2;
  nbl_test::Model m;
  // qwen2-style: 4 heads of 64; llama-style: 8 heads of 32
  nbl_test::build(m, {qwen, wtype, 2, 256, 512, qwen ? 4 : 8, 2, 3000}, (qwen ? 11 : 22) + static_cast<int>(wtype));
  const int64_t n_ctx = 256, max_batch = 32;
  ThreadPool pool(4);
  cpu::CpuBackend cpu_be(pool);
  cuda::CudaBackend gpu_be(0);
  if (!gpu_be.supports(wtype)) {
    std::printf("CudaBackend does not support the weight type\n");
    ++failures;
    return;
  }
  model::Transformer t_cpu(m.c, m.w, cpu_be, n_ctx, max_batch);
  model::Transformer t_gpu(m.c, m.w, gpu_be, n_ctx, max_batch);
  std::mt19937_64 rng(qwen ? 5 : 6);
  std::vector<int32_t> prompt(70);
  for (auto& id : prompt) id = static_cast<int32_t>(rng() % static_cast<uint64_t>(m.c.n_vocab));
  std::vector<float> lc(static_cast<size_t>(m.c.n_vocab)), lg(lc.size());
  const std::string tag = std::string(qwen ? "qwen2/" : "llama/") + type_name(wtype);
  // prefill in chunks of 32, 32 and 6 rows
  t_cpu.forward(prompt, 0, lc.data());
  t_gpu.forward(prompt, 0, lg.data());
  compare((tag + " prefill 70 tokens").c_str(), lg, lc);
  // decode: feed the CPU's argmax back in, 5 steps, plus one 3-token continuation
  int64_t pos = static_cast<int64_t>(prompt.size());
  for (int step = 0; step < 5; ++step) {
    size_t am = 0;
    for (size_t i = 1; i < lc.size(); ++i)
      if (lc[i] > lc[am]) am = i;
    const int32_t tok = static_cast<int32_t>(am);
    t_cpu.forward(std::span<const int32_t>(&tok, 1), pos, lc.data());
    t_gpu.forward(std::span<const int32_t>(&tok, 1), pos, lg.data());
    compare((tag + " decode step " + std::to_string(step)).c_str(), lg, lc);
    ++pos;
  }
  const int32_t more[3] = {1, 2, 2999};
  t_cpu.forward(std::span<const int32_t>(more, 3), pos, lc.data());
  t_gpu.forward(std::span<const int32_t>(more, 3), pos, lg.data());
  compare((tag + " 3-token continuation").c_str(), lg, lc);
  // an out-of-range token id is an Error on both backends, with the reference's message
  const int32_t bad = static_cast<int32_t>(m.c.n_vocab);
  std::string e_cpu, e_gpu;
  try {
    t_cpu.forward(std::span<const int32_t>(&bad, 1), pos + 3, lc.data());
  } catch (const Error& e) {
    e_cpu = e.what();
  }
  try {
    t_gpu.forward(std::span<const int32_t>(&bad, 1), pos + 3, lg.data());
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
    run(true, DType::F16);
    run(false, DType::F32);
    run(true, DType::Q4_0);
    run(false, DType::Q8_0);
    run(true, DType::Q5_0);
    run(false, DType::Q4_K);
    run(true, DType::Q6_K);
    run(false, DType::Q5_K);
    run(true, DType::Q5_1);
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
