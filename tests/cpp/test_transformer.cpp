// nibble's own Transformer (src/model/transformer.cpp, compiled unchanged from the reference tree into
// oracle/_ref/libnibble_ref.so) run twice on the same small random model: over nibble's CpuBackend and over this
// repository's CudaBackend. The logits of a chunked prefill and of single-token decode steps must agree.
//
// This is the drop-in check of the backend as a whole: the model code, its op order, its pointer arithmetic into
// the KV cache (K/V projected straight into cache rows, transformer.cpp:171-180) and its buffer sizes are the
// reference's; only the Backend object differs. Built by oracle/Makefile (target model-check) where the
// reference tree is present; tests/test_gpu_transformer.py runs it on a GPU.
//
// Two model variants: "qwen2"-style (Q/K/V biases, NeoX rope, theta 1e6) with F16 projection weights, and
// "llama"-style (no biases, interleaved rope with per-pair frequency factors, theta 5e5) with F32 weights. The
// prompt is longer than max_batch, so prefill runs in chunks (SGEMM-sized and GEMV-sized) before the decode steps.
//
// Tolerance: per logit vector, max |gpu - cpu| <= 1e-4 * max |cpu| (the reference's own model-level bound against
// a naive fp64 forward, tests/test_model.cpp:110-151), and the same argmax.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "cuda_backend.h"
#include "fp16.h"
#include "model/transformer.h"
#include "thread_pool.h"

using namespace nibble;

namespace {

struct Model {
  model::LlamaConfig c;
  model::Weights w;
  std::vector<std::vector<float>> f32;      // storage behind the F32 tensors
  std::vector<std::vector<uint16_t>> f16;   // storage behind the F16 tensors
};

Tensor view(DType t, int n_dims, int64_t ne0, int64_t ne1, const void* data) {
  Tensor x;
  x.type = t;
  x.n_dims = n_dims;
  x.ne = {ne0, ne1, 1, 1};
  x.data = data;
  return x;
}

// A weight matrix [out rows][in] of N(0, 1/in) values, stored F16 or F32.
Tensor matrix(Model& m, std::mt19937_64& rng, int64_t in, int64_t out, bool f16) {
  std::normal_distribution<float> nd(0.f, 1.f / std::sqrt(static_cast<float>(in)));
  std::vector<float> v(static_cast<size_t>(in * out));
  for (float& x : v) x = nd(rng);
  if (f16) {
    std::vector<uint16_t> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = fp32_to_fp16(v[i]);
    m.f16.push_back(std::move(h));
    return view(DType::F16, 2, in, out, m.f16.back().data());
  }
  m.f32.push_back(std::move(v));
  return view(DType::F32, 2, in, out, m.f32.back().data());
}

Tensor vec(Model& m, std::mt19937_64& rng, int64_t n, float mean, float sd) {
  std::normal_distribution<float> nd(mean, sd);
  std::vector<float> v(static_cast<size_t>(n));
  for (float& x : v) x = nd(rng);
  m.f32.push_back(std::move(v));
  return view(DType::F32, 1, n, 1, m.f32.back().data());
}

void build(Model& m, bool qwen, uint64_t seed) {
  std::mt19937_64 rng(seed);
  auto& c = m.c;
  c.arch = qwen ? "qwen2" : "llama";
  c.n_layers = 2;
  c.n_embd = 256;
  c.n_ff = 512;
  c.n_heads = qwen ? 4 : 8;
  c.n_kv_heads = 2;
  c.head_dim = c.n_embd / c.n_heads;
  c.n_vocab = 3000;
  c.n_ctx_train = 4096;
  c.rope_base = qwen ? 1e6f : 5e5f;
  c.rms_eps = 1e-6f;
  c.rope_neox = qwen;
  c.qkv_bias = qwen;
  m.f32.reserve(64);  // tensors keep pointers into these vectors: no reallocation of the outer vectors
  m.f16.reserve(64);
  const bool f16 = qwen;
  const int64_t E = c.n_embd, Q = c.n_heads * c.head_dim, KV = c.n_kv_heads * c.head_dim;
  m.w.token_embd = matrix(m, rng, E, c.n_vocab, f16);
  m.w.output_norm = vec(m, rng, E, 1.f, 0.1f);
  m.w.output = matrix(m, rng, E, c.n_vocab, f16);
  if (!qwen) {
    std::vector<float> ff(static_cast<size_t>(c.head_dim / 2));
    for (size_t i = 0; i < ff.size(); ++i) ff[i] = i < ff.size() / 2 ? 1.f : 8.f;  // llama-3 style low/high bands
    m.f32.push_back(std::move(ff));
    m.w.rope_freqs = view(DType::F32, 1, c.head_dim / 2, 1, m.f32.back().data());
  }
  for (int64_t l = 0; l < c.n_layers; ++l) {
    model::LayerWeights L;
    L.attn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.wq = matrix(m, rng, E, Q, f16);
    L.wk = matrix(m, rng, E, KV, f16);
    L.wv = matrix(m, rng, E, KV, f16);
    L.wo = matrix(m, rng, Q, E, f16);
    L.ffn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.w_gate = matrix(m, rng, E, c.n_ff, f16);
    L.w_up = matrix(m, rng, E, c.n_ff, f16);
    L.w_down = matrix(m, rng, c.n_ff, E, f16);
    if (qwen) {
      L.bq = vec(m, rng, Q, 0.f, 0.5f);
      L.bk = vec(m, rng, KV, 0.f, 0.5f);
      L.bv = vec(m, rng, KV, 0.f, 0.5f);
    }
    m.w.layers.push_back(L);
  }
}

int failures = 0;

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
  const bool ok = rel <= 1e-4 && am_g == am_c;
  std::printf("%-34s max|gpu-cpu|/max|cpu| = %.3e  argmax %zu/%zu  %s\n", what, rel, am_g, am_c, ok ? "ok" : "FAIL");
  if (!ok) ++failures;
}

void run(bool qwen) {
  Model m;
  build(m, qwen, qwen ? 11 : 22);
  const int64_t n_ctx = 256, max_batch = 32;
  ThreadPool pool(4);
  cpu::CpuBackend cpu_be(pool);
  cuda::CudaBackend gpu_be(0);
  if (!gpu_be.supports(qwen ? DType::F16 : DType::F32)) {
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
  const std::string tag = qwen ? "qwen2/F16" : "llama/F32";
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
    run(true);
    run(false);
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
