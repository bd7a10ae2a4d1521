// BatchedDecoder (many sequences over one model, nibble_b200/csrc/host/batched_decoder.h) against nibble's own
// Transformer on CpuBackend: every sequence served by the batched decoder must produce the logits that nibble's
// single-sequence Transformer produces for the same tokens, whichever other sequences share its decode steps.
//
// Scenario per model: five sequences with prompts of 7, 16, 33, 1 and 20 tokens (page boundaries inside and at the
// end of a prompt) are prefilled one by one; then 12 decode steps: all open sequences together on even steps, a
// subset on odd steps; after step 5 one sequence is closed and a new one (its pages reused) is opened and
// prefilled mid-stream. Each sequence has its own CPU Transformer fed exactly the same tokens (greedy argmax of the
// CPU logits). Also: a prompt longer than the prefill chunk, and the pool-exhausted and bad-id errors.
//
// Tolerance: per logit vector max |gpu - cpu| <= tol * max |cpu|, and the same argmax unless the CPU's top two are
// closer than twice the bound. The batched decoder keeps K/V as fp16 pages where the reference keeps fp32 rows, so
// its attention inputs carry fp16 rounding (relative 2^-11); everything else is the same arithmetic as CudaBackend's.
// Float weights: tol = 5e-3 (measured worst 7e-4). Quantized weights: tol = 2e-2 (measured worst 8e-3) -- the
// reference quantizes every matmul input to Q8_0 (127 levels per 32-element block), so an activation that differs
// by an fp16 rounding can land on the neighbouring level, a difference of one quantization step (~1/254 of the
// block's largest value) instead of one rounding of the input. Q4_K: tol = 3e-2 (measured worst 2.5e-2); its
// activations are Q8_K blocks of 256, whose step is set by the largest of 256 values rather than 32.
// Built by oracle/Makefile (target batched-check) where the reference tree is present.
#include <cmath>
#include <cstdio>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "batched_decoder.h"
#include "random_model.h"
#include "thread_pool.h"

using namespace nibble;

namespace {

int failures = 0;
double worst = 0, tol = 5e-3;

size_t argmax(const float* v, int64_t n) {
  size_t a = 0;
  for (int64_t i = 1; i < n; ++i)
    if (v[i] > v[a]) a = static_cast<size_t>(i);
  return a;
}

void compare(const std::string& what, const float* gpu, const std::vector<float>& cpu) {
  double mx = 0, err = 0;
  for (size_t i = 0; i < cpu.size(); ++i) {
    mx = std::max(mx, static_cast<double>(std::fabs(cpu[i])));
    err = std::max(err, static_cast<double>(std::fabs(gpu[i] - cpu[i])));
    if (!std::isfinite(gpu[i])) err = INFINITY;
  }
  const double rel = err / mx;
  const size_t ac = argmax(cpu.data(), static_cast<int64_t>(cpu.size()));
  const size_t ag = argmax(gpu, static_cast<int64_t>(cpu.size()));
  float second = -INFINITY;
  for (size_t i = 0; i < cpu.size(); ++i)
    if (i != ac) second = std::max(second, cpu[i]);
  const bool tie = cpu[ac] - second < 2 * tol * mx;
  const bool ok = rel <= tol && (ag == ac || tie);
  worst = std::max(worst, rel);
  if (!ok) {
    std::printf("%-40s max|gpu-cpu|/max|cpu| = %.3e  argmax %zu/%zu  FAIL\n", what.c_str(), rel, ag, ac);
    ++failures;
  }
}

struct Ref {  // one sequence on nibble's own Transformer (CpuBackend, fp32 KV)
  std::unique_ptr<model::Transformer> tf;
  int64_t pos = 0;
  std::vector<float> logits;
};

void run(bool qwen, DType wtype) {
  worst = 0;
  tol = wtype == DType::F16 || wtype == DType::F32 ? 5e-3 : wtype == DType::Q4_K ? 3e-2 : 2e-2;
  nbl_test::Model m;
  // head_dim 64 (the paged kernels): qwen2-style 4 heads / 2 KV heads, llama-style 8 heads / 2 KV heads
  nbl_test::build(m, {qwen, wtype, 2, qwen ? 256 : 512, 512, qwen ? 4 : 8, 2, 3000}, 77 + static_cast<int>(wtype));
  const std::string tag =
      std::string(qwen ? "qwen2/" : "llama/") +
      (wtype == DType::F16 ? "F16" : wtype == DType::Q4_0 ? "Q4_0" : wtype == DType::Q4_K ? "Q4_K" : "F32");
  ThreadPool pool(4);
  cpu::CpuBackend cpu_be(pool);
  cuda::CudaBackend gpu_be(0);
  const int64_t n_ctx = 160, V = m.c.n_vocab;
  cuda::BatchedDecoder bd(gpu_be, m.c, m.w, 6, n_ctx, 0, 24);  // prefill chunks of 24: the 33-token prompt splits
  std::mt19937_64 rng(qwen ? 3 : 4);
  std::map<int, Ref> refs;
  std::vector<float> lg(static_cast<size_t>(6 * V));
  auto open_seq = [&](int len) {
    const int id = bd.open();
    Ref& r = refs[id];
    r.tf = std::make_unique<model::Transformer>(m.c, m.w, cpu_be, n_ctx);
    r.pos = 0;
    r.logits.assign(static_cast<size_t>(V), 0.f);
    std::vector<int32_t> prompt(static_cast<size_t>(len));
    for (auto& t : prompt) t = static_cast<int32_t>(rng() % static_cast<uint64_t>(V));
    r.tf->forward(prompt, 0, r.logits.data());
    r.pos = len;
    bd.prefill(id, prompt, lg.data());
    compare(tag + " prefill seq " + std::to_string(id) + " (" + std::to_string(len) + " tokens)", lg.data(), r.logits);
    if (bd.n_past(id) != len) {
      std::printf("%s n_past %lld != %d  FAIL\n", tag.c_str(), static_cast<long long>(bd.n_past(id)), len);
      ++failures;
    }
    return id;
  };
  for (int len : {7, 16, 33, 1, 20}) open_seq(len);
  for (int step = 0; step < 12; ++step) {
    if (step == 6) {  // close one sequence, open another that takes its pages, mid-stream
      const int victim = refs.begin()->first == 0 ? 1 : refs.begin()->first;
      const int64_t before = bd.free_pages();
      bd.close(victim);
      refs.erase(victim);
      if (bd.free_pages() <= before) {
        std::printf("%s close returned no pages  FAIL\n", tag.c_str());
        ++failures;
      }
      open_seq(12);
    }
    std::vector<int> ids;
    for (auto& [id, r] : refs)
      if (step % 2 == 0 || id % 2 == 1) ids.push_back(id);  // odd steps: a subset
    std::vector<int32_t> toks;
    for (int id : ids) toks.push_back(static_cast<int32_t>(argmax(refs[id].logits.data(), V)));
    bd.decode(ids, toks, lg.data());
    for (size_t i = 0; i < ids.size(); ++i) {
      Ref& r = refs[ids[i]];
      r.tf->forward(std::span<const int32_t>(&toks[i], 1), r.pos, r.logits.data());
      ++r.pos;
      compare(tag + " decode step " + std::to_string(step) + " seq " + std::to_string(ids[i]),
              lg.data() + static_cast<int64_t>(i) * V, r.logits);
    }
  }
  // errors: an unknown sequence, and a pool too small for the prompt
  std::string e1, e2;
  try {
    const int32_t t = 0;
    const int closed = refs.begin()->first;
    bd.close(closed);
    refs.erase(refs.begin());
    bd.decode(std::vector<int>{closed}, std::span<const int32_t>(&t, 1), lg.data());
  } catch (const Error& e) {
    e1 = e.what();
  }
  try {
    cuda::BatchedDecoder small(gpu_be, m.c, m.w, 2, n_ctx, 3, 24);  // 3 pages of 16 tokens per layer
    const int id = small.open();
    std::vector<int32_t> prompt(60, 1);
    small.prefill(id, prompt, lg.data());
  } catch (const Error& e) {
    e2 = e.what();
  }
  const bool ok1 = e1.find("not open") != std::string::npos, ok2 = e2.find("exhausted") != std::string::npos;
  std::printf("%-40s closed id: \"%s\"  small pool: \"%s\"  %s\n", (tag + " errors").c_str(), e1.c_str(), e2.c_str(),
              ok1 && ok2 ? "ok" : "FAIL");
  if (!ok1 || !ok2) ++failures;
  std::printf("%-40s worst max|gpu-cpu|/max|cpu| = %.3e (bound %.0e)\n", tag.c_str(), worst, tol);
}

}  // namespace

int main() {
  try {
    run(true, DType::F16);
    run(false, DType::F32);
    run(true, DType::Q4_0);
    run(false, DType::Q4_K);
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
