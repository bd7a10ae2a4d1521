// `nibble bench` (cli/cmd_bench.cpp:140-253) on this repository's CudaBackend, next to nibble's CpuBackend: nibble's
// own Transformer (src/model/transformer.cpp, compiled unchanged into oracle/_ref/libnibble_ref.so) timed the way
// the reference times it -- ppP = one forward of a P-token prompt at position 0, tgN = N single-token forwards
// (greedy argmax fed back) after one token at position 0, each repeated R times after an untimed warm-up, median /
// min / max tokens per second -- on a random in-memory model of a named shape (no model file exists here, so the
// loader and tokenizer are not involved; the prompt is token i % n_vocab as in the reference).
//
//   nbl_model_bench [--backend cuda|cpu] [--shape tinyllama|qwen05] [--type F16|F32|Q4_0|Q5_0|Q8_0|Q5_1|Q4_K|Q5_K|Q6_K] [-p 512]
//                   [-n 128] [-r 5] [-t threads] [--kv paged|flat] [--out file.jsonl]
// --kv (CUDA only): paged (default) keeps the K/V cache as fp16 pages served by the fused append, the split-K decode
// and the tcgen05 prefill kernels; flat keeps the reference's fp32 cache and the fp32 CUDA-core attention.
//
// Prints the reference's table and, with --out, appends its JSON line per test with a "backend" field added.
// Built by oracle/Makefile (target model-bench) where the reference tree is present.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <ctime>
#include <fstream>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "backend/cpu/cpu_backend.h"
#include "backend/cpu/simd/dispatch.h"
#include "cuda_backend.h"
#include "random_model.h"
#include "thread_pool.h"

using namespace nibble;
using clock_ = std::chrono::steady_clock;

namespace {

struct Stats {
  double med, mn, mx;
};

Stats stats(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  const size_t n = v.size();
  return {n % 2 ? v[n / 2] : (v[n / 2 - 1] + v[n / 2]) / 2, v.front(), v.back()};
}

double secs(clock_::time_point t0) { return std::chrono::duration<double>(clock_::now() - t0).count(); }

std::string iso_now() {
  const std::time_t t = std::time(nullptr);
  char b[32];
  std::tm tm{};
  gmtime_r(&t, &tm);
  std::strftime(b, sizeof b, "%Y-%m-%dT%H:%M:%SZ", &tm);
  return b;
}

nbl_test::Shape shape_of(const std::string& name, DType t) {
  if (name == "tinyllama") return {false, t, 22, 2048, 5632, 32, 4, 32000};  // TinyLlama-1.1B, llama
  if (name == "qwen05") return {true, t, 24, 896, 4864, 14, 2, 151936};     // Qwen2.5-0.5B, qwen2
  throw Error("unknown --shape '" + name + "' (tinyllama or qwen05)");
}

DType type_of(const std::string& name) {
  if (name == "F32") return DType::F32;
  if (name == "F16") return DType::F16;
  if (name == "Q4_0") return DType::Q4_0;
  if (name == "Q5_0") return DType::Q5_0;
  if (name == "Q8_0") return DType::Q8_0;
  if (name == "Q5_1") return DType::Q5_1;
  if (name == "Q4_K") return DType::Q4_K;
  if (name == "Q5_K") return DType::Q5_K;
  if (name == "Q6_K") return DType::Q6_K;
  throw Error("unknown --type '" + name + "' (F32, F16, Q4_0, Q5_0, Q8_0, Q5_1, Q4_K, Q5_K, Q6_K)");
}

}  // namespace

int main(int argc, char** argv) {
  std::string backend = "cuda", shape_name = "tinyllama", type_name = "F16", out_path, kv_mode = "paged";
  long p = 512, n = 128, r = 5;
  int threads = 0;
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string a = argv[i], v = argv[i + 1];
    if (a == "--backend") backend = v;
    else if (a == "--shape") shape_name = v;
    else if (a == "--type") type_name = v;
    else if (a == "-p") p = std::stol(v);
    else if (a == "-n") n = std::stol(v);
    else if (a == "-r") r = std::stol(v);
    else if (a == "-t") threads = std::stoi(v);
    else if (a == "--out") out_path = v;
    else if (a == "--kv") kv_mode = v;
    else {
      std::fprintf(stderr, "unknown argument %s\n", a.c_str());
      return 2;
    }
  }
  if (r < 1 || p < 1 || n < 1) {
    std::fprintf(stderr, "-p, -n and -r must be at least 1\n");
    return 2;
  }
  try {
    const nbl_test::Shape shape = shape_of(shape_name, type_of(type_name));
    nbl_test::Model m;
    nbl_test::build(m, shape, 1234);
    if (threads <= 0) threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    std::unique_ptr<ThreadPool> pool;
    std::unique_ptr<Backend> be;
    std::string kernels;
    if (backend == "cuda") {
      if (kv_mode != "paged" && kv_mode != "flat") throw Error("unknown --kv '" + kv_mode + "' (paged or flat)");
      be = std::make_unique<cuda::CudaBackend>(0, kv_mode == "paged");
      kernels = "cuda-sm100a-kv-" + kv_mode;
      threads = 1;
    } else {
      pool = std::make_unique<ThreadPool>(threads);
      be = std::make_unique<cpu::CpuBackend>(*pool);
      kernels = simd::kernel_set();
    }
    const int64_t n_ctx = std::max<int64_t>(p, n + 1) + 1;
    model::Transformer tf(m.c, m.w, *be, n_ctx);
    std::vector<int32_t> prompt(static_cast<size_t>(p));
    for (int64_t i = 0; i < p; ++i) prompt[static_cast<size_t>(i)] = static_cast<int32_t>(i % m.c.n_vocab);
    std::vector<float> logits(static_cast<size_t>(m.c.n_vocab));
    std::printf("%-8s %7s %10s %10s %10s\n", "test", "threads", "median", "min", "max");
    std::vector<double> pp, tg;
    for (long rep = -1; rep < r; ++rep) {  // rep -1 is the untimed warm-up (it also uploads the weights)
      auto t0 = clock_::now();
      tf.forward(prompt, 0, logits.data());
      const double pp_s = secs(t0);
      const int32_t first = 0;
      tf.forward(std::span<const int32_t>(&first, 1), 0, logits.data());
      t0 = clock_::now();
      for (long i = 0; i < n; ++i) {
        const int32_t next = static_cast<int32_t>(std::max_element(logits.begin(), logits.end()) - logits.begin());
        tf.forward(std::span<const int32_t>(&next, 1), 1 + i, logits.data());
      }
      const double tg_s = secs(t0);
      if (rep >= 0) {
        pp.push_back(static_cast<double>(p) / pp_s);
        tg.push_back(static_cast<double>(n) / tg_s);
      }
    }
    const std::string date = iso_now();
    std::ofstream out;
    if (!out_path.empty()) out.open(out_path, std::ios::app);
    const std::string model_name = "random " + shape_name + " " + type_name;
    for (int k = 0; k < 2; ++k) {
      const std::string test = (k == 0 ? "pp" + std::to_string(p) : "tg" + std::to_string(n));
      const Stats s = stats(k == 0 ? pp : tg);
      std::printf("%-8s %7d %10.2f %10.2f %10.2f  tok/s  (%s)\n", test.c_str(), threads, s.med, s.mn, s.mx,
                  backend.c_str());
      if (out.is_open()) {
        char line[512];
        std::snprintf(line, sizeof line,
                      "{\"tool\":\"nibble\",\"backend\":\"%s\",\"kernels\":\"%s\",\"model\":\"%s\",\"test\":\"%s\","
                      "\"threads\":%d,\"reps\":%ld,\"median\":%.4f,\"min\":%.4f,\"max\":%.4f,\"unit\":\"tok/s\","
                      "\"date\":\"%s\"}\n",
                      backend.c_str(), kernels.c_str(), model_name.c_str(), test.c_str(), threads, r, s.med, s.mn,
                      s.mx, date.c_str());
        out << line;
      }
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
