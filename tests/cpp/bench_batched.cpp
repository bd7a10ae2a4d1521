// Aggregate decode throughput of BatchedDecoder (nibble_b200/csrc/host/batched_decoder.h): N sequences of one
// model decoding together, against the reference's serving model of one Session per Model, whose throughput for N
// users is one sequence's tg rate (nibble's Transformer decodes one token of one sequence per forward pass).
//
//   nbl_batched_bench [--shape tinyllama|qwen05] [--type F16|F32|Q4_0|Q5_0|Q8_0|Q5_1|Q4_K|Q5_K|Q6_K] [-p 128] [-n 64]
//                     [--seqs 1,8,32,64] [--out file.jsonl]
//
// For each N: N sequences are opened and each is prefilled with a P-token prompt (token i % n_vocab, shifted per
// sequence), then n decode steps run all N sequences at once (greedy argmax fed back); the timed region is the n
// steps, wall clock as `nibble bench` measures (cli/cmd_bench.cpp:140-253), logits copied to the host every step.
// Random in-memory model of the named shape (no model file exists here). Built by oracle/Makefile (target
// batched-bench) where the reference tree is present.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <ctime>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "batched_decoder.h"
#include "random_model.h"

using namespace nibble;

namespace {

nbl_test::Shape shape_of(const std::string& name, DType t) {
  if (name == "tinyllama") return {false, t, 22, 2048, 5632, 32, 4, 32000};
  if (name == "qwen05") return {true, t, 24, 896, 4864, 14, 2, 151936};
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
  throw Error("unknown --type '" + name + "'");
}

}  // namespace

int main(int argc, char** argv) {
  std::string shape_name = "tinyllama", type_name = "F16", out_path, seq_list = "1,8,32,64";
  long p = 128, n = 64;
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string a = argv[i], v = argv[i + 1];
    if (a == "--shape") shape_name = v;
    else if (a == "--type") type_name = v;
    else if (a == "-p") p = std::stol(v);
    else if (a == "-n") n = std::stol(v);
    else if (a == "--seqs") seq_list = v;
    else if (a == "--out") out_path = v;
    else {
      std::fprintf(stderr, "unknown argument %s\n", a.c_str());
      return 2;
    }
  }
  try {
    std::vector<int> counts;
    std::stringstream ss(seq_list);
    for (std::string tok; std::getline(ss, tok, ',');) counts.push_back(std::stoi(tok));
    const int max_n = *std::max_element(counts.begin(), counts.end());
    nbl_test::Model m;
    nbl_test::build(m, shape_of(shape_name, type_of(type_name)), 1234);
    cuda::CudaBackend be(0);
    const int64_t V = m.c.n_vocab;
    cuda::BatchedDecoder bd(be, m.c, m.w, max_n, p + n + 1, 0, 512);
    std::ofstream out;
    if (!out_path.empty()) out.open(out_path, std::ios::app);
    std::vector<float> logits(static_cast<size_t>(max_n * V));
    std::printf("%-8s %6s %12s %12s %10s\n", "model", "seqs", "tok/s", "ms/step", "prefill");
    for (int N : counts) {
      std::vector<int> ids;
      const auto t0 = std::chrono::steady_clock::now();
      for (int s = 0; s < N; ++s) {
        const int id = bd.open();
        std::vector<int32_t> prompt(static_cast<size_t>(p));
        for (long i = 0; i < p; ++i) prompt[static_cast<size_t>(i)] = static_cast<int32_t>((i + 7 * s) % V);
        bd.prefill(id, prompt, logits.data() + static_cast<int64_t>(s) * V);
        ids.push_back(id);
      }
      const double pre_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      std::vector<int32_t> toks(static_cast<size_t>(N));
      auto pick = [&] {
        for (int s = 0; s < N; ++s) {
          const float* row = logits.data() + static_cast<int64_t>(s) * V;
          toks[static_cast<size_t>(s)] = static_cast<int32_t>(std::max_element(row, row + V) - row);
        }
      };
      pick();
      bd.decode(ids, toks, logits.data());  // warm-up step (first use of the batch sizes)
      pick();
      const auto t1 = std::chrono::steady_clock::now();
      for (long step = 1; step < n; ++step) {
        bd.decode(ids, toks, logits.data());
        pick();
      }
      const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count();
      const double tps = static_cast<double>(N) * static_cast<double>(n - 1) / el;
      std::printf("%-8s %6d %12.1f %12.3f %9.2fs\n", shape_name.c_str(), N, tps, 1e3 * el / static_cast<double>(n - 1),
                  pre_s);
      if (out.is_open()) {
        char line[512];
        std::snprintf(line, sizeof line,
                      "{\"tool\":\"nbl_batched_bench\",\"model\":\"random %s %s\",\"sequences\":%d,\"prompt\":%ld,"
                      "\"steps\":%ld,\"decode_tok_s\":%.2f,\"ms_per_step\":%.4f,\"prefill_s\":%.3f}\n",
                      shape_name.c_str(), type_name.c_str(), N, p, n - 1, tps, 1e3 * el / static_cast<double>(n - 1),
                      pre_s);
        out << line;
      }
      for (int id : ids) bd.close(id);
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
