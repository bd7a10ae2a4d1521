// A random decoder-only model held in memory: nibble's LlamaConfig and Weights (Tensor views into host vectors),
// shaped like a qwen2 or llama GGUF model, for tests and measurements that run nibble's own Transformer without a
// model file. Values: projections N(0, 1/in), norms N(1, 0.1), biases N(0, 0.5); F16 or F32 projection weights.
#pragma once
#include <cmath>
#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "fp16.h"
#include "model/transformer.h"

namespace nbl_test {

using nibble::DType;
using nibble::Tensor;
namespace model = nibble::model;

struct Shape {
  bool qwen;  // qwen2 (Q/K/V biases, NeoX rope, theta 1e6) or llama (interleaved rope, freq factors, theta 5e5)
  bool f16;   // projection and embedding weights F16 (else F32)
  int64_t n_layers, n_embd, n_ff, n_heads, n_kv_heads, n_vocab;
};

struct Model {
  model::LlamaConfig c;
  model::Weights w;
  std::vector<std::vector<float>> f32;     // storage behind the F32 tensors
  std::vector<std::vector<uint16_t>> f16;  // storage behind the F16 tensors
};

inline Tensor view(DType t, int n_dims, int64_t ne0, int64_t ne1, const void* data) {
  Tensor x;
  x.type = t;
  x.n_dims = n_dims;
  x.ne = {ne0, ne1, 1, 1};
  x.data = data;
  return x;
}

// splitmix64 stream -> approximately normal values (sum of four uniforms, variance-matched): fast enough for
// billion-parameter models; the distribution only needs to be model-like.
struct Rng {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float normal(float mean, float sd) {
    const uint64_t a = next(), b = next();
    const float u = float(a & 0xFFFFFFFFu) + float(a >> 32) + float(b & 0xFFFFFFFFu) + float(b >> 32);
    return mean + sd * (u * (1.0f / 4294967296.0f) - 2.0f) * 1.7320508f;
  }
};

inline Tensor matrix(Model& m, Rng& rng, int64_t in, int64_t out, bool f16) {
  const float sd = 1.f / std::sqrt(static_cast<float>(in));
  if (f16) {
    std::vector<uint16_t> h(static_cast<size_t>(in * out));
    for (auto& x : h) x = nibble::fp32_to_fp16(rng.normal(0.f, sd));
    m.f16.push_back(std::move(h));
    return view(DType::F16, 2, in, out, m.f16.back().data());
  }
  std::vector<float> v(static_cast<size_t>(in * out));
  for (float& x : v) x = rng.normal(0.f, sd);
  m.f32.push_back(std::move(v));
  return view(DType::F32, 2, in, out, m.f32.back().data());
}

inline Tensor vec(Model& m, Rng& rng, int64_t n, float mean, float sd) {
  std::vector<float> v(static_cast<size_t>(n));
  for (float& x : v) x = rng.normal(mean, sd);
  m.f32.push_back(std::move(v));
  return view(DType::F32, 1, n, 1, m.f32.back().data());
}

// Fills m for the given shape (tensors point into m's vectors, which must not be copied afterwards).
inline void build(Model& m, const Shape& s, uint64_t seed) {
  Rng rng{seed};
  auto& c = m.c;
  c.arch = s.qwen ? "qwen2" : "llama";
  c.n_layers = s.n_layers;
  c.n_embd = s.n_embd;
  c.n_ff = s.n_ff;
  c.n_heads = s.n_heads;
  c.n_kv_heads = s.n_kv_heads;
  c.head_dim = c.n_embd / c.n_heads;
  c.n_vocab = s.n_vocab;
  c.n_ctx_train = 4096;
  c.rope_base = s.qwen ? 1e6f : 5e5f;
  c.rms_eps = 1e-6f;
  c.rope_neox = s.qwen;
  c.qkv_bias = s.qwen;
  const int64_t E = c.n_embd, Q = c.n_heads * c.head_dim, KV = c.n_kv_heads * c.head_dim;
  m.w.token_embd = matrix(m, rng, E, c.n_vocab, s.f16);
  m.w.output_norm = vec(m, rng, E, 1.f, 0.1f);
  m.w.output = matrix(m, rng, E, c.n_vocab, s.f16);
  if (!s.qwen) {
    std::vector<float> ff(static_cast<size_t>(c.head_dim / 2));
    for (size_t i = 0; i < ff.size(); ++i) ff[i] = i < ff.size() / 2 ? 1.f : 8.f;  // llama-3 style low/high bands
    m.f32.push_back(std::move(ff));
    m.w.rope_freqs = view(DType::F32, 1, c.head_dim / 2, 1, m.f32.back().data());
  }
  for (int64_t l = 0; l < c.n_layers; ++l) {
    model::LayerWeights L;
    L.attn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.wq = matrix(m, rng, E, Q, s.f16);
    L.wk = matrix(m, rng, E, KV, s.f16);
    L.wv = matrix(m, rng, E, KV, s.f16);
    L.wo = matrix(m, rng, Q, E, s.f16);
    L.ffn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.w_gate = matrix(m, rng, E, c.n_ff, s.f16);
    L.w_up = matrix(m, rng, E, c.n_ff, s.f16);
    L.w_down = matrix(m, rng, c.n_ff, E, s.f16);
    if (s.qwen) {
      L.bq = vec(m, rng, Q, 0.f, 0.5f);
      L.bk = vec(m, rng, KV, 0.f, 0.5f);
      L.bv = vec(m, rng, KV, 0.f, 0.5f);
    }
    m.w.layers.push_back(L);
  }
}

}  // namespace nbl_test
