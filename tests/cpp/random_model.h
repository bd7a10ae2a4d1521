// A random decoder-only model held in memory: nibble's LlamaConfig and Weights (Tensor views into host vectors),
// shaped like a qwen2 or llama GGUF model, for tests and measurements that run nibble's own Transformer without a
// model file. Values: projections N(0, 1/in) (or quantized blocks of that spread), norms N(1, 0.1), biases
// N(0, 0.5); F32, F16 or quantized (Q4_0, Q5_0, Q8_0, Q5_1, Q4_K, Q5_K, Q6_K) projection, embedding and output
// weights.
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
  bool qwen;    // qwen2 (Q/K/V biases, NeoX rope, theta 1e6) or llama (interleaved rope, freq factors, theta 5e5)
  DType wtype;  // projection, embedding and output weights: F32, F16 or a quantized type
  int64_t n_layers, n_embd, n_ff, n_heads, n_kv_heads, n_vocab;
};

struct Model {
  model::LlamaConfig c;
  model::Weights w;
  std::vector<std::vector<float>> f32;     // storage behind the F32 tensors
  std::vector<std::vector<uint16_t>> f16;  // storage behind the F16 and quantized tensors
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

// Quantized blocks (GGUF layout; 32 elements each, 256 for the k-quants): uniformly random value bits (and packed
// sub-block scales) with fp16 scales that give the row about the same spread as a float matrix of N(0, 1/in);
// Q5_1's minimum and Q4_K / Q5_K's dmin put the block's mean near zero.
inline Tensor quant_matrix(Model& m, Rng& rng, int64_t in, int64_t out, DType t) {
  const bool kq = t == DType::Q4_K || t == DType::Q5_K || t == DType::Q6_K;
  const int64_t bb = t == DType::Q4_0 ? 18 : t == DType::Q5_0 ? 22 : t == DType::Q5_1 ? 24 : t == DType::Q8_0 ? 34
                     : t == DType::Q4_K ? 144 : t == DType::Q5_K ? 176 : 210;
  // rms of the block's integer values (k-quants: of sub-block scale x value)
  const float rms = t == DType::Q4_0 ? 4.6f : t == DType::Q5_0 ? 9.2f : t == DType::Q5_1 ? 9.2f : t == DType::Q8_0 ? 73.9f
                    : t == DType::Q4_K ? 160.f : t == DType::Q5_K ? 330.f : 1370.f;
  const float sd = 1.f / std::sqrt(static_cast<float>(in)) / rms;
  const int64_t nb = in / (kq ? 256 : 32) * out;
  std::vector<uint16_t> raw(static_cast<size_t>((nb * bb + 1) / 2));
  auto* bytes = reinterpret_cast<uint8_t*>(raw.data());
  auto put = [](uint8_t* p, float v) {
    const uint16_t h = nibble::fp32_to_fp16(v);
    p[0] = static_cast<uint8_t>(h & 0xFF);
    p[1] = static_cast<uint8_t>(h >> 8);
  };
  for (int64_t b = 0; b < nb; ++b) {
    uint8_t* blk = bytes + b * bb;
    const float d = sd * (0.5f + static_cast<float>(rng.next() & 0xFFFF) / 65536.f);
    const int64_t first = t == DType::Q6_K ? 0 : t == DType::Q5_1 || t == DType::Q4_K || t == DType::Q5_K ? 4 : 2;
    for (int64_t i = first; i < bb; ++i) blk[i] = static_cast<uint8_t>(rng.next());
    if (t == DType::Q6_K) {
      put(blk + 208, d);
    } else {
      put(blk, d);
      if (t == DType::Q5_1) put(blk + 2, -15.5f * d);
      if (t == DType::Q4_K) put(blk + 2, 7.5f * d);
      if (t == DType::Q5_K) put(blk + 2, 15.5f * d);
    }
  }
  m.f16.push_back(std::move(raw));
  return view(t, 2, in, out, m.f16.back().data());
}

inline Tensor matrix(Model& m, Rng& rng, int64_t in, int64_t out, DType t) {
  if (t != DType::F32 && t != DType::F16) return quant_matrix(m, rng, in, out, t);
  const float sd = 1.f / std::sqrt(static_cast<float>(in));
  if (t == DType::F16) {
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
  m.w.token_embd = matrix(m, rng, E, c.n_vocab, s.wtype);
  m.w.output_norm = vec(m, rng, E, 1.f, 0.1f);
  m.w.output = matrix(m, rng, E, c.n_vocab, s.wtype);
  if (!s.qwen) {
    std::vector<float> ff(static_cast<size_t>(c.head_dim / 2));
    for (size_t i = 0; i < ff.size(); ++i) ff[i] = i < ff.size() / 2 ? 1.f : 8.f;  // llama-3 style low/high bands
    m.f32.push_back(std::move(ff));
    m.w.rope_freqs = view(DType::F32, 1, c.head_dim / 2, 1, m.f32.back().data());
  }
  for (int64_t l = 0; l < c.n_layers; ++l) {
    model::LayerWeights L;
    L.attn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.wq = matrix(m, rng, E, Q, s.wtype);
    L.wk = matrix(m, rng, E, KV, s.wtype);
    L.wv = matrix(m, rng, E, KV, s.wtype);
    L.wo = matrix(m, rng, Q, E, s.wtype);
    L.ffn_norm = vec(m, rng, E, 1.f, 0.1f);
    L.w_gate = matrix(m, rng, E, c.n_ff, s.wtype);
    L.w_up = matrix(m, rng, E, c.n_ff, s.wtype);
    L.w_down = matrix(m, rng, c.n_ff, E, s.wtype);
    if (s.qwen) {
      L.bq = vec(m, rng, Q, 0.f, 0.5f);
      L.bk = vec(m, rng, KV, 0.f, 0.5f);
      L.bv = vec(m, rng, KV, 0.f, 0.5f);
    }
    m.w.layers.push_back(L);
  }
}

}  // namespace nbl_test
