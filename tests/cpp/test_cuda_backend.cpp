// C++ tests of nibble::cuda::CudaBackend (the Backend implementation over the C ABI), written the way the
// reference tests its CPU backend (tests/test_cpu_backend.cpp in nibble): same cases, the scalar oracle as the
// expected value. Built and run by tests/test_gpu_cpp.py (needs a GPU). Exit status 0 = all passed.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "../../nibble_b200/csrc/host/cuda_backend.h"
#include "../../oracle/nbl_oracle.h"

using nibble::cuda::CudaBackend;

static int g_failed = 0;
#define CHECK(cond)                                                          \
  do {                                                                       \
    if (!(cond)) {                                                           \
      std::fprintf(stderr, "%s:%d: CHECK(%s) failed\n", __FILE__, __LINE__, #cond); \
      ++g_failed;                                                            \
    }                                                                        \
  } while (0)

static std::vector<float> rnd(size_t n, std::mt19937& g, float scale = 1.f) {
  std::normal_distribution<float> d(0.f, scale);
  std::vector<float> v(n);
  for (auto& x : v) x = d(g);
  return v;
}

static float maxdiff(const float* a, const float* b, size_t n) {
  float m = 0;
  for (size_t i = 0; i < n; ++i) m = std::fmax(m, std::fabs(a[i] - b[i]));
  return m;
}

// Backend attention agrees with the scalar attention for a grouped-query case, twice in a row (scratch reuse):
// the reference's "cpu backend attention" case (n=7, pos0=3, H=6, KV=2, D=16).
static void attention_case(CudaBackend& be) {
  std::mt19937 g(2);
  const int64_t n = 7, pos0 = 3, H = 6, KV = 2, D = 16, ctx = pos0 + n;
  auto q = rnd(n * H * D, g), k = rnd(ctx * KV * D, g), v = rnd(ctx * KV * D, g);
  std::vector<float> ref(n * H * D), got(n * H * D);
  CHECK(orc_attention(q.data(), k.data(), v.data(), ref.data(), n, pos0, H, KV, D) == 0);
  float* dq = be.alloc(n * H * D);
  float* dk = be.alloc(ctx * KV * D);
  float* dv = be.alloc(ctx * KV * D);
  float* out = be.alloc(n * H * D);
  be.write(dq, q.data(), n * H * D);
  be.write(dk, k.data(), ctx * KV * D);
  be.write(dv, v.data(), ctx * KV * D);
  for (int rep = 0; rep < 2; ++rep) {
    be.attention(dq, dk, dv, out, n, pos0, H, KV, D);
    be.read(got.data(), out, n * H * D);
    CHECK(maxdiff(ref.data(), got.data(), ref.size()) <= 1e-5f);
  }
  for (float* p : {dq, dk, dv, out}) be.free(p);
}

// Decode at every position of a reserved context, as the Transformer runs it after reserve().
static void reserve_then_decode(CudaBackend& be) {
  be.reserve({64, 6, 1, 32});
  std::mt19937 g(3);
  const int64_t H = 6, KV = 2, D = 16;
  auto k = rnd(64 * KV * D, g), v = rnd(64 * KV * D, g), q = rnd(H * D, g);
  float* dk = be.alloc(64 * KV * D);
  float* dv = be.alloc(64 * KV * D);
  float* dq = be.alloc(H * D);
  float* out = be.alloc(H * D);
  be.write(dk, k.data(), 64 * KV * D);
  be.write(dv, v.data(), 64 * KV * D);
  be.write(dq, q.data(), H * D);
  std::vector<float> ref(H * D), got(H * D);
  for (int64_t pos = 0; pos < 64; ++pos) {
    be.attention(dq, dk, dv, out, 1, pos, H, KV, D);
    be.read(got.data(), out, H * D);
    orc_attention(q.data(), k.data(), v.data(), ref.data(), 1, pos, H, KV, D);
    CHECK(maxdiff(ref.data(), got.data(), ref.size()) <= 1e-5f);
  }
  for (float* p : {dk, dv, dq, out}) be.free(p);
}

// RoPE through the backend is bit-identical to the scalar reference (NeoX with factors, and interleaved).
static void rope_case(CudaBackend& be) {
  std::mt19937 g(4);
  const int64_t n = 5, H = 4, D = 64, pos0 = 1000;
  std::vector<float> ff(D / 2);
  for (int64_t i = 0; i < D / 2; ++i) ff[i] = 1.0f + 0.25f * static_cast<float>(i);
  for (int neox = 0; neox < 2; ++neox) {
    auto x = rnd(n * H * D, g);
    auto ref = x;
    orc_rope(ref.data(), n, H, D, pos0, 5e5f, neox, neox ? ff.data() : nullptr);
    float* dx = be.alloc(n * H * D);
    be.write(dx, x.data(), n * H * D);
    be.rope(dx, n, H, D, pos0, nibble::RopeParams{5e5f, neox != 0, neox ? ff.data() : nullptr});
    std::vector<float> got(n * H * D);
    be.read(got.data(), dx, n * H * D);
    CHECK(std::memcmp(got.data(), ref.data(), got.size() * sizeof(float)) == 0);
    be.free(dx);
  }
}

// add_bias takes the bias as a host weight Tensor (uploaded once, cached by address).
static void add_bias_case(CudaBackend& be) {
  std::mt19937 g(5);
  auto x = rnd(3 * 40, g), b = rnd(40, g);
  nibble::Tensor t;
  t.type = nibble::DType::F32;
  t.n_dims = 1;
  t.ne = {40, 1, 1, 1};
  t.data = b.data();
  float* dx = be.alloc(120);
  be.write(dx, x.data(), 120);
  be.add_bias(dx, t, 3);
  be.add_bias(dx, t, 3);
  std::vector<float> got(120), ref = x;
  orc_add_bias(ref.data(), b.data(), 40, 3);
  orc_add_bias(ref.data(), b.data(), 40, 3);
  be.read(got.data(), dx, 120);
  CHECK(std::memcmp(got.data(), ref.data(), 120 * sizeof(float)) == 0);
  be.free(dx);
}

// alloc is zeroed; free(nullptr) and freeing twice are tolerated; bad sizes and weights without data throw Error.
static void contracts(CudaBackend& be) {
  float* p = be.alloc(100);
  std::vector<float> h(100, 1.f);
  be.read(h.data(), p, 100);
  bool zero = true;
  for (float x : h) zero &= x == 0.f;
  CHECK(zero);
  be.free(p);
  be.free(p);
  be.free(nullptr);
  bool threw = false;
  try {
    be.alloc(-1);
  } catch (const nibble::Error& e) {
    threw = std::string(e.what()).find("negative") != std::string::npos;
  }
  CHECK(threw);
  threw = false;
  try {
    be.matmul(nibble::Tensor{}, nullptr, nullptr, 1);
  } catch (const nibble::Error&) {
    threw = true;
  }
  CHECK(threw);
  // every weight type the reference supports runs on the GPU (src/tensor.h:21-31)
  CHECK(be.supports(nibble::DType::F32) && be.supports(nibble::DType::F16));
  CHECK(be.supports(nibble::DType::Q4_0) && be.supports(nibble::DType::Q5_0) && be.supports(nibble::DType::Q8_0));
  CHECK(be.supports(nibble::DType::Q5_1) && be.supports(nibble::DType::Q4_K) && be.supports(nibble::DType::Q5_K) &&
        be.supports(nibble::DType::Q6_K));
  threw = false;
  try {
    be.attention(nullptr, nullptr, nullptr, nullptr, 1, 0, 6, 4, 16);
  } catch (const nibble::Error&) {
    threw = true;
  }
  CHECK(threw);
  be.synchronize();
}

int main() {
  try {
    CudaBackend be(0);
    attention_case(be);
    reserve_then_decode(be);
    rope_case(be);
    add_bias_case(be);
    contracts(be);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "unexpected exception: %s\n", e.what());
    return 2;
  }
  if (g_failed) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failed);
    return 1;
  }
  std::puts("test_cuda_backend: all passed");
  return 0;
}
