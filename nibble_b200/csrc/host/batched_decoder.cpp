// BatchedDecoder: many sequences over one model (see batched_decoder.h).
#include "batched_decoder.h"

#include <algorithm>
#include <string>

#include "nibble/error.h"

namespace nibble::cuda {

namespace {

// The device pointer of an F32 bias vector (uploaded through the backend's weight cache), or null.
const float* bias_ptr(CudaBackend& be, const std::optional<Tensor>& b) {
  if (!b) return nullptr;
  const void* dev = nullptr;
  check(nbl_weight_data(be.device_weight(*b), &dev, nullptr, nullptr, nullptr));
  return static_cast<const float*>(dev);
}

}  // namespace

BatchedDecoder::BatchedDecoder(CudaBackend& be, const model::LlamaConfig& c, const model::Weights& w, int max_seqs,
                               int64_t max_ctx, int64_t n_pages, int64_t max_batch)
    : be_(be), ctx_(be.handle()), c_(c), w_(w), max_seqs_(max_seqs), max_ctx_(max_ctx), max_batch_(max_batch) {
  if (max_seqs <= 0 || max_ctx <= 0 || max_batch <= 0) throw Error("batched decoder: sizes must be positive");
  if (c.head_dim != 64 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads != 0 || c.n_heads / c.n_kv_heads > 8)
    throw Error("batched decoder: the paged kernels take head_dim 64 and at most 8 query heads per KV head (got " +
                std::to_string(c.head_dim) + ", " + std::to_string(c.n_heads) + "/" + std::to_string(c.n_kv_heads) +
                ")");
  if (static_cast<int64_t>(w.layers.size()) != c.n_layers) throw Error("batched decoder: layer count mismatch");
  stride_ = (max_ctx + kPageSize - 1) / kPageSize;
  n_pages_ = n_pages > 0 ? n_pages : stride_ * max_seqs;
  max_rows_ = std::max<int64_t>(max_batch, max_seqs);
  rope_.freq_base = c.rope_base;
  rope_.neox = c.rope_neox ? 1 : 0;
  rope_.freq_factors = w.rope_freqs ? static_cast<const float*>(w.rope_freqs->data) : nullptr;
  const int64_t E = c.n_embd, Q = c.n_heads * c.head_dim, KVW = c.n_kv_heads * c.head_dim;
  try {
    const nbl_kv_config kc{n_pages_, static_cast<int32_t>(c.n_kv_heads), static_cast<int32_t>(c.head_dim),
                           static_cast<int32_t>(kPageSize), NBL_F16};
    for (int64_t l = 0; l < c.n_layers; ++l) {
      nbl_kv* kv = nullptr;
      check(nbl_kv_create(ctx_, &kc, &kv));
      kv_.push_back(kv);
    }
    x_ = grab(max_rows_ * E);
    h_ = grab(max_rows_ * E);
    q_ = grab(max_rows_ * Q);
    k_ = grab(max_rows_ * KVW);
    v_ = grab(max_rows_ * KVW);
    q16_ = grab((max_rows_ * Q + 1) / 2);  // fp16 queries for the prefill kernel
    attn_ = grab(max_rows_ * Q);
    gate_ = grab(max_rows_ * c.n_ff);
    up_ = grab(max_rows_ * c.n_ff);
    last_ = grab(static_cast<int64_t>(max_seqs) * E);
    logits_ = grab(static_cast<int64_t>(max_seqs) * c.n_vocab);
    meta_h_.assign(static_cast<size_t>(2 * max_rows_ + max_seqs + max_seqs * stride_ + 3), 0);
    meta_ = reinterpret_cast<int32_t*>(grab(static_cast<int64_t>(meta_h_.size())));
    check(nbl_reserve(ctx_, max_ctx, c.n_heads, max_rows_, std::max(c.n_ff, E)));
  } catch (...) {
    release();
    throw;
  }
  free_.resize(static_cast<size_t>(n_pages_));
  for (int64_t i = 0; i < n_pages_; ++i) free_[static_cast<size_t>(i)] = static_cast<int32_t>(n_pages_ - 1 - i);
  seqs_.resize(static_cast<size_t>(max_seqs));
}

BatchedDecoder::~BatchedDecoder() { release(); }

float* BatchedDecoder::grab(int64_t n_floats) {
  float* p = nullptr;
  check(nbl_alloc(ctx_, n_floats, &p));
  owned_.push_back(p);
  return p;
}

void BatchedDecoder::release() noexcept {
  for (nbl_kv* kv : kv_) nbl_kv_destroy(kv);
  kv_.clear();
  for (float* p : owned_) nbl_free(ctx_, p);
  owned_.clear();
}

BatchedDecoder::Seq& BatchedDecoder::seq_at(int seq) {
  if (seq < 0 || seq >= max_seqs_ || !seqs_[static_cast<size_t>(seq)].open)
    throw Error("batched decoder: sequence " + std::to_string(seq) + " is not open");
  return seqs_[static_cast<size_t>(seq)];
}

int BatchedDecoder::open() {
  for (int i = 0; i < max_seqs_; ++i) {
    Seq& s = seqs_[static_cast<size_t>(i)];
    if (!s.open) {
      s = Seq{};
      s.open = true;
      return i;
    }
  }
  throw Error("batched decoder: all " + std::to_string(max_seqs_) + " sequences are open");
}

void BatchedDecoder::close(int seq) {
  Seq& s = seq_at(seq);
  for (auto it = s.pages.rbegin(); it != s.pages.rend(); ++it) free_.push_back(*it);
  s = Seq{};
}

int64_t BatchedDecoder::n_past(int seq) const {
  if (seq < 0 || seq >= max_seqs_ || !seqs_[static_cast<size_t>(seq)].open)
    throw Error("batched decoder: sequence " + std::to_string(seq) + " is not open");
  return seqs_[static_cast<size_t>(seq)].n_past;
}

void BatchedDecoder::ensure_pages(Seq& s, int64_t n_tokens) {
  if (n_tokens > max_ctx_)
    throw Error("context overflow: " + std::to_string(n_tokens) + " tokens exceeds max_ctx " + std::to_string(max_ctx_));
  const size_t need = static_cast<size_t>((n_tokens + kPageSize - 1) / kPageSize);
  if (need > s.pages.size() && need - s.pages.size() > free_.size())
    throw Error("batched decoder: KV pool exhausted (" + std::to_string(n_pages_) + " pages of " +
                std::to_string(kPageSize) + " tokens)");
  while (s.pages.size() < need) {
    s.pages.push_back(free_.back());
    free_.pop_back();
  }
}

// One transformer block for n rows (run_chunk's per-layer body, src/model/transformer.cpp:165-219). Prefill: the
// rows are consecutive tokens of one sequence at positions pos0.., attending causally through page-table row 0.
// Decode: row r is one token of its own sequence, attending seq_lens[r] keys through page-table row r.
void BatchedDecoder::layer(int64_t l, int64_t n, const int32_t* tok_row, const int32_t* tok_pos, const int32_t* table,
                           bool prefill, int64_t pos0, const int32_t* seq_lens, int32_t max_len) {
  const model::LayerWeights& L = w_.layers[static_cast<size_t>(l)];
  const int64_t E = c_.n_embd;
  const int32_t H = static_cast<int32_t>(c_.n_heads);
  check(nbl_rmsnorm(ctx_, x_, be_.device_weight(L.attn_norm), h_, n, c_.rms_eps));
  const nbl_weight* qkv_w[3] = {be_.device_weight(L.wq), be_.device_weight(L.wk), be_.device_weight(L.wv)};
  float* const qkv_y[3] = {q_, k_, v_};
  check(nbl_matmul_multi(ctx_, qkv_w, 3, h_, qkv_y, n));
  const float* bq = bias_ptr(be_, L.bq);
  const float* bk = bias_ptr(be_, L.bk);
  const float* bv = bias_ptr(be_, L.bv);
  nbl_kv* kv = kv_[static_cast<size_t>(l)];
  const int32_t stride = static_cast<int32_t>(stride_);
  if (prefill) {
    // biased, roped fp16 queries for the tensor-core prefill; K/V straight into the sequence's pages
    check(nbl_rope_kv_append(ctx_, kv, q_, k_, v_, NBL_F32, bq, bk, bv, q16_, NBL_F16, tok_row, tok_pos, table, stride,
                             n, H, &rope_));
    const int32_t* one = meta_ + 2 * max_rows_ + max_seqs_ + max_seqs_ * stride_;  // q_start, q_len, kv_pos0
    check(nbl_attn_prefill(ctx_, kv, q16_, NBL_F16, n, one, one + 1, one + 2, table, stride, 1, H,
                           static_cast<int32_t>(n), attn_, NBL_F32));
    (void)pos0;
  } else {
    check(nbl_rope_kv_append(ctx_, kv, q_, k_, v_, NBL_F32, bq, bk, bv, q_, NBL_F32, tok_row, tok_pos, table, stride,
                             n, H, &rope_));
    check(nbl_attn_decode(ctx_, kv, q_, table, stride, seq_lens, max_len, static_cast<int32_t>(n), H, attn_, nullptr,
                          0));
  }
  check(nbl_matmul(ctx_, be_.device_weight(L.wo), attn_, h_, n));
  check(nbl_add(ctx_, x_, h_, n * E));
  check(nbl_rmsnorm(ctx_, x_, be_.device_weight(L.ffn_norm), h_, n, c_.rms_eps));
  const nbl_weight* ffn_w[2] = {be_.device_weight(L.w_gate), be_.device_weight(L.w_up)};
  float* const ffn_y[2] = {gate_, up_};
  check(nbl_matmul_multi(ctx_, ffn_w, 2, h_, ffn_y, n));
  check(nbl_silu_mul(ctx_, gate_, up_, n * c_.n_ff));
  check(nbl_matmul(ctx_, be_.device_weight(L.w_down), gate_, h_, n));
  check(nbl_add(ctx_, x_, h_, n * E));
}

void BatchedDecoder::prefill(int seq, std::span<const int32_t> tokens, float* logits) {
  Seq& s = seq_at(seq);
  const int64_t total = static_cast<int64_t>(tokens.size());
  if (total == 0) throw Error("forward: no tokens");
  ensure_pages(s, s.n_past + total);
  // metadata layout: tok_row [max_rows] | tok_pos [max_rows] | seq_lens [max_seqs] | table [max_seqs][stride] |
  // q_start, q_len, kv_pos0
  int32_t* tok_row = meta_h_.data();
  int32_t* tok_pos = tok_row + max_rows_;
  int32_t* table = tok_pos + max_rows_ + max_seqs_;
  int32_t* one = table + max_seqs_ * stride_;
  std::copy(s.pages.begin(), s.pages.end(), table);
  for (int64_t off = 0; off < total; off += max_batch_) {
    const int64_t n = std::min(max_batch_, total - off), pos0 = s.n_past;
    for (int64_t i = 0; i < n; ++i) {
      tok_row[i] = 0;
      tok_pos[i] = static_cast<int32_t>(pos0 + i);
    }
    one[0] = 0;
    one[1] = static_cast<int32_t>(n);
    one[2] = static_cast<int32_t>(pos0);
    check(nbl_write(ctx_, reinterpret_cast<float*>(meta_), reinterpret_cast<const float*>(meta_h_.data()),
                    static_cast<int64_t>(meta_h_.size())));
    check(nbl_embed(ctx_, be_.device_weight(w_.token_embd), tokens.data() + off, n, x_));
    const int32_t* d_row = meta_;
    const int32_t* d_pos = meta_ + max_rows_;
    const int32_t* d_table = meta_ + 2 * max_rows_ + max_seqs_;
    for (int64_t l = 0; l < c_.n_layers; ++l) layer(l, n, d_row, d_pos, d_table, true, pos0, nullptr, 0);
    s.n_past += n;
    if (off + n == total) {
      check(nbl_rmsnorm(ctx_, x_ + (n - 1) * c_.n_embd, be_.device_weight(w_.output_norm), last_, 1, c_.rms_eps));
      check(nbl_matmul(ctx_, be_.device_weight(w_.output), last_, logits_, 1));
      check(nbl_read(ctx_, logits, logits_, c_.n_vocab));
    }
  }
}

void BatchedDecoder::decode(std::span<const int> seqs, std::span<const int32_t> tokens, float* logits) {
  const int64_t n = static_cast<int64_t>(seqs.size());
  if (n == 0) throw Error("decode: no sequences");
  if (static_cast<int64_t>(tokens.size()) != n) throw Error("decode: one token per sequence");
  std::vector<char> seen(static_cast<size_t>(max_seqs_), 0);
  for (int id : seqs) {
    Seq& s = seq_at(id);
    if (seen[static_cast<size_t>(id)]++) throw Error("decode: sequence " + std::to_string(id) + " listed twice");
    ensure_pages(s, s.n_past + 1);
  }
  int32_t* tok_row = meta_h_.data();
  int32_t* tok_pos = tok_row + max_rows_;
  int32_t* lens = tok_pos + max_rows_;
  int32_t* table = lens + max_seqs_;
  int32_t max_len = 0;
  for (int64_t r = 0; r < n; ++r) {
    const Seq& s = seqs_[static_cast<size_t>(seqs[static_cast<size_t>(r)])];
    tok_row[r] = static_cast<int32_t>(r);
    tok_pos[r] = static_cast<int32_t>(s.n_past);
    lens[r] = static_cast<int32_t>(s.n_past + 1);
    max_len = std::max(max_len, lens[r]);
    std::copy(s.pages.begin(), s.pages.end(), table + r * stride_);
  }
  check(nbl_write(ctx_, reinterpret_cast<float*>(meta_), reinterpret_cast<const float*>(meta_h_.data()),
                  static_cast<int64_t>(meta_h_.size())));
  check(nbl_embed(ctx_, be_.device_weight(w_.token_embd), tokens.data(), n, x_));
  const int32_t* d_row = meta_;
  const int32_t* d_pos = meta_ + max_rows_;
  const int32_t* d_lens = meta_ + 2 * max_rows_;
  const int32_t* d_table = d_lens + max_seqs_;
  for (int64_t l = 0; l < c_.n_layers; ++l) layer(l, n, d_row, d_pos, d_table, false, 0, d_lens, max_len);
  check(nbl_rmsnorm(ctx_, x_, be_.device_weight(w_.output_norm), last_, n, c_.rms_eps));
  check(nbl_matmul(ctx_, be_.device_weight(w_.output), last_, logits_, n));
  check(nbl_read(ctx_, logits, logits_, n * c_.n_vocab));
  for (int id : seqs) ++seqs_[static_cast<size_t>(id)].n_past;
}

}  // namespace nibble::cuda
