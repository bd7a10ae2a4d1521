#pragma once
// nibble::cuda::BatchedDecoder -- many sequences over one model on one GPU.
//
// The reference serves one Session per Model (include/nibble/nibble.h:94-95): its Transformer owns a flat fp32 KV
// cache of n_ctx positions per layer (src/model/transformer.cpp:74-90) and decodes one token of one sequence per
// forward pass. Here the K/V of every sequence live in paged fp16 pools (one per layer, 16-token pages, page ids
// shared by all layers so one page table per sequence serves the whole stack), pages are handed out on demand and
// returned when a sequence closes, and a decode step runs one new token of each of N sequences as ONE forward pass
// of N rows: the weight matmuls read each weight once for all N tokens (GEMV up to 8 rows, GEMM above), the fused
// bias/RoPE/append kernel writes each token's K/V into its own sequence's page, and the split-K paged decode
// kernel attends every sequence over its own length.
//
// The per-layer operation order is the reference's run_chunk (src/model/transformer.cpp:147-221): rmsnorm,
// Q/K/V matmul_multi, biases, RoPE, attention, O projection, residual add, rmsnorm, gate/up matmul_multi,
// silu_mul, down projection, residual add; then the final rmsnorm and the output projection of each sequence's
// last row (forward, :128-143). The only numerical difference from nibble's Transformer is the K/V precision
// (fp16 pages instead of fp32 rows).
//
// Built inside a nibble tree (NBL_WITH_NIBBLE_TREE: it takes nibble's LlamaConfig and Weights) on top of
// CudaBackend, whose context and uploaded weights it shares. Not thread-safe (like the reference's Session).
#include <cstdint>
#include <span>
#include <vector>

#include "cuda_backend.h"
#include "model/config.h"
#include "model/weights.h"

namespace nibble::cuda {

class BatchedDecoder {
 public:
  static constexpr int64_t kPageSize = 16;

  // Up to max_seqs open sequences of up to max_ctx tokens each; prefill runs in chunks of at most max_batch
  // tokens. n_pages per layer (0: enough for every sequence at max_ctx). Throws Error for a head geometry the
  // paged kernels do not take (head_dim 64, n_heads / n_kv_heads <= 8) or when an allocation fails.
  BatchedDecoder(CudaBackend& be, const model::LlamaConfig& c, const model::Weights& w, int max_seqs,
                 int64_t max_ctx, int64_t n_pages = 0, int64_t max_batch = 512);
  ~BatchedDecoder();
  BatchedDecoder(const BatchedDecoder&) = delete;
  BatchedDecoder& operator=(const BatchedDecoder&) = delete;

  // A new empty sequence (its id); throws Error when max_seqs sequences are open.
  int open();
  // Returns the sequence's pages to the pool; the id may be handed out again.
  void close(int seq);
  int64_t n_past(int seq) const;
  int64_t free_pages() const { return static_cast<int64_t>(free_.size()); }

  // Appends tokens to one sequence at its current length (like Transformer::forward at pos0 = n_past) and writes
  // the last token's logits (n_vocab floats, host memory).
  void prefill(int seq, std::span<const int32_t> tokens, float* logits);
  // One new token for each listed sequence (distinct ids), run as one forward pass; logits [seqs.size()][n_vocab]
  // in host memory, row i for seqs[i].
  void decode(std::span<const int> seqs, std::span<const int32_t> tokens, float* logits);

 private:
  struct Seq {
    bool open = false;
    int64_t n_past = 0;
    std::vector<int32_t> pages;  // page id of positions [16 p, 16 p + 16)
  };
  Seq& seq_at(int seq);
  void ensure_pages(Seq& s, int64_t n_tokens);  // pages for positions up to n_tokens - 1
  float* grab(int64_t n_floats);
  void layer(int64_t l, int64_t n, const int32_t* tok_row, const int32_t* tok_pos, const int32_t* table,
             bool prefill, int64_t pos0, const int32_t* seq_lens, int32_t max_len);
  void release() noexcept;

  CudaBackend& be_;
  nbl_ctx* ctx_;
  model::LlamaConfig c_;
  const model::Weights& w_;
  int max_seqs_;
  int64_t max_ctx_, max_batch_, max_rows_, stride_, n_pages_;
  nbl_rope_params rope_{};
  std::vector<nbl_kv*> kv_;  // one pool per layer, same page ids
  std::vector<int32_t> free_;
  std::vector<Seq> seqs_;
  std::vector<float*> owned_;
  // device activations (rows = tokens of a prefill chunk or sequences of a decode step)
  float *x_, *h_, *q_, *k_, *v_, *q16_, *attn_, *gate_, *up_, *last_, *logits_;
  // device int32 metadata: [tok_row | tok_pos | seq_lens | page table rows | q_start, q_len, kv_pos0]
  int32_t* meta_;
  std::vector<int32_t> meta_h_;
};

}  // namespace nibble::cuda
