/* nibble_cuda.h -- C ABI of the B200 (sm_100a) attention backend for nibble.
 *
 * This is the boundary a nibble build binds to replace its CPU attention path. Every entry point is
 * extern "C" with plain pointers and sizes; no C++ or torch type crosses it. Device pointers are CUDA
 * device addresses on the context's device. All kernels run on the context's stream, in call order.
 *
 * Each declaration names the reference interface it replaces (paths inside the nibble source tree):
 *   src/backend/backend.h          the abstract Backend the Transformer calls (alloc/free/read/reserve/
 *                                  add_bias/rope/attention)
 *   src/backend/cpu/cpu_backend.*  its CPU implementation
 *   src/model/transformer.cpp      the caller: K/V projected into cache rows, bias, rope, attention
 *
 * Error convention. Every function returns an nbl_status (0 = NBL_OK). On failure, nbl_last_error() gives a
 * self-contained message for the calling thread, the way nibble::Error::what() does (include/nibble/error.h);
 * the C++ host layer (nibble_b200/csrc/host/cuda_backend.h) rethrows non-zero statuses as nibble::Error.
 * Bad sizes and null pointers are rejected on the host before any launch. Device-resident indices (page
 * tables, sequence lengths) are range-checked inside the kernels: an out-of-range entry is skipped and sets
 * a sticky flag that nbl_ctx_check() reports as NBL_E_DEVICE.
 */
#ifndef NIBBLE_CUDA_H
#define NIBBLE_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NBL_ABI_VERSION 1

/* The library is built with hidden visibility; only the entry points below are exported. */
#if defined(__GNUC__)
#define NBL_API __attribute__((visibility("default")))
#else
#define NBL_API
#endif

typedef enum {
  NBL_OK = 0,
  NBL_E_INVALID = 1,     /* bad argument (size, null pointer, unsupported shape) */
  NBL_E_CUDA = 2,        /* a CUDA runtime call failed */
  NBL_E_NOMEM = 3,       /* device allocation failed */
  NBL_E_UNSUPPORTED = 4, /* valid request this build does not run (e.g. head_dim != 64 on a paged kernel) */
  NBL_E_DEVICE = 5       /* a kernel found an out-of-range device-side index (see nbl_ctx_check) */
} nbl_status;

/* Element types. The quantized weight types are GGUF's block formats byte for byte (src/quant.h:30-99):
 * Q4_0 (18-byte blocks of 32), Q5_0 (22-byte blocks), Q8_0 (34-byte blocks), Q5_1 (24-byte blocks of 32), and the
 * k-quants Q4_K (144-byte blocks of 256), Q5_K (176-byte blocks) and Q6_K (210-byte blocks). */
typedef enum {
  NBL_F32 = 0,
  NBL_F16 = 1,
  NBL_BF16 = 2,
  NBL_Q4_0 = 3,
  NBL_Q5_0 = 4,
  NBL_Q8_0 = 5,
  NBL_Q5_1 = 6,
  NBL_Q4_K = 7,
  NBL_Q5_K = 8,
  NBL_Q6_K = 9
} nbl_dtype;

typedef struct nbl_ctx nbl_ctx; /* device, stream, scratch, RoPE tables, allocation registry */
typedef struct nbl_kv nbl_kv;   /* one paged K/V pool */
typedef struct nbl_weight nbl_weight; /* one weight tensor uploaded to the device */

/* Rotary-embedding options; same fields and meaning as nibble::RopeParams (src/backend/backend.h:16-20).
 * freq_factors is HOST memory (head_dim/2 floats) or NULL. */
typedef struct {
  float freq_base;
  int32_t neox; /* nonzero: rotate (i, i + head_dim/2); zero: rotate (2i, 2i + 1) */
  const float* freq_factors;
} nbl_rope_params;

/* Paged K/V pool. A page holds page_size consecutive token positions of one sequence for every KV head:
 *   pool[page][2 (K then V)][n_kv_heads][page_size][head_dim]  (dtype F16 or BF16)
 * so the K rows of one (page, KV head) are one contiguous page_size*head_dim block. Sequences own pages
 * through page tables (int32 page ids, row-major [rows, pt_stride]); pages need not be contiguous or
 * ordered. Replaces the flat fp32 per-layer cache of src/model/transformer.cpp:74-90. */
typedef struct {
  int64_t n_pages;
  int32_t n_kv_heads;
  int32_t head_dim;  /* 64 on the TMA/tensor-core kernels */
  int32_t page_size; /* 16 */
  int32_t dtype;     /* NBL_F16 or NBL_BF16 */
} nbl_kv_config;

/* ABI version the library was built with (NBL_ABI_VERSION). */
NBL_API int nbl_abi_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to cap) and returns its full
 * length. Mirrors nibble::Error::what(). */
NBL_API size_t nbl_last_error(char* buf, size_t cap);

/* ---- context (the Backend object itself; CpuBackend ctor/dtor src/backend/cpu/cpu_backend.cpp:20,70) ---- */
NBL_API int nbl_ctx_create(int device, nbl_ctx** out);
/* Frees every allocation, pool and table the context still owns (CpuBackend::~CpuBackend frees unfreed
 * blocks, cpu_backend.cpp:70-72). */
NBL_API int nbl_ctx_destroy(nbl_ctx* ctx);
/* Runs later launches on `stream` (a cudaStream_t; NULL is CUDA's default stream). A new context runs on a
 * stream of its own until this is called. */
NBL_API int nbl_ctx_set_stream(nbl_ctx* ctx, void* stream);
/* Returns the context to its own stream. */
NBL_API int nbl_ctx_use_own_stream(nbl_ctx* ctx);
NBL_API void* nbl_ctx_stream(nbl_ctx* ctx);
/* Waits for the context's queued work (with the paged route on, recorded query-row ops are launched first). */
NBL_API int nbl_ctx_sync(nbl_ctx* ctx);
/* Synchronises (as nbl_ctx_sync), then returns NBL_E_DEVICE (and clears the flag) if any kernel since the last check
 * skipped an out-of-range page id, position or length, or gave up a bounded wait. */
NBL_API int nbl_ctx_check(nbl_ctx* ctx);

/* Serves the drop-in Backend ops below from fp16 pages (on != 0) or keeps the reference's flat fp32 K/V blocks
 * (on == 0, the default of a new context; nibble_b200/csrc/host/cuda_backend.h's CudaBackend turns it on).
 * With it on, the first nbl_attention on a pair of K/V blocks from nbl_alloc with head_dim 64 binds them: from
 * then on their rows are fp16 pages inside the K block's own memory (no allocation), a matmul output aimed at
 * their rows is staged, nbl_add_bias / nbl_rope on those rows and on the query rows are recorded, and
 * nbl_attention runs them as one fused bias + RoPE + fp16 append launch followed by the split-K decode kernel
 * (n <= 8 rows, fp32 accuracy) or the tcgen05 prefill kernel (n > 8 rows, fp16 operands). Every other access to
 * such a block (nbl_read, nbl_copy, ...) first turns it back into flat fp32 rows (values rounded to fp16), so each
 * op keeps its Backend meaning; a recorded query op is applied before anything else reads the rows. Call it
 * before nbl_reserve and before allocating the K/V blocks (the reserve sizes the staging; K/V-shaped blocks then
 * get room for whole 16-position pages). Turning it off returns every bound block to flat fp32 rows. Replaces
 * the flat fp32 cache of src/model/transformer.cpp:74-90 behind the unchanged Backend calls (:171-202). */
NBL_API int nbl_ctx_set_paged_kv(nbl_ctx* ctx, int32_t on);

/* ---- Backend memory ops ---- */
/* Backend::reserve (backend.h:42-45; CpuBackend::reserve cpu_backend.cpp:24-67): sizes the split-K scratch and
 * the RoPE tables for up to n_ctx positions and n_heads heads, the token-id staging for max_rows tokens, and
 * (max_rows > 8) the SGEMM handle and its workspace, so later calls within those limits allocate nothing.
 * max_width is accepted for interface parity. */
NBL_API int nbl_reserve(nbl_ctx* ctx, int64_t n_ctx, int64_t n_heads, int64_t max_rows, int64_t max_width);
/* Backend::alloc (backend.h:46-47): zeroed device block of n_floats floats (256-byte aligned). n_floats < 0 or
 * an allocation failure is an error. */
NBL_API int nbl_alloc(nbl_ctx* ctx, int64_t n_floats, float** out);
/* Backend::free (backend.h:48-51): NULL is a no-op; a pointer this context did not allocate is ignored. */
NBL_API int nbl_free(nbl_ctx* ctx, float* p);
/* Backend::read (backend.h:52-53): copies n floats device -> host; returns after the copy completes. */
NBL_API int nbl_read(nbl_ctx* ctx, float* host_dst, const float* src, int64_t n);
/* Host -> device copy of n floats (no Backend counterpart: the CPU backend's memory is host memory, so the
 * model writes activations directly; a device backend needs this for inputs). */
NBL_API int nbl_write(nbl_ctx* ctx, float* dst, const float* host_src, int64_t n);

/* ---- Backend ops on fp32 device activations (the drop-in path) ---- */
/* Backend::add_bias (backend.h:63; ref_ops.cpp:156-161): x[t, i] += bias[i] for t < n, i < width. bias is a
 * device pointer. */
NBL_API int nbl_add_bias(nbl_ctx* ctx, float* x, const float* bias, int64_t width, int64_t n);
/* Backend::rope (backend.h:64; ref_ops.cpp:166-185): in place on x[n, n_heads, head_dim] at positions pos0..
 * Angles and cos/sin are evaluated in double on the host, as the reference does, and cached per
 * (freq_base, head_dim, freq_factors); the rotation is two uncontracted float products. Bit-identical to
 * nibble's cpu::rope. */
NBL_API int nbl_rope(nbl_ctx* ctx, float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0,
             const nbl_rope_params* rope);
/* Backend::attention (backend.h:66-69; CpuBackend::attention cpu_backend.cpp:272-290): q,out [n, n_heads,
 * head_dim]; k,v [>= pos0+n, n_kv_heads, head_dim], all fp32 device memory; row t has position pos0+t and
 * attends to 0..pos0+t. n_heads % n_kv_heads == 0, head_dim <= 256 (any parity, as in the reference). */
NBL_API int nbl_attention(nbl_ctx* ctx, const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                  int64_t n_heads, int64_t n_kv_heads, int64_t head_dim);

/* ---- weights and the model's other ops (backend.h:54-70), fp32 device activations ---- */
/* Uploads a host weight tensor of ne1 rows x ne0 elements, dtype NBL_F32, NBL_F16 or a quantized type (the GGUF
 * block bytes row after row, ne0 a multiple of the block: 32, or 256 for the k-quants; Q4_0 / Q5_0 / Q8_0 are
 * repacked into an internal aligned layout, Q5_1 and the k-quants stay as they are), to device memory owned by the context: the device form of a weight Tensor view (src/tensor.h:57-70;
 * nibble's are views of the mmap'd GGUF). An F16 matrix gets an fp32 copy on its first matmul with more than 8 rows (the SGEMM path; decode-only use
 * never holds it). Freed by nbl_weight_destroy or with the context. Returns after the upload has completed (the
 * host buffer may be released). */
NBL_API int nbl_weight_create(nbl_ctx* ctx, const void* host, int32_t dtype, int64_t ne0, int64_t ne1,
                              nbl_weight** out);
NBL_API int nbl_weight_destroy(nbl_weight* w);
/* The uploaded tensor: device address of its elements (F32/F16: in its own dtype; Q4_0/Q5_0/Q8_0: the internal
 * layout; Q5_1 and the k-quants: the GGUF blocks as uploaded), dtype and shape. Any out pointer may be NULL. An F32 vector's address is what nbl_add_bias takes. */
NBL_API int nbl_weight_data(const nbl_weight* w, const void** dev, int32_t* dtype, int64_t* ne0, int64_t* ne1);
/* Backend::embed (backend.h:54-55; cpu::embed ref_ops.cpp:80-98): out[t, :] = row ids[t] of table, widened to
 * fp32 (bit-identical). ids is HOST memory (a std::span in the reference); an id outside [0, ne1) is
 * NBL_E_INVALID with the reference's message and nothing is written. */
NBL_API int nbl_embed(nbl_ctx* ctx, const nbl_weight* table, const int32_t* ids, int64_t n, float* out);
/* Backend::matmul (backend.h:56; cpu::matmul_rows ref_ops.cpp:109-136): y[n, ne1] = x[n, ne0] . W^T.
 * F32/F16 weights: fp32 arithmetic (F16 widened exactly); n <= 8 streams the weight once (GEMV kernel), larger n
 * runs SGEMM (cuBLAS, no TF32); results differ from the CPU's only by fp32 summation order. Quantized weights: x is
 * quantized to Q8_0 blocks and each output is the reference's sum of per-block terms (src/quant.cpp:310-366),
 * bit-identical to nibble's CPU result, for any n (in chunks of 8 rows). */
NBL_API int nbl_matmul(nbl_ctx* ctx, const nbl_weight* w, const float* x, float* y, int64_t n);
/* Backend::matmul_multi (backend.h:57-60; CpuBackend::matmul_multi cpu_backend.cpp:146-233): ys[i] = x . ws[i]^T
 * for `count` weights sharing one input x [n, ne0] (all ws[i] have the same ne0); results equal separate
 * nbl_matmul calls. For n <= 8 and count <= 4 this is one GEMV launch over all the weights' rows (the model's
 * Q/K/V and gate/up projections). ws and ys are HOST arrays of count entries. */
NBL_API int nbl_matmul_multi(nbl_ctx* ctx, const nbl_weight* const* ws, int32_t count, const float* x,
                             float* const* ys, int64_t n);
/* Backend::rmsnorm (backend.h:61; cpu::rmsnorm ref_ops.cpp:138-148): y[t] = x[t] / sqrt(mean(x[t]^2) + eps) *
 * weight, evaluated in double like the reference and rounded once to float. weight is an F32 vector (ne1 = 1)
 * of width d = ne0; x, y are [n, d]. */
NBL_API int nbl_rmsnorm(nbl_ctx* ctx, const float* x, const nbl_weight* weight, float* y, int64_t n, float eps);
/* Backend::add (backend.h:62; ref_ops.cpp:151-153): x[i] += y[i] for i < count (bit-identical). */
NBL_API int nbl_add(nbl_ctx* ctx, float* x, const float* y, int64_t count);
/* Backend::copy (backend.h:65; CpuBackend::copy cpu_backend.cpp:260-264): dst[i] = src[i]; the ranges must not
 * overlap (the reference's memmove allows it; its only caller, the Transformer, never overlaps). */
NBL_API int nbl_copy(nbl_ctx* ctx, float* dst, const float* src, int64_t count);
/* Backend::silu_mul (backend.h:70; ref_ops.cpp:217-222): gate[i] = g / (1 + e^-g) * up[i], g = gate[i], in
 * float (within a few ulp of the reference: CUDA's expf against the C library's). */
NBL_API int nbl_silu_mul(nbl_ctx* ctx, float* gate, const float* up, int64_t count);

/* ---- paged K/V path (B200-native layout; the reference keeps fp32 flat caches) ---- */
/* Allocates and zeroes a pool (see nbl_kv_config) and the TMA descriptors over it. */
NBL_API int nbl_kv_create(nbl_ctx* ctx, const nbl_kv_config* cfg, nbl_kv** out);
NBL_API int nbl_kv_destroy(nbl_kv* kv);
/* Base device address and size of the pool (for bulk fills and read-back in tests). */
NBL_API int nbl_kv_pool(const nbl_kv* kv, void** base, int64_t* bytes);

/* Fused bias -> RoPE -> narrowing -> page write for new tokens: the sequence transformer.cpp:171-198 runs as
 * matmul_multi into cache rows, add_bias(q/k/v), rope(q), rope(k). For token r (r < n_tok):
 *   q_out[r] = rope(q_in[r] + bq) at position tok_pos[r]            (n_heads heads, dtype q_out_dtype)
 *   page(tok_row[r], tok_pos[r]) <- narrow(rope(k_in[r] + bk)), narrow(v_in[r] + bv)   (n_kv_heads heads)
 * where page(row, pos) is slot pos % page_size of page page_table[row * pt_stride + pos / page_size].
 * q_in/k_in/v_in are [n_tok, heads, head_dim] of in_dtype (F32, F16 or BF16); biases are fp32 device vectors or
 * NULL; q_out may alias q_in when the dtypes match. All index arrays are device memory. */
NBL_API int nbl_rope_kv_append(nbl_ctx* ctx, nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                       int32_t in_dtype, const float* bq, const float* bk, const float* bv, void* q_out,
                       int32_t q_out_dtype, const int32_t* tok_row, const int32_t* tok_pos, const int32_t* page_table,
                       int32_t pt_stride, int64_t n_tok, int32_t n_heads, const nbl_rope_params* rope);

/* Single-token decode (Backend::attention with n = 1, backend.h:66-69) over the paged pool, for n_rows
 * independent (sequence, layer) rows at once. Row r: query q[r] ([n_heads, head_dim] fp32, already roped),
 * keys/values 0..seq_lens[r]-1 through page-table row r. Writes out[r] ([n_heads, head_dim] fp32) and, if lse
 * is non-NULL, lse[r, h] = ln(sum_j exp(score_j)) (natural log; the partial form the LSE merge consumes).
 * seq_lens[r] == 0 gives out = 0 and lse = -inf. max_seq_len bounds every seq_lens[r] (it sizes the splits;
 * the kernel also checks each length against pt_stride * page_size). n_splits: KV splits per row (0 = chosen
 * from the sizes); more than one uses context scratch sized by nbl_reserve (grown on demand otherwise).
 * head_dim 64, n_heads / n_kv_heads <= 8. */
NBL_API int nbl_attn_decode(nbl_ctx* ctx, const nbl_kv* kv, const float* q, const int32_t* page_table, int32_t pt_stride,
                    const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows, int32_t n_heads, float* out,
                    float* lse, int32_t n_splits);

/* One decode step from host memory with the transfers overlapped -- nbl_write of the new tokens,
 * nbl_rope_kv_append, nbl_attn_decode and nbl_read of the outputs in one call. Row r gets one new token: its
 * q/k/v (q_in_h [n_rows, n_heads, head_dim], k_in_h / v_in_h [n_rows, n_kv_heads, head_dim], fp32 host memory;
 * pinned memory lets the copies overlap) are biased (bq/bk/bv: fp32 device vectors or NULL), roped and appended
 * at position seq_lens[r] - 1 (seq_lens counts the new token, so every seq_lens[r] >= 1), then row r attends keys
 * 0..seq_lens[r]-1 and out_h[r] ([n_heads, head_dim] fp32 host) receives the result. page_table/seq_lens are
 * device memory as for nbl_attn_decode. The rows are cut into n_chunks ranges (0 = chosen by the library): each
 * range's upload runs on a copy stream while earlier ranges' append + decode run (on the context's stream and,
 * when no split partials are needed, a second internal one so consecutive ranges overlap),
 * and each range's results are copied back while the next range computes. Results equal the separate calls'
 * (per-range split counts may differ, within the decode tolerance). Device staging (5 row-sized fp32 buffers)
 * is context-owned and grown on demand. Returns once out_h is complete. No direct counterpart in the reference
 * (its decode reads host-resident activations in place); this is the host-buffer form of the decode step. */
NBL_API int nbl_decode_step_host(nbl_ctx* ctx, nbl_kv* kv, const float* q_in_h, const float* k_in_h,
                                 const float* v_in_h, const float* bq, const float* bk, const float* bv,
                                 const int32_t* page_table, int32_t pt_stride, const int32_t* seq_lens,
                                 int32_t max_seq_len, int32_t n_rows, int32_t n_heads, const nbl_rope_params* rope,
                                 float* out_h, int32_t n_chunks);

/* Same arguments and results as nbl_attn_decode, but the call allocates no device memory: the split partials
 * live in a fixed 8 MiB array inside the library (held on every GPU the library has created a context on, until
 * the process exits) instead of context scratch. For callers that may not allocate once running -- e.g. an
 * engine that owns all device memory through its own pool, or a decode loop that cannot take cudaMalloc's
 * device-wide sync. nbl_ctx_create sets the array up (loads it, resolves its device address) and loads the
 * decode kernels, so every call of this entry point, the first included, allocates nothing.
 * An explicit n_splits whose partials (n_splits * n_rows * n_heads * 65 floats) exceed the array is rejected
 * with NBL_E_INVALID; with n_splits = 0 the split count is reduced until they fit. All calls on a device share
 * the array (each call writes every partial it reads, so nothing needs clearing); calls whose kernels overlap
 * on the GPU race on it and must be serialised. No counterpart in the reference (nibble's CPU backend sizes its
 * scratch once in reserve()). */
NBL_API int nbl_attn_decode_static(nbl_ctx* ctx, const nbl_kv* kv, const float* q, const int32_t* page_table,
                                   int32_t pt_stride, const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows,
                                   int32_t n_heads, float* out, float* lse, int32_t n_splits);

/* Causal prefill (Backend::attention with n >= 1) over the paged pool for n_items independent items. q and out
 * hold n_q_rows rows of [n_heads, head_dim]. Item i: query rows q[q_start[i] .. q_start[i] + q_len[i])
 * (q_dtype = the pool dtype, already roped) at positions kv_pos0[i] + t, attending keys 0..kv_pos0[i]+t of
 * page-table row i (those keys must already be in the pool). max_q_len bounds every q_len[i]. Writes the
 * items' out rows in out_dtype (F32 or the pool dtype). Tensor-core kernel (tcgen05): bf16/fp16 operands, fp32
 * accumulation in TMEM. */
NBL_API int nbl_attn_prefill(nbl_ctx* ctx, const nbl_kv* kv, const void* q, int32_t q_dtype, int64_t n_q_rows,
                     const int32_t* q_start, const int32_t* q_len, const int32_t* kv_pos0, const int32_t* page_table,
                     int32_t pt_stride, int32_t n_items, int32_t n_heads, int32_t max_q_len, void* out,
                     int32_t out_dtype);

/* Log-sum-exp merge of n_parts partial results of the same rows (e.g. per-GPU KV chunks after an
 * all-gather): part_o [n_parts, rows, head_dim] normalised outputs, part_lse [n_parts, rows] natural-log
 * sums. Writes out [rows, head_dim] and, if non-NULL, lse [rows]. Parts with lse = -inf are ignored. */
NBL_API int nbl_lse_merge(nbl_ctx* ctx, const float* part_o, const float* part_lse, int32_t n_parts, int64_t rows,
                  int32_t head_dim, float* out, float* lse);

/* nbl_lse_merge over the layout one all-gather of per-rank partials produces: part p occupies
 * packed[p * rows * (head_dim + 1) ...] as [rows, head_dim] outputs followed by [rows] lse, so a rank can
 * decode straight into its send buffer and merge the gathered buffer in place. No reference counterpart (the
 * reference never splits a softmax across devices). */
NBL_API int nbl_lse_merge_packed(nbl_ctx* ctx, const float* packed, int32_t n_parts, int64_t rows, int32_t head_dim,
                                 float* out, float* lse);

/* The long-context exchange without a collective library: every rank's (O, lse) partials cross NVLink as plain stores
 * into the other ranks' memory, and each rank merges once all have arrived (nbl_lse_merge_packed's arithmetic).
 * send: this rank's packed partials [rows * head_dim outputs | rows lse] (device). recv_bufs[p] / flag_bufs[p]: rank
 * p's receive buffer ([2][world][rows * (head_dim + 1)] floats) and flag words ([world] uint32, zero before the first
 * call), as device addresses valid in this process (peer memory mapped by the caller, e.g. a symmetric-memory
 * allocation); sync: two uint32 of this rank's device memory, zero before the first call. Two launches on the
 * context's stream: the push (stores, then per-rank release flags at system scope) and the merge (waits on its own
 * flags with acquire loads, bounded by the library's 2 s wait limit: a rank that never arrives ends the merge with
 * NBL_E_DEVICE at nbl_ctx_check and no output). Every rank must make the same sequence of calls. world <= 8. No
 * reference counterpart (the reference never splits a softmax across devices); replaces the all-gather +
 * nbl_lse_merge_packed pair for GPUs that reach each other's memory (NVLink / NVSwitch). */
NBL_API int nbl_lse_exchange_peers(nbl_ctx* ctx, const float* send, int64_t rows, int32_t head_dim, int32_t world,
                                   int32_t rank, void* const* recv_bufs, void* const* flag_bufs, uint32_t* sync,
                                   float* out, float* lse);

/* nbl_attn_decode with the exchange of nbl_lse_exchange_peers fused into it: the decode kernel stores each
 * (row, head)'s final (O, lse) -- this rank's partial over its KV chunk -- straight into slot `rank` of every rank's
 * receive buffer (over NVLink for the other ranks), and its last finalising CTA raises this rank's flag word on every
 * rank (system-scope release); then the merge waits for all ranks' flags (bounded, as in nbl_lse_exchange_peers) and
 * writes out [n_rows, n_heads, 64] and, if non-NULL, lse [n_rows, n_heads]. No send buffer and no separate push
 * launch. recv_bufs / flag_bufs / sync as for nbl_lse_exchange_peers with rows = n_rows * n_heads and head_dim 64;
 * the pool and its arguments as for nbl_attn_decode (the library chooses the split count). Every rank must make the
 * same sequence of calls; world <= 8. No reference counterpart (the reference never splits a softmax across
 * devices). */
NBL_API int nbl_attn_decode_peers(nbl_ctx* ctx, const nbl_kv* kv, const float* q, const int32_t* page_table,
                                  int32_t pt_stride, const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows,
                                  int32_t n_heads, int32_t world, int32_t rank, void* const* recv_bufs,
                                  void* const* flag_bufs, uint32_t* sync, float* out, float* lse);

/* ---- diagnostics ---- */
/* Runs the library's bounded device wait (the routine every TMA / tensor-core completion wait uses) in a one-thread
 * kernel against an mbarrier that nothing arrives on, with a limit of limit_ns (0 < limit_ns <= 1e9): the wait gives
 * up, the kernel returns, and the next nbl_ctx_check reports NBL_E_DEVICE ("a bounded wait ... gave up") and clears
 * the flag, after which the context runs normally. Shows that a lost completion ends a launch with an error instead
 * of a hang, without faulting anything. Until that check, later waits of the context give up at once (the timeout
 * bit is sticky). No reference counterpart; the reference reports failures as nibble::Error
 * (include/nibble/error.h:8-13). */
NBL_API int nbl_selftest_bounded_wait(nbl_ctx* ctx, int64_t limit_ns);

#ifdef __cplusplus
}
#endif
#endif
