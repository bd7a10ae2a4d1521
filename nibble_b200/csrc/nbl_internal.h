// Internal host-side declarations shared by the C-ABI layer (api.cu) and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/nibble_cuda.h"
#include "nbl_errors.h"

namespace nbl {

// A failure carrying the status the C ABI returns; thrown inside the library, caught at the ABI boundary.
struct Failure : std::runtime_error {
  int status;
  Failure(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(int status, const std::string& msg) { throw Failure(status, msg); }
inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(NBL_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Cached cos/sin table for one RoPE configuration: tab[pos * half + i] = (cos, sin) of
// pos * base^(-2i/head_dim) / freq_factors[i], evaluated in double on the host.
struct RopeTable {
  float base = 0.f;
  int64_t head_dim = 0;
  std::vector<float> factors;  // empty when none
  int64_t n_pos = 0;
  float2* dev = nullptr;
};

}  // namespace nbl

struct nbl_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;                        // device error word (nbl_ctx_check)
  struct Alloc {
    size_t bytes;    // allocated (rounded up, padded for whole K/V pages when the paged route is on)
    int64_t floats;  // requested
  };
  std::map<void*, Alloc> allocs;               // Backend::alloc registry
  void* route = nullptr;                       // nbl::Route when the paged K/V route is on (backend_route.cu)
  void* scratch = nullptr;                     // split-K partials
  size_t scratch_bytes = 0;
  unsigned* split_counts = nullptr;            // split-K arrival counters, one per (row, KV head); 0 between launches
  int64_t split_counts_n = 0;
  int64_t reserved_ctx = 0, reserved_heads = 0;
  std::vector<nbl::RopeTable> rope_tables;
  std::vector<nbl_kv*> kvs;
  // nbl_decode_step_host: staging for the step's inputs/outputs and the two copy streams with their events
  void* io = nullptr;
  size_t io_bytes = 0;
  cudaStream_t up_stream = nullptr, down_stream = nullptr, aux_stream = nullptr;
  std::vector<cudaEvent_t> events;
  // the model's other ops (model_ops.cu): uploaded weights, the token-id staging buffer
  std::vector<nbl_weight*> weights;
  int32_t* ids = nullptr;
  int64_t ids_cap = 0;
  void* qgemm_act = nullptr;  // activations quantized for the quantized tensor-core matmul
  size_t qgemm_act_bytes = 0;
  void* fgemm_act = nullptr;  // activations split into tf32 terms for the float tensor-core matmul
  size_t fgemm_act_bytes = 0;
  void* qgemv_act = nullptr;  // activations quantized for the quantized GEMV (up to 8 rows)
  size_t qgemv_act_bytes = 0;
  void* qblock_act = nullptr;  // activations quantized to Q8_1 / Q8_K for Q5_1 and k-quant weights
  size_t qblock_act_bytes = 0;
};

struct nbl_kv {
  nbl_ctx* ctx = nullptr;
  nbl_kv_config cfg{};
  void* pool = nullptr;
  size_t bytes = 0;
  CUtensorMap tmap;  // 2-D view [n_pages*2*n_kv_heads*page_size rows, head_dim], box page_size x head_dim, 128B swizzle
  bool has_tmap = false;
};

namespace nbl {

// Stores msg as the calling thread's nbl_last_error() message and returns status (for entry points defined
// outside api.cu).
int record_error(int status, const std::string& msg);

// cudaMalloc that fails with NBL_E_NOMEM and a message naming `what`.
void* device_alloc(size_t bytes, const char* what);
// Grows the context's split-K scratch to at least `bytes` (waits for queued work before freeing the old buffer).
void ensure_scratch(nbl_ctx* ctx, size_t bytes);
// The context's split-K arrival counters for `units` (row, KV head) pairs: zeroed when allocated, and every
// decode launch leaves the counters it used at 0 again. Grows like ensure_scratch.
unsigned* split_counts(nbl_ctx* ctx, int64_t units);
// The device cos/sin table for (base, head_dim, factors) covering positions [0, n_pos), built on first use.
const RopeTable& rope_table(nbl_ctx* ctx, const nbl_rope_params& rp, int64_t head_dim, int64_t n_pos);

// Encodes a tiled TMA descriptor (driver entry point resolved once through the runtime; no libcuda link).
// dims/strides in elements/bytes as cuTensorMapEncodeTiled takes them; 128-byte swizzle unless told otherwise, zero
// OOB fill.
void encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides_bytes, const cuuint32_t* box,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// ---- launches (defined in the kernel .cu files; all asynchronous on `st`) ----
// rope.cu
void launch_add_bias(cudaStream_t st, float* x, const float* bias, int64_t width, int64_t n);
void launch_rope_f32(cudaStream_t st, float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0,
                     bool neox, const float2* tab, int* err);
void launch_rope_kv_append(cudaStream_t st, const nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                           int in_dtype, const float* bq, const float* bk, const float* bv, void* q_out,
                           int q_out_dtype, const int32_t* tok_row, const int32_t* tok_pos,
                           const int32_t* page_table, int32_t pt_stride, int64_t n_tok, int n_heads, bool neox,
                           const float2* tab, int64_t tab_pos, int* err,
                           int32_t row_base = 0, const int32_t* lens = nullptr);
// attn_f32.cu
void launch_attention_f32(cudaStream_t st, const float* q, const float* k, const float* v, float* out, int64_t n,
                          int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, float scale,
                          int num_sms);
// decode.cu
struct DecodePlan {
  int n_splits = 1;
  int pages_per_split = 0;
  size_t scratch_bytes = 0;
};
DecodePlan plan_decode(int n_rows, int n_kv_heads, int group, int n_heads, int max_seq_len, int page_size,
                       int num_sms, int requested_splits);
void launch_decode(cudaStream_t st, const nbl_kv* kv, const float* q, const int32_t* page_table, int32_t pt_stride,
                   const int32_t* seq_lens, int n_rows, int n_heads, float* out, float* lse, const DecodePlan& plan,
                   void* scratch, int* err, unsigned* counts = nullptr);
// Loads the decode and merge kernels on the current device and sets their shared-memory attribute, so a later
// launch needs no module load (which allocates device memory).
void preload_decode();
// decode_static.cu: places the allocation-free decode's static partials array on the current device (device id
// `device`), resolves its address and preloads the decode kernels. Called by nbl_ctx_create, while allocation is
// still allowed, so nbl_attn_decode_static itself allocates nothing.
void prepare_static_decode(int device);
void launch_lse_merge(cudaStream_t st, const float* part_o, const float* part_lse, int n_parts, int64_t rows,
                      int head_dim, float* out, float* lse,
                      int64_t o_stride = -1, int64_t lse_stride = -1);
// backend_route.cu: the drop-in Backend ops served from fp16 pages (nbl_ctx_set_paged_kv). Every hook is a no-op
// returning "not handled" while the route is off.
// kWrite: the op overwrites the whole range without reading it; kRecord: an elementwise op about to be recorded on
// the range (a recorded projection writing exactly that range may stay recorded: the op will run after it).
enum class Access { kRead, kWrite, kReadWrite, kRecord };
void route_enable(nbl_ctx* ctx, bool on);
// Ends the route; restore_blocks: paged blocks go back to flat fp32 rows first (not needed when the context is
// being destroyed).
void route_destroy(nbl_ctx* ctx, bool restore_blocks);
// Size to allocate for a Backend::alloc of n_floats (candidate K/V blocks get room for whole 16-position pages).
int64_t route_alloc_floats(nbl_ctx* ctx, int64_t n_floats);
void route_reserve(nbl_ctx* ctx, int64_t n_ctx, int64_t n_heads, int64_t max_rows, int64_t max_width);
// Before an op accesses [p, p + n_floats): recorded ops on it are applied (or dropped when it is overwritten whole),
// paged K/V blocks it overlaps are turned back into flat fp32 rows.
void route_touch(nbl_ctx* ctx, const void* p, int64_t n_floats, Access access);
// Where a matmul writes its n x width output meant for y (staging for rows of a paged K/V block; else y).
float* route_output(nbl_ctx* ctx, float* y, int64_t n, int64_t width);
// Backend::matmul_multi of {wq, wk, wv} into {q, K rows, V rows} of a paged pair for up to 8 rows with float weights:
// recorded (true) so attention() can run it with the bias + RoPE + append in its epilogue; false: run it normally.
bool route_matmul_multi(nbl_ctx* ctx, const nbl_weight* const* ws, int32_t count, const float* x, float* const* ys,
                        int64_t n);
// true: recorded or applied; false: the caller launches the ordinary kernel.
bool route_add_bias(nbl_ctx* ctx, float* x, const float* bias, int64_t width, int64_t n);
bool route_rope(nbl_ctx* ctx, float* x, int64_t n, int64_t heads, int64_t head_dim, int64_t pos0,
                const nbl_rope_params& rp);
bool route_attention(nbl_ctx* ctx, const float* q, const float* k, const float* v, float* out, int64_t n,
                     int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim);
// Before Backend::free of p (the surviving block of a paged pair is turned back into flat rows).
void route_free(nbl_ctx* ctx, void* p);
// Launches a recorded Q/K/V projection (before the scratch it reads is replaced).
void route_flush_projection(nbl_ctx* ctx);
// Applies recorded query ops (before entry points outside the Backend set read arbitrary device memory).
void route_flush_queries(nbl_ctx* ctx);

// decode.cu: the long-context exchange over peer memory (nbl_lse_exchange_peers); at most kMaxPeers ranks.
constexpr int kMaxPeers = 8;
void launch_lse_exchange_peers(cudaStream_t st, const float* send, int64_t rows, int head_dim, int world, int rank,
                               float* const* recv, uint32_t* const* flags, uint32_t* sync, float* out, float* lse,
                               int* err, int num_sms);
// The decode with that exchange fused in (nbl_attn_decode_peers): the decode kernel stores every finished
// (row, head) straight into every rank's receive buffer and raises the flags; then the merge.
void launch_decode_peers(cudaStream_t st, const nbl_kv* kv, const float* q, const int32_t* page_table,
                         int32_t pt_stride, const int32_t* seq_lens, int n_rows, int n_heads, const DecodePlan& plan,
                         void* scratch, unsigned* counts, int world, int rank, float* const* recv,
                         uint32_t* const* flags, uint32_t* sync, float* out, float* lse, int* err, int num_sms);

// prefill.cu
void launch_prefill(cudaStream_t st, const nbl_kv* kv, const void* q, int64_t n_q_rows, const int32_t* q_start,
                    const int32_t* q_len, const int32_t* kv_pos0, const int32_t* page_table, int32_t pt_stride,
                    int n_items, int n_heads, int max_q_len, void* out, int out_dtype, int* err);

}  // namespace nbl
