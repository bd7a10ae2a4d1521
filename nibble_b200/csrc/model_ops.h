// Device weights and the launches of the model's non-attention ops (model_ops.cu), shared with api.cu.
#pragma once

#include "nbl_internal.h"

namespace nbl {

// Activation rows up to which a matmul runs as the weight-streaming GEMV (decode); more rows use a GEMM.
constexpr int64_t kGemvMaxRows = 8;

// A quantized weight's device arrays (quant_ops.cu): fp16 scale bits [rows][blocks], value bytes
// [rows][blocks][16 or 32] (16-byte aligned), Q5_0's high bits [rows][blocks].
struct QWeightView {
  const uint16_t* d = nullptr;
  const uint8_t* qs = nullptr;
  const uint32_t* qh = nullptr;
};

// The operands of the tensor-core path of a quantized matmul (quant_gemm.cu), made on the weight's first multi-row
// matmul: its values as int8 [rows][ne0] (Q8_0's device values themselves; an unpacked copy for Q4_0 and Q5_0) and
// its block scales as fp32 [blocks][rows padded to 4], with their TMA descriptors.
struct QGemmOperand {
  CUtensorMap vmap, smap;
  const int8_t* vals = nullptr;
  int8_t* owned = nullptr;
  float* scales_t = nullptr;
};

// One weight tensor on the device: ne1 rows of ne0 elements (F32, F16 or a quantized type). For a quantized type
// `dev` holds the arrays `q` points into.
struct Weight {
  int32_t dtype = NBL_F32;
  int64_t ne0 = 0, ne1 = 0;
  void* dev = nullptr;
  float *tf_hi = nullptr, *tf_lo = nullptr;  // an F32 matrix split into two tf32 terms for the tensor-core GEMM
  QWeightView q;
  QGemmOperand* qg = nullptr;
};

void launch_embed(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out, int num_sms);
// Up to kMaxMulti weights sharing one input, run as one GEMV launch (rows numbered consecutively).
constexpr int kMaxMulti = 4;
struct GemvBatch {
  const void* w[kMaxMulti];
  float* y[kMaxMulti];
  int64_t row_end[kMaxMulti];  // cumulative row counts
  int count;
};
struct QBatch {
  QWeightView w[kMaxMulti];
  float* y[kMaxMulti];
  int64_t row_end[kMaxMulti];  // cumulative row counts
  int count;
};
void launch_gemv(cudaStream_t st, const Weight& w, const float* x, float* y, int64_t n, int num_sms);
// The epilogue of the fused Q/K/V projection (launch_gemv_qkv): what the reference does to the projections' outputs
// before attention (src/model/transformer.cpp:171-198), applied to the dot products before they are stored.
struct QkvEpilogue {
  const float* bq = nullptr;  // biases (fp32, device) or null
  const float* bk = nullptr;
  const float* bv = nullptr;
  float* q_out = nullptr;     // [n][n_heads * 64] fp32: rope(x . Wq^T + bq)
  void* pool = nullptr;       // fp16 pages [n_pages][2][n_kv_heads][16][64]
  int64_t n_pages = 0;
  const int32_t* page_table = nullptr;  // the sequence's page ids (one row)
  int32_t pt_stride = 0;
  const float2* tab = nullptr;          // RoPE (cos, sin) [tab_pos][32]
  int64_t tab_pos = 0;
  int32_t pos0 = 0;                     // position of activation row 0 (row t is at pos0 + t)
  int32_t n_heads = 0, n_kv_heads = 0;
  int32_t neox = 0;
  int* err = nullptr;
};
// y = x . W^T for the Q, K and V weights (ws[0..2], F32 or F16, head_dim 64) of n <= kGemvMaxRows activation rows, with
// the epilogue fused: each warp computes both members of a RoPE pair (NeoX (i, i+32) or interleaved (2i, 2i+1)) of
// one head, adds the bias, rotates Q and K at the row's position, writes q to e.q_out and K / V narrowed to fp16 (RNE)
// into their page slots. The same arithmetic as the GEMV followed by nbl_rope_kv_append, bit for bit. False when the
// weights do not qualify (caller runs the unfused path).
bool gemv_qkv_ok(const Weight* const* ws, const float* x, int64_t n, int64_t n_heads, int64_t n_kv_heads);
bool launch_gemv_qkv(cudaStream_t st, const Weight* const* ws, const float* x, int64_t n, const QkvEpilogue& e,
                     int num_sms);
// All weights share ne0; n rows of x. Weights of mixed dtype, or unaligned ones, run one scalar launch each.
void launch_gemv_multi(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x,
                       int64_t n, int num_sms);
// y[n][ne1] = x . W^T for an F32 / F16 weight whose row width the tensor-core GEMM cannot tile (fgemm_supported
// false): an fp32 CUDA-core GEMM of this library, any shape.
void launch_gemm_fallback(cudaStream_t st, const Weight& w, const float* x, float* y, int64_t n);
// f32_gemm.cu: the float matmul for more than kGemvMaxRows rows on the tensor cores at fp32 accuracy (activations
// split into two 11-bit terms), for up to kMaxMulti weights of one type sharing x and ne0 in one launch. F16 weights:
// w_hi[i] = the device fp16 matrix, w_lo[i] = NULL (kind::f16); F32 weights: w_hi[i] / w_lo[i] = the matrix's two
// tf32 terms (kind::tf32). act holds the activation terms, their scales and the split-K partials
// (fgemm_act_bytes over the weights' total rows). Row widths TMA cannot tile are refused (fgemm_supported).
bool fgemm_supported(int32_t dtype, int64_t ne0);
size_t fgemm_act_bytes(int64_t n, int64_t rows, int64_t ne0);
void split_tf32(cudaStream_t st, const float* x, float* hi, float* lo, int64_t count, int num_sms);
void launch_fgemm(cudaStream_t st, const void* const* w_hi, const float* const* w_lo, const int64_t* rows,
                  float* const* ys, int count, int64_t ne0, const float* x, int64_t n, void* act, int num_sms,
                  int* err);
// quant_ops.cu: the Q8_0-activation weight family (Q4_0, Q5_0, Q8_0)
bool is_quant(int32_t dtype);
int64_t quant_block_bytes(int32_t dtype);  // GGUF bytes per 32-element block
int64_t quant_qs_bytes(int32_t dtype);     // value bytes per block in the device layout
// Weights of one quantized type sharing ne0 and the fp32 activations x (n rows, in chunks of kGemvMaxRows, each
// quantized to Q8_0 blocks into `act` -- gemv_q_act_bytes(ne0) -- by a launch of its own).
size_t gemv_q_act_bytes(int64_t ne0);
void launch_gemv_q(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x, int64_t n,
                   void* act, int num_sms);
void launch_embed_q(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out);
// The fused Q/K/V projection (see launch_gemv_qkv) for Q4_0 / Q5_0 / Q8_0 weights: x quantized into act, then the
// quantized GEMV with the bias + RoPE + fp16 page write in its epilogue; block dots bit-identical to launch_gemv_q.
// The context's scratch for the quantized GEMV's activations (grown to gemv_q_act_bytes(ne0) on first need).
void* qgemv_scratch(nbl_ctx* ctx, int64_t ne0);
bool gemv_q_qkv_ok(const Weight* const* ws, int64_t n, int64_t n_heads, int64_t n_kv_heads);
bool launch_gemv_q_qkv(cudaStream_t st, const Weight* const* ws, const float* x, int64_t n, void* act,
                       const QkvEpilogue& e, int num_sms);
// quant_gemm.cu: the same matmul for more than kGemvMaxRows activation rows, on the tensor cores. prepare_qgemm
// makes a weight's operands (once); launch_qgemm quantizes x into `act` (qgemm_act_bytes) and runs weights of one
// quantized type sharing ne0 (count <= kMaxMulti, each prepared).
void prepare_qgemm(cudaStream_t st, Weight& w, int num_sms);
void release_qgemm(QGemmOperand* g);
size_t qgemm_act_bytes(int64_t n, int64_t ne0);
void launch_qgemm(cudaStream_t st, const Weight* const* ws, float* const* ys, int count, const float* x, int64_t n,
                  void* act, int num_sms, int* err);

// quant_blocks.cu: Q5_1 (Q8_1 activations) and the k-quants Q4_K / Q5_K / Q6_K (Q8_K activations), weights kept
// in their GGUF block layout. launch_qblock_matmul quantizes the n rows of x into `act` (qblock_act_bytes) and
// runs the block dots.
bool is_qblock(int32_t dtype);
int64_t qblock_elems(int32_t dtype);  // elements per block: 32 or 256
int64_t qblock_bytes(int32_t dtype);  // GGUF bytes per block
size_t qblock_act_bytes(int32_t dtype, int64_t n, int64_t ne0);
void launch_qblock_matmul(cudaStream_t st, const Weight& w, float* y, const float* x, int64_t n, void* act,
                          int num_sms);
void launch_embed_qblock(cudaStream_t st, const Weight& table, const int32_t* ids, int64_t n, float* out,
                         int num_sms);

void launch_rmsnorm(cudaStream_t st, const float* x, const float* w, float* y, int64_t n, int64_t d, float eps);
void launch_add(cudaStream_t st, float* x, const float* y, int64_t count, int num_sms);
void launch_silu_mul(cudaStream_t st, float* gate, const float* up, int64_t count, int num_sms);

}  // namespace nbl

struct nbl_weight {
  nbl_ctx* ctx = nullptr;
  nbl::Weight w;
};
