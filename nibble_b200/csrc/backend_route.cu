// The drop-in Backend path onto the paged kernels: nibble's Transformer hands CudaBackend flat fp32 K/V blocks
// ([n_ctx, n_kv_heads, head_dim] per layer, src/model/transformer.cpp:74-90) and writes them through ordinary ops
// (matmul_multi straight into cache rows, add_bias, rope, transformer.cpp:171-198) before calling attention (:201).
// With the route on (nbl_ctx_set_paged_kv), the library serves those same calls from fp16 pages:
//
//   * recognition: the first attention() on a (k, v) pair of blocks from nbl_alloc binds them; the pair's pages
//     live inside k's own memory (a page = 16 positions x [K | V] x n_kv_heads x 64 fp16 = exactly the bytes of
//     16 fp32 rows of one block), so page p sits where fp32 rows 16p..16p+15 of k were and conversion runs in
//     place, one CTA per page; v's memory is then unused. No allocation happens after reserve.
//   * deferral: while a pair is paged, a matmul output aimed at its rows lands in a staging buffer instead, and
//     add_bias / rope on those rows, and add_bias / rope on the query rows, are recorded rather than launched;
//   * fusion: attention() then runs ONE bias + RoPE + fp16 append launch (rope_kv_append) writing the new rows
//     into their pages and the roped queries, followed by the split-K decode kernel (n <= 8 rows) or the tcgen05
//     prefill kernel (n > 8 rows, queries narrowed to fp16 by the same launch). For up to 8 rows with float or
//     Q4_0 / Q5_0 / Q8_0 weights the Q/K/V matmul_multi itself is recorded too, and attention() runs it as the projection GEMV with the
//     bias + RoPE + page write in its epilogue (launch_gemv_qkv): projection, append and rotation in one launch.
//
// Anything else that touches a paged pair (a read, a copy into its rows, an op on the staged rows) first turns
// it back into flat fp32 rows -- pages widened in place, staged rows written out with their deferred ops applied
// -- so every Backend op keeps its meaning; the next attention() re-binds the pair. Deferred query ops are applied
// as soon as anything but attention() reads the rows. The results are the reference's with K/V stored in fp16:
// the bias add, the rotation (cpu::rope's separately rounded products, src/backend/cpu/ref_ops.cpp:166-185) and
// the RNE narrowing are the same operations in the fused kernel as in the unfused ones, so both orders give the
// same bits.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "model_ops.h"
#include "nbl_internal.h"

namespace nbl {

namespace {

constexpr int kPage = 16;
constexpr int kHd = 64;
constexpr int kDecodeRows = 8;                 // up to this many query rows run as decode rows (fp32 accuracy)
constexpr int kMaxPageBytes = 200 * 1024;      // shared memory of the in-place page conversion (n_kv_heads <= 50)

// ---------------------------------------------------------------- kernels
// Page image in shared memory: [2 (K, V)][n_kv_heads][16 slots][64] fp16, the pool's page layout. A chunk is 8
// consecutive elements of one row (one uint4 of fp16, two float4 of fp32).

__device__ __forceinline__ uint4 narrow8(const float* src) {
  const float4 a = reinterpret_cast<const float4*>(src)[0];
  const float4 b = reinterpret_cast<const float4*>(src)[1];
  uint4 r;
  __half2 h;
  h = __floats2half2_rn(a.x, a.y);
  r.x = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2half2_rn(a.z, a.w);
  r.y = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2half2_rn(b.x, b.y);
  r.z = *reinterpret_cast<uint32_t*>(&h);
  h = __floats2half2_rn(b.z, b.w);
  r.w = *reinterpret_cast<uint32_t*>(&h);
  return r;
}

__device__ __forceinline__ void widen8(uint4 v, float* dst) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    const float2 x = __half22float2(h);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
  reinterpret_cast<float4*>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// Writes positions [row0, row0 + n) into pages page0 + blockIdx.x: K from src_k, V from src_v (fp32 rows of kvw
// floats; row r holds position src_pos0 + r; a NULL side is left as it is), narrowed to fp16 (RNE). Every CTA
// reads all of its page's rows into shared memory before writing, so a source may be the pool memory itself
// (in-place conversion of a flat block: page p's bytes are rows 16p..16p+15 of that block).
__global__ void __launch_bounds__(256) pages_from_rows_kernel(uint4* __restrict__ pool, const float* src_k,
                                                              const float* src_v, int64_t src_pos0, int64_t row0,
                                                              int64_t n, int kvh, int64_t page0) {
  extern __shared__ uint4 img[];
  const int64_t page = page0 + blockIdx.x;
  const int kvw = kvh * kHd, cpr = kvw / 8;  // chunks per row
  const int64_t lo = max(row0, page * kPage), hi = min(row0 + n, page * kPage + kPage);
  const int rows = static_cast<int>(hi - lo);
  const int total = 2 * rows * cpr;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int side = i / (rows * cpr), rem = i % (rows * cpr), r = rem / cpr, c = rem % cpr;
    const float* src = side ? src_v : src_k;
    if (!src) continue;
    const int64_t pos = lo + r;
    const int slot = static_cast<int>(pos - page * kPage), h = c >> 3;
    img[((side * kvh + h) * kPage + slot) * 8 + (c & 7)] = narrow8(src + (pos - src_pos0) * kvw + c * 8);
  }
  __syncthreads();
  uint4* dst = pool + page * int64_t(kvh) * 256;  // 2 * kvh * 16 * 64 halves = kvh * 256 uint4
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int side = i / (rows * cpr), rem = i % (rows * cpr), r = rem / cpr, c = rem % cpr;
    if (!(side ? src_v : src_k)) continue;
    const int slot = static_cast<int>(lo + r - page * kPage), h = c >> 3;
    const int idx = ((side * kvh + h) * kPage + slot) * 8 + (c & 7);
    dst[idx] = img[idx];
  }
}

// Widens page blockIdx.x back into fp32 rows 16p..16p+15: K into dst_k, V into dst_v (NULL: that side is not
// written). The page is read whole into shared memory first, so dst_k may be the pool memory itself.
__global__ void __launch_bounds__(256) rows_from_pages_kernel(const uint4* pool, float* dst_k, float* dst_v,
                                                              int kvh) {
  extern __shared__ uint4 img[];
  const int64_t page = blockIdx.x;
  const int kvw = kvh * kHd, cpr = kvw / 8, words = kvh * 256;
  const uint4* src = pool + page * int64_t(words);
  for (int i = threadIdx.x; i < words; i += blockDim.x) img[i] = src[i];
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * kPage * cpr; i += blockDim.x) {
    const int side = i / (kPage * cpr), rem = i % (kPage * cpr), slot = rem / cpr, c = rem % cpr;
    float* dst = side ? dst_v : dst_k;
    if (!dst) continue;
    const int h = c >> 3;
    widen8(img[((side * kvh + h) * kPage + slot) * 8 + (c & 7)], dst + (page * kPage + slot) * kvw + c * 8);
  }
}

// The per-chunk index arrays the paged kernels read: tok_row[i] = 0 (one sequence), tok_pos[i] = pos0 + i,
// lens[i] = pos0 + i + 1 (decode row i attends its causal prefix), and one prefill item {q_start 0, q_len n,
// kv_pos0 pos0}.
__global__ void route_meta_kernel(int32_t* meta, int64_t cap, int32_t pos0, int32_t n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    meta[i] = 0;
    meta[cap + i] = pos0 + i;
    meta[2 * cap + i] = pos0 + i + 1;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    meta[3 * cap] = 0;
    meta[3 * cap + 1] = n;
    meta[3 * cap + 2] = pos0;
  }
}

// rows x cols identity page table: t[r][c] = c.
__global__ void iota_rows_kernel(int32_t* t, int64_t rows, int64_t cols) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < rows * cols; i += int64_t(gridDim.x) * blockDim.x)
    t[i] = static_cast<int32_t>(i % cols);
}

// fp32 -> fp16 (RNE), for queries roped outside the fused append.
__global__ void narrow_kernel(const float* __restrict__ x, __half* __restrict__ y, int64_t count) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    y[i] = __float2half_rn(x[i]);
}

}  // namespace

// ---------------------------------------------------------------- host state
struct RouteRope {
  bool on = false;
  int64_t heads = 0, head_dim = 0, pos0 = 0;
  float base = 0.f;
  int32_t neox = 0;
  std::vector<float> factors;
  nbl_rope_params params() const { return {base, neox, factors.empty() ? nullptr : factors.data()}; }
  bool same_params(const RouteRope& o) const { return base == o.base && neox == o.neox && factors == o.factors; }
};

// Elementwise work recorded instead of launched on n rows of `width` floats at p: a bias add, then a rotation.
struct Deferred {
  bool on = false;
  float* p = nullptr;
  int64_t n = 0, width = 0;
  const float* bias = nullptr;
  RouteRope rope;
};

// K or V rows [row0, row0 + n) of a paged pair, held in the staging buffer (p) until attention() appends them.
struct Staged : Deferred {
  int64_t row0 = 0;
};

struct Binding {
  float* k = nullptr;
  float* v = nullptr;
  int64_t n_ctx = 0, n_pages = 0, kvw = 0;
  int kvh = 0;
  nbl_kv kv{};  // pool view over k's memory (not owned, not in ctx->kvs)
  bool paged = false;
  Staged sk, sv;
  bool overlaps(uintptr_t a, uintptr_t b) const {
    const uintptr_t k0 = reinterpret_cast<uintptr_t>(k), v0 = reinterpret_cast<uintptr_t>(v);
    const uintptr_t span = static_cast<uintptr_t>(n_pages) * kPage * static_cast<uintptr_t>(kvw) * sizeof(float);
    return (a < k0 + span && k0 < b) || (a < v0 + span && v0 < b);
  }
};

// A recorded Q/K/V projection: matmul_multi({wq, wk, wv}, x, {q, K rows, V rows}, n) whose K/V outputs are the
// staged rows of `b`; not yet launched.
struct Projection {
  bool on = false;
  const Weight* w[3] = {nullptr, nullptr, nullptr};
  const float* x = nullptr;
  int64_t n = 0;
  float* q = nullptr;
  Binding* b = nullptr;
  void* act = nullptr;  // quantized weights: the activation scratch of the quantized GEMV
};

struct Route {
  float* stage = nullptr;  // [2 (K, V)][stage_rows][stage_width] fp32
  int64_t stage_rows = 0, stage_width = 0;
  __half* q16 = nullptr;  // roped queries for the prefill kernel
  int64_t q16_elems = 0;
  int32_t* meta = nullptr;  // tok_row | tok_pos | lens (meta_rows each) | q_start, q_len, kv_pos0
  int64_t meta_rows = 0;
  int32_t* ident = nullptr;  // kDecodeRows identity page-table rows of ident_pages entries
  int64_t ident_pages = 0;
  int64_t meta_pos0 = -1, meta_n = -1;
  cudaStream_t meta_stream = nullptr;
  std::vector<std::unique_ptr<Binding>> binds;
  Deferred pq;  // recorded bias / rope on a buffer that is not K/V (the query rows)
  Projection proj;
};

namespace {

Route* route_of(nbl_ctx* ctx) { return ctx ? static_cast<Route*>(ctx->route) : nullptr; }

void launch_check(const char* what) { check_cuda(cudaGetLastError(), what); }

// A recorded projection, launched as the plain GEMV into its outputs (the query rows and the K/V staging).
void flush_projection(nbl_ctx* ctx, Route& r) {
  if (!r.proj.on) return;
  Projection& p = r.proj;
  float* ys[3] = {p.q, p.b->sk.p, p.b->sv.p};
  if (is_quant(p.w[0]->dtype)) launch_gemv_q(ctx->stream, p.w, ys, 3, p.x, p.n, p.act, ctx->num_sms);
  else launch_gemv_multi(ctx->stream, p.w, ys, 3, p.x, p.n, ctx->num_sms);
  launch_check("projection launch");
  p = Projection{};
}

bool range_overlaps(const void* p, int64_t floats, const void* q, int64_t q_floats) {
  const auto a = reinterpret_cast<uintptr_t>(p), b = a + static_cast<uintptr_t>(floats) * sizeof(float);
  const auto c = reinterpret_cast<uintptr_t>(q), d = c + static_cast<uintptr_t>(q_floats) * sizeof(float);
  return a < d && c < b;
}

int grid_for(int64_t work, int num_sms) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, int64_t(num_sms) * 8)));
}

void set_page_smem(const void* fn, int bytes) {
  if (bytes > 48 * 1024)
    check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), "page smem attribute");
}

// Runs the recorded bias / rotation of d on its rows (the same kernels nbl_add_bias / nbl_rope launch), after the
// recorded projection that writes those rows.
void apply(nbl_ctx* ctx, Deferred& d) {
  Route& r = *route_of(ctx);
  if ((d.bias || d.rope.on) && r.proj.on &&
      (d.p == r.proj.q || d.p == r.proj.b->sk.p || d.p == r.proj.b->sv.p))
    flush_projection(ctx, r);
  if (d.bias) {
    launch_add_bias(ctx->stream, d.p, d.bias, d.width, d.n);
    launch_check("add_bias launch");
    d.bias = nullptr;
  }
  if (d.rope.on) {
    const nbl_rope_params rp = d.rope.params();
    const auto& tab = rope_table(ctx, rp, d.rope.head_dim, d.rope.pos0 + d.n);
    launch_rope_f32(ctx->stream, d.p, d.n, d.rope.heads, d.rope.head_dim, d.rope.pos0, rp.neox != 0, tab.dev,
                    ctx->d_err);
    launch_check("rope launch");
    d.rope.on = false;
  }
}

void convert_rows_to_pages(nbl_ctx* ctx, Binding& b, const float* src_k, const float* src_v, int64_t src_pos0,
                           int64_t row0, int64_t n) {
  if (n <= 0) return;
  const int64_t p0 = row0 / kPage, p1 = (row0 + n - 1) / kPage + 1;
  const int smem = b.kvh * 4096;
  set_page_smem(reinterpret_cast<const void*>(pages_from_rows_kernel), smem);
  pages_from_rows_kernel<<<static_cast<unsigned>(p1 - p0), 256, smem, ctx->stream>>>(
      static_cast<uint4*>(b.kv.pool), src_k, src_v, src_pos0, row0, n, b.kvh, p0);
  launch_check("page conversion launch");
}

// Staged rows of one side: deferred ops applied, then narrowed into their pages.
void flush_staged(nbl_ctx* ctx, Binding& b, Staged& s, bool is_v) {
  if (!s.on) return;
  if (route_of(ctx)->proj.on && route_of(ctx)->proj.b == &b) flush_projection(ctx, *route_of(ctx));
  apply(ctx, s);
  convert_rows_to_pages(ctx, b, is_v ? nullptr : s.p, is_v ? s.p : nullptr, s.row0, s.row0, s.n);
  s = Staged{};
}

// Pages -> flat fp32 rows (K in place, V into v's block when write_v), then staged rows written over their rows.
void demote(nbl_ctx* ctx, Binding& b, bool write_k = true, bool write_v = true) {
  if (!b.paged) return;
  if (route_of(ctx)->proj.on && route_of(ctx)->proj.b == &b) flush_projection(ctx, *route_of(ctx));
  apply(ctx, b.sk);
  apply(ctx, b.sv);
  const int smem = b.kvh * 4096;
  set_page_smem(reinterpret_cast<const void*>(rows_from_pages_kernel), smem);
  rows_from_pages_kernel<<<static_cast<unsigned>(b.n_pages), 256, smem, ctx->stream>>>(
      static_cast<const uint4*>(b.kv.pool), write_k ? b.k : nullptr, write_v ? b.v : nullptr, b.kvh);
  launch_check("page widening launch");
  for (Staged* s : {&b.sk, &b.sv}) {
    if (!s->on) continue;
    float* base = s == &b.sk ? b.k : b.v;
    if ((s == &b.sk && write_k) || (s == &b.sv && write_v))
      check_cuda(cudaMemcpyAsync(base + s->row0 * b.kvw, s->p, static_cast<size_t>(s->n * b.kvw) * sizeof(float),
                                 cudaMemcpyDeviceToDevice, ctx->stream),
                 "staged rows copy");
    *s = Staged{};
  }
  b.paged = false;
}

void adopt(nbl_ctx* ctx, Binding& b) {
  if (b.paged) return;
  convert_rows_to_pages(ctx, b, b.k, b.v, 0, 0, b.n_pages * kPage);
  b.paged = true;
}

void unbind(nbl_ctx* ctx, Route& r, Binding* b, bool write_k, bool write_v) {
  demote(ctx, *b, write_k, write_v);
  r.binds.erase(std::remove_if(r.binds.begin(), r.binds.end(), [&](const auto& p) { return p.get() == b; }),
                r.binds.end());
}

bool overlaps(const Deferred& d, uintptr_t a, uintptr_t b) {
  const uintptr_t p0 = reinterpret_cast<uintptr_t>(d.p);
  return d.on && a < p0 + static_cast<uintptr_t>(d.n * d.width) * sizeof(float) && p0 < b;
}

// The paged pair whose k or v block holds address p, or null.
Binding* binding_at(Route& r, const void* p, bool* is_v = nullptr) {
  const auto a = reinterpret_cast<uintptr_t>(p);
  for (auto& b : r.binds) {
    const uintptr_t span = static_cast<uintptr_t>(b->n_pages) * kPage * static_cast<uintptr_t>(b->kvw) * sizeof(float);
    const auto k0 = reinterpret_cast<uintptr_t>(b->k), v0 = reinterpret_cast<uintptr_t>(b->v);
    if (a >= k0 && a < k0 + span) {
      if (is_v) *is_v = false;
      return b.get();
    }
    if (a >= v0 && a < v0 + span) {
      if (is_v) *is_v = true;
      return b.get();
    }
  }
  return nullptr;
}

void fill_meta(nbl_ctx* ctx, Route& r, int64_t pos0, int64_t n) {
  if (r.meta_pos0 == pos0 && r.meta_n == n && r.meta_stream == ctx->stream) return;
  route_meta_kernel<<<grid_for(n, ctx->num_sms), 256, 0, ctx->stream>>>(r.meta, r.meta_rows, static_cast<int32_t>(pos0),
                                                                         static_cast<int32_t>(n));
  launch_check("route meta launch");
  r.meta_pos0 = pos0;
  r.meta_n = n;
  r.meta_stream = ctx->stream;
}

template <class T>
void grow(nbl_ctx* ctx, T*& buf, size_t bytes, const char* what) {
  if (buf) {
    check_cuda(cudaStreamSynchronize(ctx->stream), what);
    cudaFree(buf);
    buf = nullptr;
  }
  buf = static_cast<T*>(device_alloc(bytes, what));
}

void ensure_ident(nbl_ctx* ctx, Route& r, int64_t pages) {
  if (r.ident_pages >= pages) return;
  grow(ctx, r.ident, static_cast<size_t>(kDecodeRows * pages) * sizeof(int32_t), "identity page table");
  iota_rows_kernel<<<grid_for(kDecodeRows * pages, ctx->num_sms), 256, 0, ctx->stream>>>(r.ident, kDecodeRows, pages);
  launch_check("identity page table");
  r.ident_pages = pages;
}

// The pair (k, v) bound, or bound now if the blocks qualify; null when they do not (the flat kernels run).
Binding* bind(nbl_ctx* ctx, Route& r, const float* k, const float* v, int64_t kvh, int64_t pos0, int64_t n) {
  for (auto& b : r.binds)
    if (b->k == k && b->v == v && b->kvh == kvh) return b.get();
  // blocks bound in another pairing or geometry go back to flat rows first
  for (const float* p : {k, v})
    while (Binding* other = binding_at(r, p)) unbind(ctx, r, other, true, true);
  if (kvh <= 0 || kvh * 4096 > kMaxPageBytes) return nullptr;
  const auto ik = ctx->allocs.find(const_cast<float*>(k)), iv = ctx->allocs.find(const_cast<float*>(v));
  if (ik == ctx->allocs.end() || iv == ctx->allocs.end() || k == v) return nullptr;
  const int64_t kvw = kvh * kHd;
  if (ik->second.floats != iv->second.floats || ik->second.floats % kvw) return nullptr;
  const int64_t n_ctx = ik->second.floats / kvw, n_pages = (n_ctx + kPage - 1) / kPage;
  const size_t need = static_cast<size_t>(n_pages) * kPage * static_cast<size_t>(kvw) * sizeof(float);
  if (pos0 + n > n_ctx || ik->second.bytes < need || iv->second.bytes < need) return nullptr;
  const uint64_t rows = static_cast<uint64_t>(n_pages) * 2u * static_cast<uint64_t>(kvh) * kPage;
  if (rows >= (1ull << 31)) return nullptr;
  ensure_ident(ctx, r, n_pages);
  auto b = std::make_unique<Binding>();
  b->k = const_cast<float*>(k);
  b->v = const_cast<float*>(v);
  b->n_ctx = n_ctx;
  b->n_pages = n_pages;
  b->kvw = kvw;
  b->kvh = static_cast<int>(kvh);
  b->kv.ctx = ctx;
  b->kv.cfg = nbl_kv_config{n_pages, static_cast<int32_t>(kvh), kHd, kPage, NBL_F16};
  b->kv.pool = b->k;
  b->kv.bytes = rows * kHd * 2u;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHd), rows};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHd) * 2u};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kHd), static_cast<cuuint32_t>(kPage)};
  encode_tmap(&b->kv.tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b->kv.pool, dims, strides, box);
  b->kv.has_tmap = true;
  r.binds.push_back(std::move(b));
  return r.binds.back().get();
}

}  // namespace

// ---------------------------------------------------------------- hooks (declared in nbl_internal.h)
void route_enable(nbl_ctx* ctx, bool on) {
  Route* r = route_of(ctx);
  if (on) {
    if (!r) ctx->route = new Route();
    return;
  }
  if (r) route_destroy(ctx, true);
}

void route_destroy(nbl_ctx* ctx, bool restore_blocks) {
  Route* r = route_of(ctx);
  if (!r) return;
  if (restore_blocks) {
    // every block back to flat fp32 rows and every recorded op applied, so the blocks stay valid without the route
    flush_projection(ctx, *r);
    if (r->pq.on) apply(ctx, r->pq);
    while (!r->binds.empty()) unbind(ctx, *r, r->binds.back().get(), true, true);
    check_cuda(cudaStreamSynchronize(ctx->stream), "leaving the paged route");
  }
  if (r->stage) cudaFree(r->stage);
  if (r->q16) cudaFree(r->q16);
  if (r->meta) cudaFree(r->meta);
  if (r->ident) cudaFree(r->ident);
  delete r;
  ctx->route = nullptr;
}

int64_t route_alloc_floats(nbl_ctx* ctx, int64_t n_floats) {
  if (!route_of(ctx) || ctx->reserved_ctx <= 0 || n_floats <= 0 || n_floats % ctx->reserved_ctx) return n_floats;
  const int64_t w = n_floats / ctx->reserved_ctx;
  if (w % kHd) return n_floats;
  // a candidate K/V block: room for whole 16-position pages
  return (ctx->reserved_ctx + kPage - 1) / kPage * kPage * w;
}

void route_reserve(nbl_ctx* ctx, int64_t n_ctx, int64_t n_heads, int64_t max_rows, int64_t max_width) {
  Route* r = route_of(ctx);
  if (!r || max_rows <= 0) return;
  const int64_t width = std::max(max_width, n_heads * kHd);
  if (r->stage_rows < max_rows || r->stage_width < width) {
    const int64_t rows = std::max(r->stage_rows, max_rows), w = std::max(r->stage_width, width);
    grow(ctx, r->stage, static_cast<size_t>(2 * rows * w) * sizeof(float), "K/V staging");
    r->stage_rows = rows;
    r->stage_width = w;
  }
  if (r->q16_elems < max_rows * width) {
    grow(ctx, r->q16, static_cast<size_t>(max_rows * width) * sizeof(__half), "fp16 queries");
    r->q16_elems = max_rows * width;
  }
  if (r->meta_rows < max_rows) {
    grow(ctx, r->meta, static_cast<size_t>(3 * max_rows + 3) * sizeof(int32_t), "route index arrays");
    r->meta_rows = max_rows;
    r->meta_pos0 = r->meta_n = -1;
  }
  ensure_ident(ctx, *r, (n_ctx + kPage - 1) / kPage);
  // split-K partials for up to kDecodeRows decode rows at this context length, for any KV head count
  size_t worst = 0;
  for (int64_t kvh = 1; kvh <= n_heads; ++kvh) {
    if (n_heads % kvh || n_heads / kvh > 8) continue;
    for (int rows = 1; rows <= kDecodeRows; ++rows) {
      const auto p = plan_decode(rows, static_cast<int>(kvh), static_cast<int>(n_heads / kvh), static_cast<int>(n_heads),
                                 static_cast<int>(std::min<int64_t>(n_ctx, INT32_MAX)), kPage, ctx->num_sms, 0);
      worst = std::max(worst, p.scratch_bytes);
    }
  }
  if (worst) ensure_scratch(ctx, worst);
}

void route_touch(nbl_ctx* ctx, const void* p, int64_t n_floats, Access access) {
  Route* r = route_of(ctx);
  if (!r || !p || n_floats <= 0) return;
  const auto a = reinterpret_cast<uintptr_t>(p), b = a + static_cast<uintptr_t>(n_floats) * sizeof(float);
  if (r->proj.on) {
    const Projection& pj = r->proj;
    const bool same_q = p == pj.q && n_floats == pj.n * pj.w[0]->ne1;
    const bool hits_q = range_overlaps(p, n_floats, pj.q, pj.n * pj.w[0]->ne1) && !(access == Access::kRecord && same_q);
    const bool writes_x = access != Access::kRead && range_overlaps(p, n_floats, pj.x, pj.n * pj.w[0]->ne0);
    if (hits_q || writes_x) flush_projection(ctx, *r);
  }
  if (overlaps(r->pq, a, b)) {
    const auto q0 = reinterpret_cast<uintptr_t>(r->pq.p);
    const auto q1 = q0 + static_cast<uintptr_t>(r->pq.n * r->pq.width) * sizeof(float);
    if (access == Access::kWrite && a <= q0 && q1 <= b) r->pq = Deferred{};  // overwritten whole: nothing to apply
    else {
      apply(ctx, r->pq);
      r->pq = Deferred{};
    }
  }
  for (auto& bd : r->binds)
    if (bd->paged && bd->overlaps(a, b)) demote(ctx, *bd);
}

float* route_output(nbl_ctx* ctx, float* y, int64_t n, int64_t width) {
  Route* r = route_of(ctx);
  if (!r) return y;
  bool is_v = false;
  Binding* b = binding_at(*r, y, &is_v);
  if (!b || !b->paged) {
    route_touch(ctx, y, n * width, Access::kWrite);
    return y;
  }
  float* base = is_v ? b->v : b->k;
  const int64_t off = y - base;
  if (width == b->kvw && off % b->kvw == 0 && n <= r->stage_rows && off / b->kvw + n <= b->n_ctx) {
    Staged& s = is_v ? b->sv : b->sk;
    if (s.on) flush_staged(ctx, *b, s, is_v);  // rows staged earlier and never attended: into their pages now
    s.on = true;
    s.row0 = off / b->kvw;
    s.n = n;
    s.width = b->kvw;
    s.p = r->stage + (is_v ? r->stage_rows * r->stage_width : 0);
    return s.p;
  }
  route_touch(ctx, y, n * width, Access::kWrite);
  return y;
}

bool route_matmul_multi(nbl_ctx* ctx, const nbl_weight* const* ws, int32_t count, const float* x,
                        float* const* ys, int64_t n) {
  Route* r = route_of(ctx);
  if (!r || count != 3 || n < 1 || n > kDecodeRows) return false;
  bool kv_is_v = true, vv_is_v = false;
  Binding* b = binding_at(*r, ys[1], &kv_is_v);
  if (!b || !b->paged || kv_is_v || binding_at(*r, ys[2], &vv_is_v) != b || !vv_is_v || binding_at(*r, ys[0]))
    return false;
  const Weight* w[3] = {&ws[0]->w, &ws[1]->w, &ws[2]->w};
  if (w[0]->ne1 % kHd || w[1]->ne1 != b->kvw) return false;
  const bool quant = gemv_q_qkv_ok(w, n, w[0]->ne1 / kHd, b->kvh);
  if (!quant && !gemv_qkv_ok(w, x, n, w[0]->ne1 / kHd, b->kvh)) return false;
  const int64_t off_k = ys[1] - b->k, off_v = ys[2] - b->v;
  if (off_k != off_v || off_k % b->kvw || off_k / b->kvw + n > b->n_ctx || n > r->stage_rows) return false;
  if (range_overlaps(x, n * w[0]->ne0, ys[0], n * w[0]->ne1)) return false;
  // the same bookkeeping a plain matmul_multi does: earlier recorded work on these buffers runs or is dropped
  route_touch(ctx, x, n * w[0]->ne0, Access::kRead);
  route_touch(ctx, ys[0], n * w[0]->ne1, Access::kWrite);
  flush_projection(ctx, *r);
  void* act = quant ? qgemv_scratch(ctx, w[0]->ne0) : nullptr;  // sized as the plain quantized GEMV would
  for (bool is_v : {false, true}) {
    Staged& st = is_v ? b->sv : b->sk;
    if (st.on) flush_staged(ctx, *b, st, is_v);
    st.on = true;
    st.row0 = off_k / b->kvw;
    st.n = n;
    st.width = b->kvw;
    st.p = r->stage + (is_v ? r->stage_rows * r->stage_width : 0);
  }
  r->proj.on = true;
  for (int i = 0; i < 3; ++i) r->proj.w[i] = w[i];
  r->proj.x = x;
  r->proj.n = n;
  r->proj.q = ys[0];
  r->proj.b = b;
  r->proj.act = act;
  return true;
}

// Exactly the staged rows of one side, or null.
static Staged* staged_exact(Binding& b, bool is_v, const float* x, int64_t n, int64_t width) {
  Staged& s = is_v ? b.sv : b.sk;
  float* base = is_v ? b.v : b.k;
  if (!s.on || x != base + s.row0 * b.kvw || n != s.n || width != b.kvw) return nullptr;
  return &s;
}

bool route_add_bias(nbl_ctx* ctx, float* x, const float* bias, int64_t width, int64_t n) {
  Route* r = route_of(ctx);
  if (!r) return false;
  bool is_v = false;
  if (Binding* b = binding_at(*r, x, &is_v); b && b->paged) {
    if (Staged* s = staged_exact(*b, is_v, x, n, width)) {
      apply(ctx, *s);  // a bias after an earlier bias or rotation: those run first
      s->bias = bias;
      return true;
    }
    demote(ctx, *b);
    return false;
  }
  if (r->pq.on && r->pq.p == x && r->pq.n == n && r->pq.width == width && !r->pq.bias && !r->pq.rope.on) {
    r->pq.bias = bias;
    return true;
  }
  route_touch(ctx, x, n * width, Access::kRecord);
  if (r->pq.on) return false;
  r->pq = Deferred{};
  r->pq.on = true;
  r->pq.p = x;
  r->pq.n = n;
  r->pq.width = width;
  r->pq.bias = bias;
  return true;
}

bool route_rope(nbl_ctx* ctx, float* x, int64_t n, int64_t heads, int64_t head_dim, int64_t pos0,
                const nbl_rope_params& rp) {
  Route* r = route_of(ctx);
  if (!r) return false;
  RouteRope rr;
  rr.on = true;
  rr.heads = heads;
  rr.head_dim = head_dim;
  rr.pos0 = pos0;
  rr.base = rp.freq_base;
  rr.neox = rp.neox ? 1 : 0;
  if (rp.freq_factors) rr.factors.assign(rp.freq_factors, rp.freq_factors + head_dim / 2);
  bool is_v = false;
  if (Binding* b = binding_at(*r, x, &is_v); b && b->paged) {
    if (Staged* s = staged_exact(*b, is_v, x, n, heads * head_dim)) {
      if (s->rope.on) apply(ctx, *s);
      if (!is_v && heads == b->kvh && head_dim == kHd && pos0 == s->row0) {
        s->rope = std::move(rr);
        return true;
      }
    }
    demote(ctx, *b);
    return false;
  }
  if (r->pq.on && r->pq.p == x && r->pq.n == n && r->pq.width == heads * head_dim && !r->pq.rope.on) {
    r->pq.rope = std::move(rr);
    return true;
  }
  route_touch(ctx, x, n * heads * head_dim, Access::kRecord);
  if (r->pq.on) return false;
  r->pq = Deferred{};
  r->pq.on = true;
  r->pq.p = x;
  r->pq.n = n;
  r->pq.width = heads * head_dim;
  r->pq.rope = std::move(rr);
  return true;
}

bool route_attention(nbl_ctx* ctx, const float* q, const float* k, const float* v, float* out, int64_t n,
                     int64_t pos0, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
  Route* r = route_of(ctx);
  if (!r || head_dim != kHd || n_heads % n_kv_heads || r->stage_rows == 0 || n > r->stage_rows ||
      n * n_heads * kHd > r->q16_elems || pos0 + n > INT32_MAX)
    return false;
  if (n > r->meta_rows || n_kv_heads * kHd > r->stage_width) return false;
  Binding* b = bind(ctx, *r, k, v, n_kv_heads, pos0, n);
  if (!b) return false;
  if (pos0 + n > b->n_ctx)
    fail(NBL_E_INVALID, "attention: positions " + std::to_string(pos0) + ".." + std::to_string(pos0 + n - 1) +
                            " exceed the K/V block's " + std::to_string(b->n_ctx) + " rows");
  const int64_t H = n_heads, G = n_heads / n_kv_heads;
  const bool decode = n <= kDecodeRows && G <= 8;
  if (!b->paged) {
    // a recorded op on rows of the flat blocks runs before they are converted
    const int64_t span = b->n_pages * kPage * b->kvw;
    route_touch(ctx, b->k, span, Access::kRead);
    route_touch(ctx, b->v, span, Access::kRead);
    adopt(ctx, *b);
  }
  Staged &sk = b->sk, &sv = b->sv;
  Deferred& pq = r->pq;
  const bool fused = sk.on && sv.on && sk.row0 == pos0 && sk.n == n && sv.row0 == pos0 && sv.n == n && sk.rope.on &&
                     sk.rope.pos0 == pos0 && !sv.rope.on && pq.on && pq.p == q && pq.n == n &&
                     pq.width == H * kHd && pq.rope.on && pq.rope.heads == H && pq.rope.head_dim == kHd &&
                     pq.rope.pos0 == pos0 && pq.rope.same_params(sk.rope);
  fill_meta(ctx, *r, pos0, n);
  const int32_t* tok_row = r->meta;
  const int32_t* tok_pos = r->meta + r->meta_rows;
  const int32_t* lens = r->meta + 2 * r->meta_rows;
  const int32_t* item = r->meta + 3 * r->meta_rows;
  float* qw = const_cast<float*>(q);  // the deferred rope(q) of the reference writes q in place
  const bool fused_proj = fused && decode && r->proj.on && r->proj.b == b && r->proj.q == q && r->proj.n == n &&
                          r->proj.w[0]->ne1 == H * kHd;
  if (fused_proj) {
    // the recorded Q/K/V projection with bias + RoPE + fp16 page write in its epilogue: one launch
    const nbl_rope_params rp = sk.rope.params();
    const auto& tab = rope_table(ctx, rp, kHd, b->n_pages * kPage);
    QkvEpilogue e;
    e.bq = pq.bias;
    e.bk = sk.bias;
    e.bv = sv.bias;
    e.q_out = qw;
    e.pool = b->kv.pool;
    e.n_pages = b->n_pages;
    e.page_table = r->ident;
    e.pt_stride = static_cast<int32_t>(r->ident_pages);
    e.tab = tab.dev;
    e.tab_pos = tab.n_pos;
    e.pos0 = static_cast<int32_t>(pos0);
    e.n_heads = static_cast<int32_t>(H);
    e.n_kv_heads = b->kvh;
    e.neox = rp.neox;
    e.err = ctx->d_err;
    const bool launched = is_quant(r->proj.w[0]->dtype)
                              ? launch_gemv_q_qkv(ctx->stream, r->proj.w, r->proj.x, n, r->proj.act, e, ctx->num_sms)
                              : launch_gemv_qkv(ctx->stream, r->proj.w, r->proj.x, n, e, ctx->num_sms);
    if (!launched)
      fail(NBL_E_CUDA, "attention: the recorded projection no longer qualifies for the fused launch");
    launch_check("fused projection launch");
    r->proj = Projection{};
    sk = Staged{};
    sv = Staged{};
    pq = Deferred{};
  } else if (fused) {
    flush_projection(ctx, *r);
    const nbl_rope_params rp = sk.rope.params();
    const auto& tab = rope_table(ctx, rp, kHd, b->n_pages * kPage);
    launch_rope_kv_append(ctx->stream, &b->kv, q, sk.p, sv.p, NBL_F32, pq.bias, sk.bias, sv.bias,
                          decode ? static_cast<void*>(qw) : static_cast<void*>(r->q16), decode ? NBL_F32 : NBL_F16,
                          tok_row, tok_pos, r->ident, static_cast<int32_t>(r->ident_pages), n, static_cast<int>(H),
                          rp.neox != 0, tab.dev, tab.n_pos, ctx->d_err);
    launch_check("fused append launch");
    sk = Staged{};
    sv = Staged{};
    if (decode) pq = Deferred{};  // q now holds rope(q + bq), as after the reference's in-place ops
  } else {
    flush_staged(ctx, *b, sk, false);
    flush_staged(ctx, *b, sv, true);
    route_touch(ctx, q, n * H * kHd, Access::kRead);  // applies recorded ops on q
    if (!decode) {
      narrow_kernel<<<grid_for(n * H * kHd, ctx->num_sms), 256, 0, ctx->stream>>>(q, r->q16, n * H * kHd);
      launch_check("query narrowing launch");
    }
  }
  route_touch(ctx, out, n * H * kHd, Access::kWrite);
  if (decode) {
    const auto plan = plan_decode(static_cast<int>(n), b->kvh, static_cast<int>(G), static_cast<int>(H),
                                  static_cast<int>(pos0 + n), kPage, ctx->num_sms, 0);
    unsigned* counts = nullptr;
    if (plan.scratch_bytes) {
      ensure_scratch(ctx, plan.scratch_bytes);
      counts = split_counts(ctx, n * b->kvh);
    }
    launch_decode(ctx->stream, &b->kv, q, r->ident, static_cast<int32_t>(r->ident_pages), lens, static_cast<int>(n),
                  static_cast<int>(H), out, nullptr, plan, ctx->scratch, ctx->d_err, counts);
  } else {
    launch_prefill(ctx->stream, &b->kv, r->q16, n, item, item + 1, item + 2, r->ident,
                   static_cast<int32_t>(r->ident_pages), 1, static_cast<int>(H), static_cast<int>(n), out, NBL_F32,
                   ctx->d_err);
  }
  return true;
}

void route_free(nbl_ctx* ctx, void* p) {
  Route* r = route_of(ctx);
  if (!r || !p) return;
  flush_projection(ctx, *r);  // its inputs or outputs may be in the block
  auto it = ctx->allocs.find(p);
  const int64_t floats = it == ctx->allocs.end() ? 0 : it->second.floats;
  const auto a = reinterpret_cast<uintptr_t>(p), e = a + static_cast<uintptr_t>(floats) * sizeof(float);
  if (overlaps(r->pq, a, std::max(e, a + 1))) r->pq = Deferred{};  // its rows are going away
  Binding* hit = nullptr;
  for (auto& b : r->binds)
    if (b->k == p || b->v == p) hit = b.get();
  // the surviving block of the pair keeps its rows as flat fp32 (the freed one's are not written)
  if (hit) unbind(ctx, *r, hit, hit->k != p, hit->v != p);
}

void route_flush_projection(nbl_ctx* ctx) {
  Route* r = route_of(ctx);
  if (r && r->proj.on) flush_projection(ctx, *r);
}

void route_flush_queries(nbl_ctx* ctx) {
  Route* r = route_of(ctx);
  if (r && r->proj.on) {
    check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    flush_projection(ctx, *r);
  }
  if (r && r->pq.on) {
    check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    apply(ctx, r->pq);
    r->pq = Deferred{};
  }
}

}  // namespace nbl
