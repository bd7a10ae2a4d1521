// The C ABI (include/nibble_cuda.h): argument validation, context state and kernel dispatch.
//
// Every entry point catches everything at the boundary and turns it into an nbl_status plus a thread-local
// message, the C-side form of nibble's "throw nibble::Error with a self-contained message" convention
// (include/nibble/error.h). No exception crosses the ABI.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "model_ops.h"
#include "nbl_internal.h"

namespace {

thread_local std::string g_last_error;

int set_error(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

template <class F>
int guarded(F&& f) {
  try {
    f();
    return NBL_OK;
  } catch (const nbl::Failure& e) {
    return set_error(e.status, e.what());
  } catch (const std::bad_alloc&) {
    return set_error(NBL_E_NOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return set_error(NBL_E_INVALID, e.what());
  }
}

void require(bool ok, const std::string& msg) {
  if (!ok) nbl::fail(NBL_E_INVALID, msg);
}

// Makes the context's device current for the calling thread.
void use_device(nbl_ctx* ctx) { nbl::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice"); }

}  // namespace

void* nbl::device_alloc(size_t bytes, const char* what) {
  void* p = nullptr;
  const cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error so later calls are not poisoned
    nbl::fail(NBL_E_NOMEM, std::string(what) + ": cannot allocate " + std::to_string(bytes) + " bytes of device memory (" +
                               cudaGetErrorString(e) + ")");
  }
  return p;
}

// Grows the context's split-K scratch to at least `bytes` (device allocation; not during stream capture).
void nbl::ensure_scratch(nbl_ctx* ctx, size_t bytes) {
  if (ctx->scratch_bytes >= bytes) return;
  void* p = device_alloc(bytes, "attention scratch");
  if (ctx->scratch) {
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "scratch sync");
    cudaFree(ctx->scratch);
  }
  ctx->scratch = p;
  ctx->scratch_bytes = bytes;
}

unsigned* nbl::split_counts(nbl_ctx* ctx, int64_t units) {
  if (ctx->split_counts_n >= units) return ctx->split_counts;
  const int64_t n = std::max<int64_t>(units, 4096);
  auto* p = static_cast<unsigned*>(device_alloc(size_t(n) * sizeof(unsigned), "split-K counters"));
  nbl::check_cuda(cudaMemset(p, 0, size_t(n) * sizeof(unsigned)), "split-K counters");
  if (ctx->split_counts) {
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "split-K counters sync");
    cudaFree(ctx->split_counts);
  }
  ctx->split_counts = p;
  ctx->split_counts_n = n;
  return p;
}

// Returns the device cos/sin table for (base, head_dim, factors) covering positions [0, n_pos), building it
// on the host in double with the reference's expression (src/backend/cpu/ref_ops.cpp:173-176) if needed.
const nbl::RopeTable& nbl::rope_table(nbl_ctx* ctx, const nbl_rope_params& rp, int64_t head_dim, int64_t n_pos) {
  const int64_t half = head_dim / 2;
  // the cache hit is the per-call path (every layer of every token): compare in place, allocate nothing
  auto same_factors = [&](const nbl::RopeTable& t) {
    if (!rp.freq_factors) return t.factors.empty();
    return t.factors.size() == static_cast<size_t>(half) &&
           std::memcmp(t.factors.data(), rp.freq_factors, static_cast<size_t>(half) * sizeof(float)) == 0;
  };
  for (auto& t : ctx->rope_tables)
    if (t.base == rp.freq_base && t.head_dim == head_dim && t.n_pos >= n_pos && same_factors(t)) return t;
  std::vector<float> ff;
  if (rp.freq_factors) ff.assign(rp.freq_factors, rp.freq_factors + half);
  // Build (grow to the larger of the request and the reserved context length).
  const int64_t want = std::max<int64_t>(n_pos, ctx->reserved_ctx);
  std::vector<float2> host(static_cast<size_t>(want * half));
  for (int64_t pos = 0; pos < want; ++pos)
    for (int64_t i = 0; i < half; ++i) {
      double theta = static_cast<double>(pos) *
                     std::pow(static_cast<double>(rp.freq_base), -2.0 * static_cast<double>(i) / static_cast<double>(head_dim));
      if (!ff.empty()) theta /= ff[static_cast<size_t>(i)];
      host[static_cast<size_t>(pos * half + i)] = make_float2(static_cast<float>(std::cos(theta)), static_cast<float>(std::sin(theta)));
    }
  auto* dev = static_cast<float2*>(device_alloc(host.size() * sizeof(float2), "RoPE table"));
  nbl::check_cuda(cudaMemcpyAsync(dev, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice, ctx->stream),
                  "RoPE table upload");
  nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "RoPE table upload");
  for (auto it = ctx->rope_tables.begin(); it != ctx->rope_tables.end(); ++it)
    if (it->base == rp.freq_base && it->head_dim == head_dim && it->factors == ff) {  // replace a smaller table
      cudaFree(it->dev);
      ctx->rope_tables.erase(it);
      break;
    }
  nbl::RopeTable t;
  t.base = rp.freq_base;
  t.head_dim = head_dim;
  t.factors = std::move(ff);
  t.n_pos = want;
  t.dev = dev;
  ctx->rope_tables.push_back(std::move(t));
  return ctx->rope_tables.back();
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) nbl::fail(NBL_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

}  // namespace

void nbl::encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base, const cuuint64_t* dims,
                      const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = tensor_map_encoder()(map, dtype, static_cast<cuuint32_t>(rank), base, dims, strides_bytes, box,
                                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) nbl::fail(NBL_E_CUDA, "cuTensorMapEncodeTiled failed (CUresult " + std::to_string(r) + ")");
}

int nbl::record_error(int status, const std::string& msg) { return set_error(status, msg); }

using nbl::device_alloc;
using nbl::ensure_scratch;
using nbl::rope_table;

void* nbl::qgemv_scratch(nbl_ctx* ctx, int64_t ne0) {
  const size_t need = nbl::gemv_q_act_bytes(ne0);
  if (ctx->qgemv_act_bytes < need) {
    nbl::route_flush_projection(ctx);  // a recorded projection reads the old buffer
    if (ctx->qgemv_act) {
      nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "quant gemv scratch");
      cudaFree(ctx->qgemv_act);
      ctx->qgemv_act = nullptr;
      ctx->qgemv_act_bytes = 0;
    }
    ctx->qgemv_act = device_alloc(need, "quant gemv activations");
    ctx->qgemv_act_bytes = need;
  }
  return ctx->qgemv_act;
}

namespace {

bool is_dtype(int32_t d) { return d == NBL_F32 || d == NBL_F16 || d == NBL_BF16; }

// Grows the device token-id staging buffer to n ids.
void ensure_ids(nbl_ctx* ctx, int64_t n) {
  if (ctx->ids_cap >= n) return;
  void* p = device_alloc(static_cast<size_t>(n) * sizeof(int32_t), "token ids");
  if (ctx->ids) {
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "ids sync");
    cudaFree(ctx->ids);
  }
  ctx->ids = static_cast<int32_t*>(p);
  ctx->ids_cap = n;
}

void release_weight(nbl_weight* w) {
  nbl::release_qgemm(w->w.qg);
  if (w->w.tf_hi) cudaFree(w->w.tf_hi);
  if (w->w.tf_lo) cudaFree(w->w.tf_lo);
  cudaFree(w->w.dev);
  delete w;
}

// Grows a context-owned scratch buffer to `need` bytes (waiting for queued work before freeing the old one).
void grow_scratch(nbl_ctx* ctx, void*& buf, size_t& bytes, size_t need, const char* what) {
  if (bytes >= need) return;
  if (buf) {
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), what);
    cudaFree(buf);
    buf = nullptr;
    bytes = 0;
  }
  buf = device_alloc(need, what);
  bytes = need;
}

// The tensor-core GEMM's operand of a float weight: an F16 matrix as uploaded (hi, lo = NULL), or the two tf32
// terms of an F32 matrix (made on its first multi-row matmul).
void fgemm_operand(nbl_ctx* ctx, const nbl_weight* cw, const void** hi, const float** lo) {
  auto* w = const_cast<nbl_weight*>(cw);
  if (w->w.dtype == NBL_F16) {
    *hi = w->w.dev;
    *lo = nullptr;
    return;
  }
  if (!w->w.tf_hi) {
    const int64_t count = w->w.ne0 * w->w.ne1;
    w->w.tf_hi = static_cast<float*>(device_alloc(static_cast<size_t>(count) * sizeof(float), "weight tf32 terms"));
    w->w.tf_lo = static_cast<float*>(device_alloc(static_cast<size_t>(count) * sizeof(float), "weight tf32 terms"));
    nbl::split_tf32(ctx->stream, static_cast<const float*>(w->w.dev), w->w.tf_hi, w->w.tf_lo, count, ctx->num_sms);
  }
  *hi = w->w.tf_hi;
  *lo = w->w.tf_lo;
}

// Float-weight matmuls of n > kGemvMaxRows activation rows for weights sharing x: groups of up to kMaxMulti
// weights of one float type whose rows TMA can tile run as one tensor-core GEMM launch; a row width TMA cannot
// tile runs the library's fp32 CUDA-core GEMM.
void float_gemm(nbl_ctx* ctx, const nbl_weight* const* ws, float* const* ys, int count, const float* x, int64_t n) {
  for (int i0 = 0; i0 < count;) {
    const nbl::Weight& w0 = ws[i0]->w;
    if (!nbl::fgemm_supported(w0.dtype, w0.ne0)) {
      nbl::launch_gemm_fallback(ctx->stream, w0, x, ys[i0], n);
      ++i0;
      continue;
    }
    int c = 1;
    while (c < nbl::kMaxMulti && i0 + c < count && ws[i0 + c]->w.dtype == w0.dtype && ws[i0 + c]->w.ne0 == w0.ne0)
      ++c;
    const void* hi[nbl::kMaxMulti];
    const float* lo[nbl::kMaxMulti];
    int64_t rows[nbl::kMaxMulti];
    int64_t total = 0;
    for (int i = 0; i < c; ++i) {
      fgemm_operand(ctx, ws[i0 + i], &hi[i], &lo[i]);
      rows[i] = ws[i0 + i]->w.ne1;
      total += rows[i];
    }
    grow_scratch(ctx, ctx->fgemm_act, ctx->fgemm_act_bytes, nbl::fgemm_act_bytes(n, total, w0.ne0),
                 "float gemm activations");
    nbl::launch_fgemm(ctx->stream, hi, lo, rows, ys + i0, c, w0.ne0, x, n, ctx->fgemm_act, ctx->num_sms, ctx->d_err);
    i0 += c;
  }
}

// A quantized matmul of n activation rows for weights of one quantized type sharing ne0 (count <= kMaxMulti):
// the GEMV for up to kGemvMaxRows rows, else the tensor-core GEMM (its weight operands made on first use, the
// activation scratch grown to fit).
void quant_matmul(nbl_ctx* ctx, const nbl_weight* const* cws, float* const* ys, int count, const float* x,
                  int64_t n) {
  const nbl::Weight* ws[nbl::kMaxMulti];
  for (int i = 0; i < count; ++i) ws[i] = &cws[i]->w;
  if (n <= nbl::kGemvMaxRows) {
    nbl::launch_gemv_q(ctx->stream, ws, ys, count, x, n, nbl::qgemv_scratch(ctx, ws[0]->ne0), ctx->num_sms);
    return;
  }
  for (int i = 0; i < count; ++i) nbl::prepare_qgemm(ctx->stream, const_cast<nbl_weight*>(cws[i])->w, ctx->num_sms);
  grow_scratch(ctx, ctx->qgemm_act, ctx->qgemm_act_bytes, nbl::qgemm_act_bytes(n, ws[0]->ne0),
               "quant gemm activations");
  nbl::launch_qgemm(ctx->stream, ws, ys, count, x, n, ctx->qgemm_act, ctx->num_sms, ctx->d_err);
}

// A matmul of n activation rows with a Q5_1 or k-quant weight: the rows quantized to Q8_1 / Q8_K blocks in the
// context's scratch (grown to fit), then the block dots.
void qblock_matmul(nbl_ctx* ctx, const nbl_weight* w, float* y, const float* x, int64_t n) {
  grow_scratch(ctx, ctx->qblock_act, ctx->qblock_act_bytes, nbl::qblock_act_bytes(w->w.dtype, n, w->w.ne0),
               "block-quant activations");
  nbl::launch_qblock_matmul(ctx->stream, w->w, y, x, n, ctx->qblock_act, ctx->num_sms);
}

void require_weight(const nbl_ctx* ctx, const nbl_weight* w, const char* what) {
  require(w != nullptr && w->ctx == ctx, std::string(what) + ": weight is NULL or belongs to another context");
}

}  // namespace

extern "C" {

int nbl_abi_version(void) { return NBL_ABI_VERSION; }

size_t nbl_last_error(char* buf, size_t cap) {
  if (buf && cap) {
    const size_t n = std::min(cap - 1, g_last_error.size());
    std::memcpy(buf, g_last_error.data(), n);
    buf[n] = 0;
  }
  return g_last_error.size();
}

int nbl_ctx_create(int device, nbl_ctx** out) {
  return guarded([&] {
    require(out != nullptr, "nbl_ctx_create: out is NULL");
    *out = nullptr;
    int count = 0;
    nbl::check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    require(device >= 0 && device < count, "nbl_ctx_create: device " + std::to_string(device) + " out of range (" +
                                               std::to_string(count) + " devices)");
    nbl::check_cuda(cudaSetDevice(device), "cudaSetDevice");
    int major = 0, minor = 0;
    nbl::check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "cc");
    nbl::check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device), "cc");
    if (major != 10 || minor != 0)
      nbl::fail(NBL_E_UNSUPPORTED, "nbl_ctx_create: this library is built for sm_100a (B200); device " +
                                       std::to_string(device) + " is sm_" + std::to_string(major) + std::to_string(minor));
    auto* ctx = new nbl_ctx();
    ctx->device = device;
    try {
      nbl::check_cuda(cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device), "SM count");
      nbl::check_cuda(cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking), "cudaStreamCreate");
      ctx->stream = ctx->own_stream;
      ctx->d_err = static_cast<int*>(device_alloc(sizeof(int), "error word"));
      nbl::check_cuda(cudaMemset(ctx->d_err, 0, sizeof(int)), "error word init");
      // nbl_attn_decode_static's fixed partials array and kernels, placed now while allocating is allowed
      nbl::prepare_static_decode(device);
    } catch (...) {
      if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
      delete ctx;
      throw;
    }
    *out = ctx;
  });
}

int nbl_ctx_destroy(nbl_ctx* ctx) {
  if (!ctx) return NBL_OK;
  return guarded([&] {
    use_device(ctx);
    nbl::route_destroy(ctx, false);
    cudaStreamSynchronize(ctx->stream);
    for (nbl_kv* kv : ctx->kvs) {
      cudaFree(kv->pool);
      delete kv;
    }
    for (nbl_weight* w : ctx->weights) release_weight(w);
    if (ctx->ids) cudaFree(ctx->ids);
    if (ctx->qgemm_act) cudaFree(ctx->qgemm_act);
    if (ctx->fgemm_act) cudaFree(ctx->fgemm_act);
    if (ctx->qgemv_act) cudaFree(ctx->qgemv_act);
    if (ctx->qblock_act) cudaFree(ctx->qblock_act);
    for (auto& a : ctx->allocs) cudaFree(a.first);
    for (auto& t : ctx->rope_tables) cudaFree(t.dev);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->split_counts) cudaFree(ctx->split_counts);
    if (ctx->io) cudaFree(ctx->io);
    for (cudaEvent_t e : ctx->events) cudaEventDestroy(e);
    if (ctx->up_stream) cudaStreamDestroy(ctx->up_stream);
    if (ctx->down_stream) cudaStreamDestroy(ctx->down_stream);
    if (ctx->aux_stream) cudaStreamDestroy(ctx->aux_stream);
    cudaFree(ctx->d_err);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
  });
}

int nbl_ctx_set_stream(nbl_ctx* ctx, void* stream) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_ctx_set_stream: ctx is NULL");
    ctx->stream = static_cast<cudaStream_t>(stream);  // NULL is CUDA's default stream, as everywhere in CUDA
  });
}

int nbl_ctx_use_own_stream(nbl_ctx* ctx) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_ctx_use_own_stream: ctx is NULL");
    ctx->stream = ctx->own_stream;
  });
}

void* nbl_ctx_stream(nbl_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int nbl_ctx_sync(nbl_ctx* ctx) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_ctx_sync: ctx is NULL");
    use_device(ctx);
    nbl::route_flush_queries(ctx);
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "stream synchronize");
  });
}

int nbl_ctx_check(nbl_ctx* ctx) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_ctx_check: ctx is NULL");
    use_device(ctx);
    nbl::route_flush_queries(ctx);
    int host = 0;
    nbl::check_cuda(cudaMemcpyAsync(&host, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream), "error word");
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "error word");
    if (host) {
      nbl::check_cuda(cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream), "error word reset");
      std::string what;
      if (host & nbl::kErrPageId) what += " page id outside the pool;";
      if (host & nbl::kErrLength) what += " sequence length or position outside the page table / RoPE table;";
      if (host & nbl::kErrTimeout) what += " a bounded wait on a copy or MMA completion gave up;";
      if (host & nbl::kErrTmemAlloc) what += " tensor-memory allocation failed;";
      if (host & nbl::kErrSmemAlign) what += " shared memory was not 1024-byte aligned;";
      nbl::fail(NBL_E_DEVICE, "device-side check failed (flags " + std::to_string(host) + "):" + what);
    }
  });
}

int nbl_ctx_set_paged_kv(nbl_ctx* ctx, int32_t on) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_ctx_set_paged_kv: ctx is NULL");
    use_device(ctx);
    nbl::route_enable(ctx, on != 0);
  });
}

int nbl_reserve(nbl_ctx* ctx, int64_t n_ctx, int64_t n_heads, int64_t max_rows, int64_t max_width) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_reserve: ctx is NULL");
    require(n_ctx >= 0 && n_heads >= 0 && max_rows >= 0 && max_width >= 0,
            "reserve: negative size (n_ctx=" + std::to_string(n_ctx) + " n_heads=" + std::to_string(n_heads) +
                " max_rows=" + std::to_string(max_rows) + " max_width=" + std::to_string(max_width) + ")");
    use_device(ctx);
    ctx->reserved_ctx = std::max(ctx->reserved_ctx, n_ctx);
    ctx->reserved_heads = std::max(ctx->reserved_heads, n_heads);
    // Split-K scratch for one decode row per head set at this context length: the planner's worst case for
    // a single row is one split per 8 pages.
    const auto plan = nbl::plan_decode(1, 1, 1, static_cast<int>(n_heads), static_cast<int>(std::min<int64_t>(n_ctx, INT32_MAX)),
                                       16, ctx->num_sms, 0);
    if (plan.scratch_bytes) ensure_scratch(ctx, plan.scratch_bytes);
    if (max_rows > 0) ensure_ids(ctx, max_rows);
    nbl::route_reserve(ctx, n_ctx, n_heads, max_rows, max_width);
  });
}

int nbl_alloc(nbl_ctx* ctx, int64_t n_floats, float** out) {
  return guarded([&] {
    require(ctx != nullptr && out != nullptr, "nbl_alloc: ctx or out is NULL");
    *out = nullptr;
    if (n_floats < 0) nbl::fail(NBL_E_INVALID, "alloc: negative size " + std::to_string(n_floats) + " floats");
    if (static_cast<uint64_t>(n_floats) > (UINT64_MAX - 255) / sizeof(float))
      nbl::fail(NBL_E_INVALID, "alloc: size of " + std::to_string(n_floats) + " floats overflows");
    use_device(ctx);
    size_t bytes = static_cast<size_t>(nbl::route_alloc_floats(ctx, n_floats)) * sizeof(float);
    bytes = std::max<size_t>((bytes + 255) & ~size_t(255), 256);
    void* p = device_alloc(bytes, "alloc");
    const cudaError_t e = cudaMemsetAsync(p, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
      cudaFree(p);
      nbl::check_cuda(e, "alloc zero-fill");
    }
    try {
      ctx->allocs.emplace(p, nbl_ctx::Alloc{bytes, n_floats});
    } catch (...) {
      cudaFree(p);
      throw;
    }
    *out = static_cast<float*>(p);
  });
}

int nbl_free(nbl_ctx* ctx, float* p) {
  return guarded([&] {
    require(ctx != nullptr, "nbl_free: ctx is NULL");
    if (!p) return;
    auto it = ctx->allocs.find(p);
    if (it == ctx->allocs.end()) return;  // not ours: ignored, like CpuBackend::free (cpu_backend.cpp:96-102)
    use_device(ctx);
    nbl::route_free(ctx, p);
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "free sync");
    cudaFree(p);
    ctx->allocs.erase(it);
  });
}

int nbl_read(nbl_ctx* ctx, float* host_dst, const float* src, int64_t n) {
  return guarded([&] {
    require(ctx && host_dst && src && n >= 0, "read: dst/src NULL or n < 0");
    use_device(ctx);
    nbl::route_touch(ctx, src, n, nbl::Access::kRead);
    nbl::check_cuda(cudaMemcpyAsync(host_dst, src, static_cast<size_t>(n) * sizeof(float), cudaMemcpyDeviceToHost,
                                    ctx->stream),
                    "read");
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "read");
  });
}

int nbl_write(nbl_ctx* ctx, float* dst, const float* host_src, int64_t n) {
  return guarded([&] {
    require(ctx && dst && host_src && n >= 0, "write: dst/src NULL or n < 0");
    use_device(ctx);
    nbl::route_touch(ctx, dst, n, nbl::Access::kWrite);
    nbl::check_cuda(cudaMemcpyAsync(dst, host_src, static_cast<size_t>(n) * sizeof(float), cudaMemcpyHostToDevice,
                                    ctx->stream),
                    "write");
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "write");
  });
}

int nbl_add_bias(nbl_ctx* ctx, float* x, const float* bias, int64_t width, int64_t n) {
  return guarded([&] {
    require(ctx && x && bias && width > 0 && n > 0, "add_bias: x/bias NULL or width/n not positive");
    use_device(ctx);
    if (nbl::route_add_bias(ctx, x, bias, width, n)) return;
    nbl::launch_add_bias(ctx->stream, x, bias, width, n);
  });
}

int nbl_rope(nbl_ctx* ctx, float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0,
             const nbl_rope_params* rope) {
  return guarded([&] {
    require(ctx && x && rope, "rope: ctx/x/params NULL");
    require(n > 0 && n_heads > 0 && head_dim > 0 && head_dim % 2 == 0 && pos0 >= 0,
            "rope: n=" + std::to_string(n) + " n_heads=" + std::to_string(n_heads) + " head_dim=" +
                std::to_string(head_dim) + " (must be even) pos0=" + std::to_string(pos0));
    use_device(ctx);
    const auto& tab = rope_table(ctx, *rope, head_dim, pos0 + n);
    if (nbl::route_rope(ctx, x, n, n_heads, head_dim, pos0, *rope)) return;
    nbl::launch_rope_f32(ctx->stream, x, n, n_heads, head_dim, pos0, rope->neox != 0, tab.dev, ctx->d_err);
  });
}

int nbl_attention(nbl_ctx* ctx, const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                  int64_t n_heads, int64_t n_kv_heads, int64_t head_dim) {
  return guarded([&] {
    require(ctx && q && k && v && out, "attention: NULL pointer");
    require(n > 0 && pos0 >= 0 && n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0 && head_dim > 0 &&
                head_dim <= 256,
            "attention: n=" + std::to_string(n) + " pos0=" + std::to_string(pos0) + " n_heads=" +
                std::to_string(n_heads) + " n_kv_heads=" + std::to_string(n_kv_heads) + " head_dim=" +
                std::to_string(head_dim) + " (n_heads must be a multiple of n_kv_heads; head_dim <= 256)");
    use_device(ctx);
    if (nbl::route_attention(ctx, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim)) return;
    nbl::route_touch(ctx, q, n * n_heads * head_dim, nbl::Access::kRead);
    nbl::route_touch(ctx, k, (pos0 + n) * n_kv_heads * head_dim, nbl::Access::kRead);
    nbl::route_touch(ctx, v, (pos0 + n) * n_kv_heads * head_dim, nbl::Access::kRead);
    nbl::route_touch(ctx, out, n * n_heads * head_dim, nbl::Access::kWrite);
    const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
    nbl::launch_attention_f32(ctx->stream, q, k, v, out, n, pos0, n_heads, n_kv_heads, head_dim, scale, ctx->num_sms);
  });
}

int nbl_kv_create(nbl_ctx* ctx, const nbl_kv_config* cfg, nbl_kv** out) {
  return guarded([&] {
    require(ctx && cfg && out, "kv_create: NULL argument");
    *out = nullptr;
    const nbl_kv_config c = *cfg;
    require(c.n_pages > 0 && c.n_kv_heads > 0 && c.head_dim > 0 && c.page_size > 0,
            "kv_create: n_pages, n_kv_heads, head_dim and page_size must be positive");
    require(c.dtype == NBL_F16 || c.dtype == NBL_BF16, "kv_create: dtype must be NBL_F16 or NBL_BF16");
    if (c.head_dim != 64 || c.page_size != 16)
      nbl::fail(NBL_E_UNSUPPORTED, "kv_create: the paged kernels take head_dim 64 and page_size 16 (got " +
                                       std::to_string(c.head_dim) + ", " + std::to_string(c.page_size) + ")");
    const uint64_t rows = static_cast<uint64_t>(c.n_pages) * 2u * static_cast<uint64_t>(c.n_kv_heads) *
                          static_cast<uint64_t>(c.page_size);
    if (rows >= (1ull << 31))
      nbl::fail(NBL_E_INVALID, "kv_create: pool of " + std::to_string(c.n_pages) +
                                   " pages exceeds 2^31 rows (tensor-map coordinate range)");
    use_device(ctx);
    auto* kv = new nbl_kv();
    kv->ctx = ctx;
    kv->cfg = c;
    kv->bytes = rows * static_cast<uint64_t>(c.head_dim) * 2u;
    try {
      kv->pool = device_alloc(kv->bytes, "kv pool");
      nbl::check_cuda(cudaMemsetAsync(kv->pool, 0, kv->bytes, ctx->stream), "kv pool zero-fill");
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(c.head_dim), rows};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(c.head_dim) * 2u};
      const cuuint32_t box[2] = {static_cast<cuuint32_t>(c.head_dim), static_cast<cuuint32_t>(c.page_size)};
      nbl::encode_tmap(&kv->tmap,
                       c.dtype == NBL_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                       kv->pool, dims, strides, box);
      kv->has_tmap = true;
      nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "kv pool zero-fill");
      ctx->kvs.push_back(kv);
    } catch (...) {
      if (kv->pool) cudaFree(kv->pool);
      delete kv;
      throw;
    }
    *out = kv;
  });
}

int nbl_kv_destroy(nbl_kv* kv) {
  if (!kv) return NBL_OK;
  return guarded([&] {
    nbl_ctx* ctx = kv->ctx;
    use_device(ctx);
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "kv_destroy sync");
    ctx->kvs.erase(std::remove(ctx->kvs.begin(), ctx->kvs.end(), kv), ctx->kvs.end());
    cudaFree(kv->pool);
    delete kv;
  });
}

int nbl_kv_pool(const nbl_kv* kv, void** base, int64_t* bytes) {
  return guarded([&] {
    require(kv && base && bytes, "kv_pool: NULL argument");
    *base = kv->pool;
    *bytes = static_cast<int64_t>(kv->bytes);
  });
}

int nbl_rope_kv_append(nbl_ctx* ctx, nbl_kv* kv, const void* q_in, const void* k_in, const void* v_in,
                       int32_t in_dtype, const float* bq, const float* bk, const float* bv, void* q_out,
                       int32_t q_out_dtype, const int32_t* tok_row, const int32_t* tok_pos, const int32_t* page_table,
                       int32_t pt_stride, int64_t n_tok, int32_t n_heads, const nbl_rope_params* rope) {
  return guarded([&] {
    require(ctx && kv && q_in && k_in && v_in && q_out && tok_row && tok_pos && page_table && rope,
            "rope_kv_append: NULL argument");
    nbl::route_flush_queries(ctx);
    require(kv->ctx == ctx, "rope_kv_append: pool belongs to another context");
    require(is_dtype(in_dtype) && is_dtype(q_out_dtype), "rope_kv_append: bad dtype");
    require(n_tok >= 0 && n_tok <= INT32_MAX && pt_stride > 0, "rope_kv_append: n_tok or pt_stride out of range");
    require(n_heads > 0 && n_heads % kv->cfg.n_kv_heads == 0, "rope_kv_append: n_heads must be a multiple of n_kv_heads");
    if (n_tok == 0) return;
    use_device(ctx);
    const int64_t max_pos = int64_t(pt_stride) * kv->cfg.page_size;
    const auto& tab = rope_table(ctx, *rope, kv->cfg.head_dim, max_pos);
    nbl::launch_rope_kv_append(ctx->stream, kv, q_in, k_in, v_in, in_dtype, bq, bk, bv, q_out, q_out_dtype, tok_row,
                               tok_pos, page_table, pt_stride, n_tok, n_heads, rope->neox != 0, tab.dev, tab.n_pos,
                               ctx->d_err);
  });
}

int nbl_attn_decode(nbl_ctx* ctx, const nbl_kv* kv, const float* q, const int32_t* page_table, int32_t pt_stride,
                    const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows, int32_t n_heads, float* out,
                    float* lse, int32_t n_splits) {
  return guarded([&] {
    require(ctx && kv && q && page_table && seq_lens && out, "attn_decode: NULL argument");
    nbl::route_flush_queries(ctx);
    require(kv->ctx == ctx, "attn_decode: pool belongs to another context");
    require(kv->cfg.dtype == NBL_F16, "attn_decode: the decode kernel reads an NBL_F16 pool");
    require(n_rows >= 0 && pt_stride > 0 && max_seq_len >= 0 && n_splits >= 0, "attn_decode: negative size");
    require(n_heads > 0 && n_heads % kv->cfg.n_kv_heads == 0 && n_heads / kv->cfg.n_kv_heads <= 8,
            "attn_decode: n_heads must be a multiple of n_kv_heads with at most 8 query heads per KV head");
    require(int64_t(max_seq_len) <= int64_t(pt_stride) * kv->cfg.page_size,
            "attn_decode: max_seq_len exceeds pt_stride * page_size");
    if (n_rows == 0) return;
    use_device(ctx);
    const auto plan = nbl::plan_decode(n_rows, kv->cfg.n_kv_heads, n_heads / kv->cfg.n_kv_heads, n_heads,
                                       max_seq_len, kv->cfg.page_size, ctx->num_sms, n_splits);
    unsigned* counts = nullptr;
    if (plan.scratch_bytes) {
      ensure_scratch(ctx, plan.scratch_bytes);
      counts = nbl::split_counts(ctx, int64_t(n_rows) * kv->cfg.n_kv_heads);
    }
    nbl::launch_decode(ctx->stream, kv, q, page_table, pt_stride, seq_lens, n_rows, n_heads, out, lse, plan,
                       ctx->scratch, ctx->d_err, counts);
  });
}

int nbl_decode_step_host(nbl_ctx* ctx, nbl_kv* kv, const float* q_in_h, const float* k_in_h, const float* v_in_h,
                         const float* bq, const float* bk, const float* bv, const int32_t* page_table,
                         int32_t pt_stride, const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows,
                         int32_t n_heads, const nbl_rope_params* rope, float* out_h, int32_t n_chunks) {
  return guarded([&] {
    require(ctx && kv && q_in_h && k_in_h && v_in_h && page_table && seq_lens && rope && out_h,
            "decode_step_host: NULL argument");
    nbl::route_flush_queries(ctx);
    require(kv->ctx == ctx, "decode_step_host: pool belongs to another context");
    require(kv->cfg.dtype == NBL_F16, "decode_step_host: the decode kernel reads an NBL_F16 pool");
    require(n_rows >= 0 && pt_stride > 0 && max_seq_len >= 1 && n_chunks >= 0,
            "decode_step_host: negative size, max_seq_len < 1 or pt_stride not positive");
    const int kvh = kv->cfg.n_kv_heads;
    require(n_heads > 0 && n_heads % kvh == 0 && n_heads / kvh <= 8,
            "decode_step_host: n_heads must be a multiple of n_kv_heads with at most 8 query heads per KV head");
    require(int64_t(max_seq_len) <= int64_t(pt_stride) * kv->cfg.page_size,
            "decode_step_host: max_seq_len exceeds pt_stride * page_size");
    if (n_rows == 0) return;
    use_device(ctx);
    const int64_t d = kv->cfg.head_dim;
    const int64_t q_row = int64_t(n_heads) * d, kv_row = int64_t(kvh) * d;  // floats per row
    const size_t need = static_cast<size_t>(n_rows) * static_cast<size_t>(3 * q_row + 2 * kv_row) * sizeof(float);
    if (ctx->io_bytes < need) {
      void* p = device_alloc(need, "decode_step_host staging");
      if (ctx->io) {
        nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "staging sync");
        cudaFree(ctx->io);
      }
      ctx->io = p;
      ctx->io_bytes = need;
    }
    float* q_in = static_cast<float*>(ctx->io);
    float* k_in = q_in + int64_t(n_rows) * q_row;
    float* v_in = k_in + int64_t(n_rows) * kv_row;
    float* q = v_in + int64_t(n_rows) * kv_row;
    float* out = q + int64_t(n_rows) * q_row;
    const auto& tab = rope_table(ctx, *rope, d, int64_t(pt_stride) * kv->cfg.page_size);
    // Chunks: each keeps at least two waves of decode CTAs (2 per SM), at most 4.
    int chunks = n_chunks;
    if (chunks == 0) chunks = static_cast<int>(std::min<int64_t>(4, std::max<int64_t>(1, int64_t(n_rows) * kvh / (4 * ctx->num_sms))));
    chunks = std::min(chunks, n_rows);
    if (!ctx->up_stream) {
      nbl::check_cuda(cudaStreamCreateWithFlags(&ctx->up_stream, cudaStreamNonBlocking), "copy stream");
      nbl::check_cuda(cudaStreamCreateWithFlags(&ctx->down_stream, cudaStreamNonBlocking), "copy stream");
      nbl::check_cuda(cudaStreamCreateWithFlags(&ctx->aux_stream, cudaStreamNonBlocking), "compute stream");
    }
    while (ctx->events.size() < size_t(2 * chunks + 1)) {
      cudaEvent_t e;
      nbl::check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
      ctx->events.push_back(e);
    }
    cudaEvent_t* ev_in = ctx->events.data() + 1;
    cudaEvent_t* ev_out = ev_in + chunks;
    std::vector<nbl::DecodePlan> plans(chunks);
    size_t scratch = 0;
    auto bounds = [&](int c) { return std::make_pair(int64_t(c) * n_rows / chunks, int64_t(c + 1) * n_rows / chunks); };
    for (int c = 0; c < chunks; ++c) {
      const auto [r0, r1] = bounds(c);
      plans[c] = nbl::plan_decode(static_cast<int>(r1 - r0), kvh, n_heads / kvh, n_heads, max_seq_len,
                                  kv->cfg.page_size, ctx->num_sms, 0);
      scratch = std::max(scratch, plans[c].scratch_bytes);
    }
    unsigned* counts = nullptr;
    if (scratch) {
      ensure_scratch(ctx, scratch);
      counts = nbl::split_counts(ctx, (n_rows + chunks - 1) / chunks * int64_t(kvh) + kvh);
    }
    // Chunks touch disjoint rows and pages, so without split partials (which share the context scratch) odd
    // chunks run on a second compute stream: one chunk's last wave overlaps the next chunk's first.
    const bool two = scratch == 0 && chunks > 1;
    // staging is free once earlier work on the compute stream is done
    nbl::check_cuda(cudaEventRecord(ctx->events[0], ctx->stream), "cudaEventRecord");
    nbl::check_cuda(cudaStreamWaitEvent(ctx->up_stream, ctx->events[0], 0), "cudaStreamWaitEvent");
    for (int c = 0; c < chunks; ++c) {
      const auto [r0, r1] = bounds(c);
      const int64_t nr = r1 - r0;
      nbl::check_cuda(cudaMemcpyAsync(q_in + r0 * q_row, q_in_h + r0 * q_row, nr * q_row * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->up_stream), "q upload");
      nbl::check_cuda(cudaMemcpyAsync(k_in + r0 * kv_row, k_in_h + r0 * kv_row, nr * kv_row * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->up_stream), "k upload");
      nbl::check_cuda(cudaMemcpyAsync(v_in + r0 * kv_row, v_in_h + r0 * kv_row, nr * kv_row * sizeof(float),
                                      cudaMemcpyHostToDevice, ctx->up_stream), "v upload");
      nbl::check_cuda(cudaEventRecord(ev_in[c], ctx->up_stream), "cudaEventRecord");
    }
    for (int c = 0; c < chunks; ++c) {
      const auto [r0, r1] = bounds(c);
      const int64_t nr = r1 - r0;
      cudaStream_t cs = two && (c & 1) ? ctx->aux_stream : ctx->stream;
      nbl::check_cuda(cudaStreamWaitEvent(cs, ev_in[c], 0), "cudaStreamWaitEvent");
      nbl::launch_rope_kv_append(cs, kv, q_in + r0 * q_row, k_in + r0 * kv_row, v_in + r0 * kv_row, NBL_F32,
                                 bq, bk, bv, q + r0 * q_row, NBL_F32, nullptr, nullptr, page_table, pt_stride, nr,
                                 n_heads, rope->neox != 0, tab.dev, tab.n_pos, ctx->d_err, static_cast<int32_t>(r0),
                                 seq_lens);
      nbl::launch_decode(cs, kv, q + r0 * q_row, page_table + r0 * pt_stride, pt_stride, seq_lens + r0,
                         static_cast<int>(nr), n_heads, out + r0 * q_row, nullptr, plans[c], ctx->scratch, ctx->d_err,
                         counts);
      nbl::check_cuda(cudaEventRecord(ev_out[c], cs), "cudaEventRecord");
      nbl::check_cuda(cudaStreamWaitEvent(ctx->down_stream, ev_out[c], 0), "cudaStreamWaitEvent");
      nbl::check_cuda(cudaMemcpyAsync(out_h + r0 * q_row, out + r0 * q_row, nr * q_row * sizeof(float),
                                      cudaMemcpyDeviceToHost, ctx->down_stream), "out download");
    }
    nbl::check_cuda(cudaStreamSynchronize(ctx->down_stream), "decode_step_host");
  });
}

int nbl_attn_prefill(nbl_ctx* ctx, const nbl_kv* kv, const void* q, int32_t q_dtype, int64_t n_q_rows,
                     const int32_t* q_start, const int32_t* q_len, const int32_t* kv_pos0, const int32_t* page_table,
                     int32_t pt_stride, int32_t n_items, int32_t n_heads, int32_t max_q_len, void* out,
                     int32_t out_dtype) {
  return guarded([&] {
    require(ctx && kv && q && q_start && q_len && kv_pos0 && page_table && out, "attn_prefill: NULL argument");
    nbl::route_flush_queries(ctx);
    require(kv->ctx == ctx, "attn_prefill: pool belongs to another context");
    require(q_dtype == kv->cfg.dtype, "attn_prefill: q must have the pool's dtype");
    require(out_dtype == NBL_F32 || out_dtype == kv->cfg.dtype, "attn_prefill: out must be F32 or the pool dtype");
    require(n_items >= 0 && pt_stride > 0 && max_q_len >= 0 && n_q_rows >= 0, "attn_prefill: negative size");
    require(kv->cfg.head_dim == 64, "attn_prefill: head_dim 64 only");
    require(n_heads > 0 && n_heads % kv->cfg.n_kv_heads == 0, "attn_prefill: n_heads must be a multiple of n_kv_heads");
    if (n_items == 0 || max_q_len == 0) return;
    use_device(ctx);
    if (n_q_rows == 0) return;
    nbl::launch_prefill(ctx->stream, kv, q, n_q_rows, q_start, q_len, kv_pos0, page_table, pt_stride, n_items,
                        n_heads, max_q_len, out, out_dtype, ctx->d_err);
  });
}

int nbl_lse_merge(nbl_ctx* ctx, const float* part_o, const float* part_lse, int32_t n_parts, int64_t rows,
                  int32_t head_dim, float* out, float* lse) {
  return guarded([&] {
    require(ctx && part_o && part_lse && out, "lse_merge: NULL argument");
    nbl::route_flush_queries(ctx);
    require(n_parts > 0 && rows >= 0 && head_dim > 0 && head_dim <= 256, "lse_merge: bad size");
    if (rows == 0) return;
    use_device(ctx);
    nbl::launch_lse_merge(ctx->stream, part_o, part_lse, n_parts, rows, head_dim, out, lse);
  });
}

int nbl_lse_merge_packed(nbl_ctx* ctx, const float* packed, int32_t n_parts, int64_t rows, int32_t head_dim,
                         float* out, float* lse) {
  return guarded([&] {
    require(ctx && packed && out, "lse_merge_packed: NULL argument");
    nbl::route_flush_queries(ctx);
    require(n_parts > 0 && rows >= 0 && head_dim > 0 && head_dim <= 256, "lse_merge_packed: bad size");
    if (rows == 0) return;
    use_device(ctx);
    const int64_t part = rows * (int64_t(head_dim) + 1);  // [rows * head_dim outputs | rows lse] per part
    nbl::launch_lse_merge(ctx->stream, packed, packed + rows * head_dim, n_parts, rows, head_dim, out, lse, part,
                          part);
  });
}

int nbl_lse_exchange_peers(nbl_ctx* ctx, const float* send, int64_t rows, int32_t head_dim, int32_t world,
                           int32_t rank, void* const* recv_bufs, void* const* flag_bufs, uint32_t* sync, float* out,
                           float* lse) {
  return guarded([&] {
    require(ctx && send && recv_bufs && flag_bufs && sync && out, "lse_exchange_peers: NULL argument");
    require(world >= 1 && world <= nbl::kMaxPeers && rank >= 0 && rank < world,
            "lse_exchange_peers: world must be 1.." + std::to_string(nbl::kMaxPeers) + " and rank in [0, world)");
    require(rows >= 0 && head_dim > 0 && head_dim <= 256, "lse_exchange_peers: bad size");
    float* recv[nbl::kMaxPeers];
    uint32_t* flags[nbl::kMaxPeers];
    for (int p = 0; p < world; ++p) {
      require(recv_bufs[p] && flag_bufs[p], "lse_exchange_peers: NULL peer buffer");
      recv[p] = static_cast<float*>(recv_bufs[p]);
      flags[p] = static_cast<uint32_t*>(flag_bufs[p]);
    }
    if (rows == 0) return;
    use_device(ctx);
    nbl::route_flush_queries(ctx);
    nbl::launch_lse_exchange_peers(ctx->stream, send, rows, head_dim, world, rank, recv, flags, sync, out, lse,
                                   ctx->d_err, ctx->num_sms);
  });
}

int nbl_attn_decode_peers(nbl_ctx* ctx, const nbl_kv* kv, const float* q, const int32_t* page_table,
                          int32_t pt_stride, const int32_t* seq_lens, int32_t max_seq_len, int32_t n_rows,
                          int32_t n_heads, int32_t world, int32_t rank, void* const* recv_bufs,
                          void* const* flag_bufs, uint32_t* sync, float* out, float* lse) {
  return guarded([&] {
    require(ctx && kv && q && page_table && seq_lens && recv_bufs && flag_bufs && sync && out,
            "attn_decode_peers: NULL argument");
    require(kv->ctx == ctx, "attn_decode_peers: pool belongs to another context");
    require(kv->cfg.dtype == NBL_F16 && kv->cfg.head_dim == 64 && kv->cfg.page_size == 16,
            "attn_decode_peers: the decode kernel reads an NBL_F16 pool of head_dim 64, 16-token pages");
    require(world >= 1 && world <= nbl::kMaxPeers && rank >= 0 && rank < world,
            "attn_decode_peers: world must be 1.." + std::to_string(nbl::kMaxPeers) + " and rank in [0, world)");
    require(n_rows >= 0 && pt_stride > 0 && max_seq_len >= 0, "attn_decode_peers: negative size");
    require(n_heads > 0 && n_heads % kv->cfg.n_kv_heads == 0 && n_heads / kv->cfg.n_kv_heads <= 8,
            "attn_decode_peers: n_heads must be a multiple of n_kv_heads with at most 8 query heads per KV head");
    require(int64_t(max_seq_len) <= int64_t(pt_stride) * kv->cfg.page_size,
            "attn_decode_peers: max_seq_len exceeds pt_stride * page_size");
    float* recv[nbl::kMaxPeers];
    uint32_t* flags[nbl::kMaxPeers];
    for (int p = 0; p < world; ++p) {
      require(recv_bufs[p] && flag_bufs[p], "attn_decode_peers: NULL peer buffer");
      recv[p] = static_cast<float*>(recv_bufs[p]);
      flags[p] = static_cast<uint32_t*>(flag_bufs[p]);
    }
    if (n_rows == 0) return;
    use_device(ctx);
    nbl::route_flush_queries(ctx);
    const auto plan = nbl::plan_decode(n_rows, kv->cfg.n_kv_heads, n_heads / kv->cfg.n_kv_heads, n_heads,
                                       max_seq_len, kv->cfg.page_size, ctx->num_sms, 0);
    unsigned* counts = nullptr;
    if (plan.scratch_bytes) {
      ensure_scratch(ctx, plan.scratch_bytes);
      counts = nbl::split_counts(ctx, int64_t(n_rows) * kv->cfg.n_kv_heads);
    }
    nbl::launch_decode_peers(ctx->stream, kv, q, page_table, pt_stride, seq_lens, n_rows, n_heads, plan,
                             ctx->scratch, counts, world, rank, recv, flags, sync, out, lse, ctx->d_err,
                             ctx->num_sms);
  });
}

// ---- weights and the model's other ops ----

int nbl_weight_create(nbl_ctx* ctx, const void* host, int32_t dtype, int64_t ne0, int64_t ne1, nbl_weight** out) {
  return guarded([&] {
    require(ctx && host && out, "weight_create: ctx, host or out is NULL");
    *out = nullptr;
    require(dtype == NBL_F32 || dtype == NBL_F16 || nbl::is_quant(dtype) || nbl::is_qblock(dtype),
            "weight_create: dtype must be NBL_F32, NBL_F16 or a quantized type (Q4_0, Q5_0, Q8_0, Q5_1, Q4_K, Q5_K, "
            "Q6_K)");
    require(ne0 > 0 && ne1 > 0, "weight_create: bad shape " + std::to_string(ne0) + " x " + std::to_string(ne1));
    require(!nbl::is_quant(dtype) || ne0 % 32 == 0, "weight_create: a quantized row must be whole 32-element blocks");
    require(!nbl::is_qblock(dtype) || ne0 % nbl::qblock_elems(dtype) == 0,
            "weight_create: a quantized row must be whole " + std::to_string(nbl::qblock_elems(dtype)) +
                "-element blocks");
    const size_t elem = dtype == NBL_F32 ? 4 : 2;
    require(static_cast<uint64_t>(ne0) <= (uint64_t(1) << 40) / static_cast<uint64_t>(ne1),
            "weight_create: tensor too large");
    const size_t count = static_cast<size_t>(ne0) * static_cast<size_t>(ne1);
    use_device(ctx);
    auto* w = new nbl_weight();
    w->ctx = ctx;
    w->w.dtype = dtype;
    w->w.ne0 = ne0;
    w->w.ne1 = ne1;
    try {
      if (nbl::is_quant(dtype)) {
        // GGUF blocks -> [scales][values][high bits], each array 256-byte aligned, split on the host
        const size_t nbk = count / 32, bb = static_cast<size_t>(nbl::quant_block_bytes(dtype));
        const size_t qsb = static_cast<size_t>(nbl::quant_qs_bytes(dtype));
        const size_t off_qs = (nbk * 2 + 255) & ~size_t(255);
        const size_t off_qh = (off_qs + nbk * qsb + 255) & ~size_t(255);
        const size_t total = off_qh + (dtype == NBL_Q5_0 ? nbk * 4 : 0);
        std::vector<uint8_t> packed(total);
        const auto* src = static_cast<const uint8_t*>(host);
        for (size_t b = 0; b < nbk; ++b) {
          const uint8_t* blk = src + b * bb;
          std::memcpy(packed.data() + b * 2, blk, 2);  // fp16 scale
          if (dtype == NBL_Q5_0) {
            std::memcpy(packed.data() + off_qh + b * 4, blk + 2, 4);  // high bits
            std::memcpy(packed.data() + off_qs + b * qsb, blk + 6, qsb);
          } else {
            std::memcpy(packed.data() + off_qs + b * qsb, blk + 2, qsb);
          }
        }
        w->w.dev = device_alloc(total, "weight");
        nbl::check_cuda(cudaMemcpyAsync(w->w.dev, packed.data(), total, cudaMemcpyHostToDevice, ctx->stream),
                        "weight upload");
        nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "weight upload");  // `packed` is released below
        auto* base = static_cast<uint8_t*>(w->w.dev);
        w->w.q.d = reinterpret_cast<const uint16_t*>(base);
        w->w.q.qs = base + off_qs;
        w->w.q.qh = dtype == NBL_Q5_0 ? reinterpret_cast<const uint32_t*>(base + off_qh) : nullptr;
      } else if (nbl::is_qblock(dtype)) {
        // GGUF blocks as they are, row after row
        const size_t bytes = static_cast<size_t>(ne1) * static_cast<size_t>(ne0 / nbl::qblock_elems(dtype)) *
                             static_cast<size_t>(nbl::qblock_bytes(dtype));
        w->w.dev = device_alloc(bytes, "weight");
        nbl::check_cuda(cudaMemcpyAsync(w->w.dev, host, bytes, cudaMemcpyHostToDevice, ctx->stream), "weight upload");
      } else {
        w->w.dev = device_alloc(count * elem, "weight");
        nbl::check_cuda(cudaMemcpyAsync(w->w.dev, host, count * elem, cudaMemcpyHostToDevice, ctx->stream),
                        "weight upload");
      }
      nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "weight upload");
      ctx->weights.push_back(w);
    } catch (...) {
      release_weight(w);
      throw;
    }
    *out = w;
  });
}

int nbl_weight_destroy(nbl_weight* w) {
  if (!w) return NBL_OK;
  return guarded([&] {
    nbl_ctx* ctx = w->ctx;
    use_device(ctx);
    nbl::check_cuda(cudaStreamSynchronize(ctx->stream), "weight destroy sync");
    ctx->weights.erase(std::remove(ctx->weights.begin(), ctx->weights.end(), w), ctx->weights.end());
    release_weight(w);
  });
}

int nbl_weight_data(const nbl_weight* w, const void** dev, int32_t* dtype, int64_t* ne0, int64_t* ne1) {
  return guarded([&] {
    require(w != nullptr, "weight_data: weight is NULL");
    if (dev) *dev = w->w.dev;
    if (dtype) *dtype = w->w.dtype;
    if (ne0) *ne0 = w->w.ne0;
    if (ne1) *ne1 = w->w.ne1;
  });
}

int nbl_embed(nbl_ctx* ctx, const nbl_weight* table, const int32_t* ids, int64_t n, float* out) {
  return guarded([&] {
    require(ctx && ids && out, "embed: ctx, ids or out is NULL");
    require_weight(ctx, table, "embed");
    require(n >= 0, "embed: n < 0");
    for (int64_t t = 0; t < n; ++t)  // the reference's check and message (ref_ops.cpp:84-87)
      if (ids[t] < 0 || ids[t] >= table->w.ne1)
        nbl::fail(NBL_E_INVALID, "embed: token id " + std::to_string(ids[t]) + " out of range (n_vocab " +
                                     std::to_string(table->w.ne1) + ")");
    if (n == 0) return;
    use_device(ctx);
    nbl::route_touch(ctx, out, n * table->w.ne0, nbl::Access::kWrite);
    ensure_ids(ctx, n);
    nbl::check_cuda(cudaMemcpyAsync(ctx->ids, ids, static_cast<size_t>(n) * sizeof(int32_t), cudaMemcpyHostToDevice,
                                    ctx->stream),
                    "embed ids");
    if (nbl::is_quant(table->w.dtype)) nbl::launch_embed_q(ctx->stream, table->w, ctx->ids, n, out);
    else if (nbl::is_qblock(table->w.dtype))
      nbl::launch_embed_qblock(ctx->stream, table->w, ctx->ids, n, out, ctx->num_sms);
    else nbl::launch_embed(ctx->stream, table->w, ctx->ids, n, out, ctx->num_sms);
    nbl::check_cuda(cudaGetLastError(), "embed launch");
  });
}

int nbl_matmul(nbl_ctx* ctx, const nbl_weight* w, const float* x, float* y, int64_t n) {
  return guarded([&] {
    require(ctx && x && y, "matmul: ctx, x or y is NULL");
    require_weight(ctx, w, "matmul");
    require(n >= 0 && n <= INT32_MAX && w->w.ne0 <= INT32_MAX && w->w.ne1 <= INT32_MAX, "matmul: bad size");
    if (n == 0) return;
    use_device(ctx);
    nbl::route_touch(ctx, x, n * w->w.ne0, nbl::Access::kRead);
    y = nbl::route_output(ctx, y, n, w->w.ne1);
    if (nbl::is_quant(w->w.dtype)) {
      quant_matmul(ctx, &w, &y, 1, x, n);
      nbl::check_cuda(cudaGetLastError(), "matmul launch");
    } else if (nbl::is_qblock(w->w.dtype)) {
      qblock_matmul(ctx, w, y, x, n);
      nbl::check_cuda(cudaGetLastError(), "matmul launch");
    } else if (n <= nbl::kGemvMaxRows) {
      nbl::launch_gemv(ctx->stream, w->w, x, y, n, ctx->num_sms);
      nbl::check_cuda(cudaGetLastError(), "matmul launch");
    } else {
      float_gemm(ctx, &w, &y, 1, x, n);
    }
  });
}

int nbl_matmul_multi(nbl_ctx* ctx, const nbl_weight* const* ws, int32_t count, const float* x, float* const* ys,
                     int64_t n) {
  return guarded([&] {
    require(ctx && ws && ys && x, "matmul_multi: NULL argument");
    require(count > 0, "matmul_multi: count must be positive");
    require(n >= 0 && n <= INT32_MAX, "matmul_multi: bad n");
    for (int32_t i = 0; i < count; ++i) {
      require_weight(ctx, ws[i], "matmul_multi");
      require(ys[i] != nullptr, "matmul_multi: output is NULL");
      require(ws[i]->w.ne0 == ws[0]->w.ne0, "matmul_multi: weights differ in input width");
      require(ws[i]->w.ne1 <= INT32_MAX, "matmul_multi: bad size");
    }
    if (n == 0) return;
    use_device(ctx);
    if (nbl::route_matmul_multi(ctx, ws, count, x, ys, n)) return;
    nbl::route_touch(ctx, x, n * ws[0]->w.ne0, nbl::Access::kRead);
    std::vector<float*> outs(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; ++i) outs[i] = nbl::route_output(ctx, ys[i], n, ws[i]->w.ne1);
    ys = outs.data();
    bool any_quant = false, all_quant_same = true;
    for (int32_t i = 0; i < count; ++i) {
      any_quant = any_quant || nbl::is_quant(ws[i]->w.dtype) || nbl::is_qblock(ws[i]->w.dtype);
      all_quant_same = all_quant_same && ws[i]->w.dtype == ws[0]->w.dtype && nbl::is_quant(ws[i]->w.dtype);
    }
    if (any_quant) {
      if (all_quant_same) {
        for (int32_t i0 = 0; i0 < count; i0 += nbl::kMaxMulti)
          quant_matmul(ctx, ws + i0, ys + i0, static_cast<int>(std::min<int32_t>(nbl::kMaxMulti, count - i0)), x,
                       n);
      } else {
        for (int32_t i = 0; i < count; ++i) {
          if (nbl::is_quant(ws[i]->w.dtype)) {
            quant_matmul(ctx, ws + i, ys + i, 1, x, n);
          } else if (nbl::is_qblock(ws[i]->w.dtype)) {
            qblock_matmul(ctx, ws[i], ys[i], x, n);
          } else if (n <= nbl::kGemvMaxRows) {
            nbl::launch_gemv(ctx->stream, ws[i]->w, x, ys[i], n, ctx->num_sms);
          } else {
            float_gemm(ctx, ws + i, ys + i, 1, x, n);
          }
        }
      }
      nbl::check_cuda(cudaGetLastError(), "matmul launch");
    } else if (n <= nbl::kGemvMaxRows) {
      for (int32_t i0 = 0; i0 < count; i0 += nbl::kMaxMulti) {
        const int c = static_cast<int>(std::min<int32_t>(nbl::kMaxMulti, count - i0));
        const nbl::Weight* w[nbl::kMaxMulti];
        float* y[nbl::kMaxMulti];
        for (int i = 0; i < c; ++i) {
          w[i] = &ws[i0 + i]->w;
          y[i] = ys[i0 + i];
        }
        nbl::launch_gemv_multi(ctx->stream, w, y, c, x, n, ctx->num_sms);
      }
      nbl::check_cuda(cudaGetLastError(), "matmul launch");
    } else {
      float_gemm(ctx, ws, ys, count, x, n);
    }
  });
}

int nbl_rmsnorm(nbl_ctx* ctx, const float* x, const nbl_weight* weight, float* y, int64_t n, float eps) {
  return guarded([&] {
    require(ctx && x && y, "rmsnorm: ctx, x or y is NULL");
    require_weight(ctx, weight, "rmsnorm");
    require(weight->w.dtype == NBL_F32 && weight->w.ne1 == 1, "rmsnorm: weight must be an F32 vector");
    require(n >= 0 && n <= INT32_MAX, "rmsnorm: bad n");
    if (n == 0) return;
    use_device(ctx);
    nbl::route_touch(ctx, x, n * weight->w.ne0, nbl::Access::kRead);
    nbl::route_touch(ctx, y, n * weight->w.ne0, nbl::Access::kWrite);
    nbl::launch_rmsnorm(ctx->stream, x, static_cast<const float*>(weight->w.dev), y, n, weight->w.ne0, eps);
    nbl::check_cuda(cudaGetLastError(), "rmsnorm launch");
  });
}

int nbl_add(nbl_ctx* ctx, float* x, const float* y, int64_t count) {
  return guarded([&] {
    require(ctx && x && y && count >= 0, "add: NULL argument or count < 0");
    if (count == 0) return;
    use_device(ctx);
    nbl::route_touch(ctx, x, count, nbl::Access::kReadWrite);
    nbl::route_touch(ctx, y, count, nbl::Access::kRead);
    nbl::launch_add(ctx->stream, x, y, count, ctx->num_sms);
    nbl::check_cuda(cudaGetLastError(), "add launch");
  });
}

int nbl_copy(nbl_ctx* ctx, float* dst, const float* src, int64_t count) {
  return guarded([&] {
    require(ctx && dst && src && count >= 0, "copy: NULL argument or count < 0");
    if (count == 0 || dst == src) return;
    use_device(ctx);
    nbl::route_touch(ctx, src, count, nbl::Access::kRead);
    nbl::route_touch(ctx, dst, count, nbl::Access::kWrite);
    nbl::check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(count) * sizeof(float), cudaMemcpyDeviceToDevice,
                                    ctx->stream),
                    "copy");
  });
}

int nbl_silu_mul(nbl_ctx* ctx, float* gate, const float* up, int64_t count) {
  return guarded([&] {
    require(ctx && gate && up && count >= 0, "silu_mul: NULL argument or count < 0");
    if (count == 0) return;
    use_device(ctx);
    nbl::route_touch(ctx, gate, count, nbl::Access::kReadWrite);
    nbl::route_touch(ctx, up, count, nbl::Access::kRead);
    nbl::launch_silu_mul(ctx->stream, gate, up, count, ctx->num_sms);
    nbl::check_cuda(cudaGetLastError(), "silu_mul launch");
  });
}

}  // extern "C"
