// nbl_attn_decode_static: the split-K decode of nbl_attn_decode with its split partials kept in a fixed,
// library-owned device array instead of context scratch, so the call never allocates device memory.
//
// Who needs it: callers that must not allocate device memory once they are running -- an engine that reserves
// all of a GPU's memory for its own pool at start-up and treats any later cudaMalloc as a failure, or a
// latency-critical decode loop that cannot afford cudaMalloc's implicit device-wide synchronisation. The
// ordinary entry point grows the context's scratch on demand (or needs nbl_reserve beforehand); this one uses
// a static array of fixed size.
//
// Limits and sharing:
//   * the array holds kStaticScratchBytes (8 MiB) on every GPU the library has created a context on, until the
//     process exits; a request whose split partials need more is rejected (NBL_E_INVALID) when the caller asked
//     for an explicit split count, and served with fewer splits (down to one split, which needs no scratch) when
//     the split count is left to the library;
//   * every call on a device shares the one array and it keeps the last call's contents; the decode kernel
//     writes every partial it later merges, so nothing has to start at zero. The splits' arrival counters (one
//     per (row, KV head), kStaticCounts of them) live in a second static array, zeroed at set-up and left at
//     zero by every launch; calls with more (row, KV head) pairs merge with a second kernel instead. Two calls
//     whose kernels overlap on the GPU (different streams, or different contexts on the same device) race on
//     the arrays: serialise them;
//   * set-up happens in nbl_ctx_create, once per device, with that device current: the module holding the array
//     is loaded (which is when CUDA places the array in device memory), its address is resolved with
//     cudaGetSymbolAddress and cached, and the decode kernels are loaded too. So the entry point's own calls,
//     the first one included, allocate nothing.
// No reference counterpart: nibble's CPU backend sizes its scratch once in reserve() (cpu_backend.cpp:24-67).
#include <mutex>
#include <new>
#include <string>

#include "nbl_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];
// 8 MiB of partials hold at most 8 MiB / (2 splits x 65 floats x 4 bytes) = 16131 (row, head) pairs, so with
// splits every (row, KV head) pair of a call that fits has a counter.
constexpr int kStaticCounts = 16384;
static __device__ unsigned g_decode_counts[kStaticCounts];

// Per-device device address of g_decode_scratch. In host code the symbol itself is only a host-side stand-in,
// never a device address, so kernels are given these resolved addresses.
std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};
unsigned* g_counts_addr[kMaxDevices] = {};

void* resolved_scratch(int device) {
  if (device < 0 || device >= kMaxDevices) nbl::fail(NBL_E_UNSUPPORTED, "attn_decode_static: device id >= 64");
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[device])
    nbl::fail(NBL_E_CUDA, "attn_decode_static: the static partials array was not set up on device " +
                              std::to_string(device) + " (nbl_ctx_create does it)");
  return g_addr[device];
}

}  // namespace

void nbl::prepare_static_decode(int device) {
  if (device < 0 || device >= kMaxDevices) return;  // such a device can only be refused by the entry point
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (g_addr[device]) return;
  void* p = nullptr;
  void* pc = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);  // the caller made `device` current
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&pc, g_decode_counts);
  if (e == cudaSuccess) e = cudaMemset(pc, 0, sizeof(g_decode_counts));
  if (e != cudaSuccess || !p || !pc) {
    cudaGetLastError();  // leave no stale error for a later launch check to report
    nbl::fail(NBL_E_CUDA, std::string("cannot set up the static decode partials array: ") + cudaGetErrorString(e));
  }
  nbl::preload_decode();
  g_addr[device] = p;
  g_counts_addr[device] = static_cast<unsigned*>(pc);
}

extern "C" NBL_API int nbl_attn_decode_static(nbl_ctx* ctx, const nbl_kv* kv, const float* q,
                                              const int32_t* page_table, int32_t pt_stride, const int32_t* seq_lens,
                                              int32_t max_seq_len, int32_t n_rows, int32_t n_heads, float* out,
                                              float* lse, int32_t n_splits) {
  try {
    auto require = [](bool ok, const char* msg) {
      if (!ok) nbl::fail(NBL_E_INVALID, msg);
    };
    require(ctx && kv && q && page_table && seq_lens && out, "attn_decode_static: NULL argument");
    require(kv->ctx == ctx, "attn_decode_static: pool belongs to another context");
    require(kv->cfg.dtype == NBL_F16, "attn_decode_static: the decode kernel reads an NBL_F16 pool");
    require(n_rows >= 0 && pt_stride > 0 && max_seq_len >= 0 && n_splits >= 0, "attn_decode_static: negative size");
    require(n_heads > 0 && n_heads % kv->cfg.n_kv_heads == 0 && n_heads / kv->cfg.n_kv_heads <= 8,
            "attn_decode_static: n_heads must be a multiple of n_kv_heads with at most 8 query heads per KV head");
    require(int64_t(max_seq_len) <= int64_t(pt_stride) * kv->cfg.page_size,
            "attn_decode_static: max_seq_len exceeds pt_stride * page_size");
    if (n_rows == 0) return NBL_OK;
    nbl::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int group = n_heads / kv->cfg.n_kv_heads;
    nbl::DecodePlan plan = nbl::plan_decode(n_rows, kv->cfg.n_kv_heads, group, n_heads, max_seq_len,
                                            kv->cfg.page_size, ctx->num_sms, n_splits);
    if (plan.scratch_bytes > kStaticScratchBytes) {
      if (n_splits > 0)
        nbl::fail(NBL_E_INVALID, "attn_decode_static: " + std::to_string(plan.n_splits) + " splits x " +
                                     std::to_string(n_rows) + " rows x " + std::to_string(n_heads) + " heads need " +
                                     std::to_string(plan.scratch_bytes) + " bytes of split partials; the static "
                                     "array holds " + std::to_string(kStaticScratchBytes) +
                                     " (ask for fewer splits, or pass 0)");
      // Library-chosen split count: the largest count whose partials fit (one split needs none). On 148 SMs the
      // planner's own counts always fit (it splits only fewer than ~240 (row, KV head) pairs, into at most ~3300
      // CTAs: <= 6.9 MB of partials); a part with more SMs could ask for more.
      const size_t per_split = size_t(n_rows) * n_heads * (64 + 1) * sizeof(float);
      const int fit = static_cast<int>(kStaticScratchBytes / per_split);
      plan = nbl::plan_decode(n_rows, kv->cfg.n_kv_heads, group, n_heads, max_seq_len, kv->cfg.page_size,
                              ctx->num_sms, fit >= 2 ? fit : 1);
    }
    void* scratch = plan.n_splits > 1 ? resolved_scratch(ctx->device) : nullptr;
    unsigned* counts = plan.n_splits > 1 && int64_t(n_rows) * kv->cfg.n_kv_heads <= kStaticCounts
                           ? g_counts_addr[ctx->device]
                           : nullptr;
    nbl::launch_decode(ctx->stream, kv, q, page_table, pt_stride, seq_lens, n_rows, n_heads, out, lse, plan, scratch,
                       ctx->d_err, counts);
    return NBL_OK;
  } catch (const nbl::Failure& e) {
    return nbl::record_error(e.status, e.what());
  } catch (const std::bad_alloc&) {
    return nbl::record_error(NBL_E_NOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return nbl::record_error(NBL_E_INVALID, e.what());
  }
}
