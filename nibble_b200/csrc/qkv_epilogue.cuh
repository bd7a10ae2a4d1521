// The fused Q/K/V projection epilogue shared by the float GEMV (model_ops.cu) and the quantized GEMV
// (quant_ops.cu): which weight row a warp computes when it walks RoPE pairs, and what it stores once both members
// of a pair are done. The arithmetic is the reference's add_bias then cpu::rope (src/backend/cpu/ref_ops.cpp:156-185)
// followed by RNE narrowing into the page slot, exactly as nbl_rope_kv_append does it.
#pragma once
#include "model_ops.h"
#include "nbl_device.cuh"

namespace nbl {

// Fused Q/K/V epilogue: virtual row vr = 2u + h is member h of pair u. Pairs are numbered Q heads' first, then K's,
// then V's, 32 per head: a Q or K pair is the RoPE pair i of its head (NeoX: elements i and i + 32; else 2i and
// 2i + 1), a V pair is elements 2i and 2i + 1. Returns the weight-row number in the batch (Q rows, then K, then V).
__device__ __forceinline__ int64_t qkv_row(int64_t vr, const QkvEpilogue& e, int& region, int& head, int& pair) {
  const int64_t u = vr >> 1;
  const int half = static_cast<int>(vr & 1);
  const int64_t qu = int64_t(e.n_heads) * 32, ku = int64_t(e.n_kv_heads) * 32;
  int64_t base, rel;
  if (u < qu) {
    region = 0;
    rel = u;
    base = 0;
  } else if (u < qu + ku) {
    region = 1;
    rel = u - qu;
    base = int64_t(e.n_heads) * 64;
  } else {
    region = 2;
    rel = u - qu - ku;
    base = (int64_t(e.n_heads) + e.n_kv_heads) * 64;
  }
  head = static_cast<int>(rel >> 5);
  pair = static_cast<int>(rel & 31);
  const int within = region != 2 && e.neox ? pair + 32 * half : 2 * pair + half;
  return base + int64_t(head) * 64 + within;
}

// The epilogue of pair (ia, ib) of one head for activation row t: bias, rotation (Q, K), and the stores.
__device__ __forceinline__ void qkv_store(const QkvEpilogue& e, int region, int head, int pair, int t, float a,
                                          float b) {
  const int ia = region != 2 && e.neox ? pair : 2 * pair;
  const int ib = region != 2 && e.neox ? pair + 32 : 2 * pair + 1;
  const float* bias = region == 0 ? e.bq : (region == 1 ? e.bk : e.bv);
  const int64_t boff = int64_t(head) * 64;
  if (bias) {
    a = __fadd_rn(a, bias[boff + ia]);
    b = __fadd_rn(b, bias[boff + ib]);
  }
  const int64_t pos = int64_t(e.pos0) + t;
  if (region != 2) {
    if (pos >= e.tab_pos) {
      flag_error(e.err, kErrLength);
      return;
    }
    rope_rotate(a, b, e.tab[pos * 32 + pair], a, b);
  }
  if (region == 0) {
    float* q = e.q_out + int64_t(t) * e.n_heads * 64 + boff;
    q[ia] = a;
    q[ib] = b;
    return;
  }
  if (pos >= int64_t(e.pt_stride) * 16) {
    flag_error(e.err, kErrLength);
    return;
  }
  const int32_t page = e.page_table[pos >> 4];
  if (page < 0 || page >= e.n_pages) {
    flag_error(e.err, kErrPageId);
    return;
  }
  __half* slot = static_cast<__half*>(e.pool) +
                 ((int64_t(page) * 2 + (region == 2 ? 1 : 0)) * e.n_kv_heads + head) * 1024 + (pos & 15) * 64;
  slot[ia] = __float2half_rn(a);
  slot[ib] = __float2half_rn(b);
}

}  // namespace nbl
