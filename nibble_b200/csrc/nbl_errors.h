// Bits of the per-context device error word that kernels set (atomicOr) when a device-side check fails;
// nbl_ctx_check() reports any nonzero value as NBL_E_DEVICE with these causes spelled out.
#pragma once

namespace nbl {
enum : int {
  kErrPageId = 1,     // a page-table entry outside [0, n_pages)
  kErrLength = 2,     // a sequence length / position outside the page table or the RoPE table
  kErrTimeout = 4,    // a bounded wait gave up (lost TMA / MMA completion)
  kErrTmemAlloc = 8,  // tensor-memory allocation failed
  kErrSmemAlign = 16, // dynamic shared memory not 1024-byte aligned (swizzled TMA tiles need it)
};
}  // namespace nbl
