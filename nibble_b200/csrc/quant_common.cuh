// Device helpers shared by the quantized GEMV (quant_ops.cu) and the quantized tensor-core GEMM (quant_gemm.cu):
// the reference's Q8_0 activation quantizer for one block (src/quant.cpp:37-51) and the unpacking of Q4_0 / Q5_0
// value bytes (src/quant.cpp:158-205).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace nbl {

// The 4-bit / 5-bit value bytes of a Q4_0 / Q5_0 block widened to the int8 values dp4a takes, in element order:
// lo[i] holds elements 4i..4i+3 (low nibbles of bytes 4i..4i+3), hi[i] elements 16+4i..16+4i+3.
__device__ __forceinline__ void unpack_nibbles(const uint4 q, int (&lo)[4], int (&hi)[4]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    lo[i] = static_cast<int>(w[i] & 0x0F0F0F0Fu);
    hi[i] = static_cast<int>((w[i] >> 4) & 0x0F0F0F0Fu);
  }
}

// Spreads bits [first, first + 4) of qh to bit 4 of four bytes (the fifth bit of four Q5_0 elements).
__device__ __forceinline__ int high_bits4(uint32_t qh, int first) {
  const uint32_t b = qh >> first;
  return static_cast<int>(((b & 1u) << 4) | ((b & 2u) << 11) | ((b & 4u) << 18) | ((b & 8u) << 25));
}

// One warp per 32-element block: amax by a max reduction (fmaxf skips NaN like std::fmax; a NaN anywhere makes d
// NaN), d = amax / 127, q = roundf(x * (1 / d)) clamped to [-127, 127] (NaN -> 0); the scale is kept as the fp32
// value of its fp16 rounding, which is what the dot products read. Lane i passes element i of the block; it gets
// back the block's scale and writes its own int8 value.
__device__ __forceinline__ float quantize_block(const float v, int8_t* q_out) {
  float amax = fabsf(v);
  bool nan = v != v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  nan = __any_sync(0xffffffffu, nan);
  const float dd = nan ? __int_as_float(0x7fc00000) : __fdiv_rn(amax, 127.f);
  const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.f;
  const float r = roundf(__fmul_rn(v, id));
  *q_out = static_cast<int8_t>(r != r ? 0 : static_cast<int>(fminf(127.f, fmaxf(-127.f, r))));
  return __half2float(__float2half_rn(dd));
}

}  // namespace nbl
