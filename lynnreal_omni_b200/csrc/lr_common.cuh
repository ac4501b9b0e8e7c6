// Shared device helpers for the W8A8 projection-path kernels (sm_100a).
//
// Arithmetic contract (what "bit-exact" means for these kernels):
//   * every fp32 product and sum is rounded on its own (no FMA contraction),
//     matching the reference's `enable_fp_fusion=False` launches
//     (model/kernels.py:270,287,302; model/int8_gemm.py:243,260);
//   * bf16 rounding points are round-to-nearest-even, written out as bf16r();
//   * divisions and the RMS reciprocal square root are IEEE round-to-nearest
//     (__fdiv_rn, __fsqrt_rn), so a CPU restatement reproduces them exactly;
//   * float -> int8 quantisation rounds half to even (cvt.rni).
//
// Reductions use one fixed tree (see block_sum): thread partial sums in column
// order, an xor butterfly inside each warp, then a fixed pairwise tree over the
// warps. The CPU oracle restates the same tree.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace lr {

// Device-side status word. Kernels OR error bits into it instead of trapping;
// the host reads and clears it with lr_device_status().
enum : unsigned int {
  kDevErrTableIndex = 1u << 0,  // an adaLN index pointed outside the table
  kDevErrWaitTimeout = 1u << 1, // a bounded mbarrier wait gave up
};

// ---------------------------------------------------------------- bf16 helpers
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf_bits(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ uint16_t f2bf_bits(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return (uint32_t)f2bf_bits(lo) | ((uint32_t)f2bf_bits(hi) << 16);
}
// Unpack eight bf16 values held in a 16-byte vector.
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf2(f[0], f[1]); v.y = pack_bf2(f[2], f[3]);
  v.z = pack_bf2(f[4], f[5]); v.w = pack_bf2(f[6], f[7]);
  return v;
}

// Symmetric int8 quantisation of one value with an fp32 row scale:
// RNE(clamp(v / s, -127, 127)), model/kernels.py:14,126 and model/int8.py:67.
__device__ __forceinline__ int quant_i8(float v, float s) {
  float q = __fdiv_rn(v, s);
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return __float2int_rn(q);
}
// Row scale from a row absmax: max(absmax, 1e-8) / 127 (model/kernels.py:13,121-122).
__device__ __forceinline__ float row_scale_from_absmax(float absmax) {
  return __fdiv_rn(fmaxf(absmax, 1.0e-8f), 127.0f);
}

// Read-only streaming loads/stores (bypass L1 allocation for one-touch data).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// ------------------------------------------------------------- block reductions
// Fixed-order block reduction over NWARPS warps. Every thread returns the same
// value. `scratch` must hold NWARPS floats; the trailing __syncthreads makes the
// scratch reusable by the next call.
template <int NWARPS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float s[NWARPS];
#pragma unroll
  for (int w = 0; w < NWARPS; ++w) s[w] = scratch[w];
  // pairwise tree: level by level, neighbours (0,1),(2,3),... then (01,23),...
#pragma unroll
  for (int width = NWARPS; width > 1; width >>= 1) {
#pragma unroll
    for (int i = 0; i < width / 2; ++i) s[i] = __fadd_rn(s[2 * i], s[2 * i + 1]);
  }
  __syncthreads();
  return s[0];
}

template <int NWARPS>
__device__ __forceinline__ float block_max(float v, float* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float m = scratch[0];
#pragma unroll
  for (int w = 1; w < NWARPS; ++w) m = fmaxf(m, scratch[w]);
  __syncthreads();
  return m;
}

}  // namespace lr
