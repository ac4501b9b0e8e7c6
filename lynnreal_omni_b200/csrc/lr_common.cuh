// Shared device helpers for the W8A8 projection-path kernels (sm_100a).
//
// Arithmetic contract (what "bit-exact" means for these kernels):
//   * every fp32 product and sum is rounded on its own (no FMA contraction),
//     matching the reference's `enable_fp_fusion=False` launches
//     (model/kernels.py:270,287,302; model/int8_gemm.py:139,156);
//   * bf16 rounding points are round-to-nearest-even;
//   * divisions and the RMS reciprocal square root either as the reference's
//     compiled kernels execute them on the GPU (div.full, rsqrt.approx) or
//     IEEE round-to-nearest (__fdiv_rn, __fsqrt_rn), which a CPU restatement
//     reproduces (see quotient());
//   * float -> int8 quantisation rounds half to even.
//
// Packed bf16 arithmetic. Where the reference computes an fp32 product or sum
// of two bf16 values and rounds it to bf16, these kernels use one
// mul.rn.bf16x2 / add.rn.bf16x2 per two elements. The results are identical:
// the fp32 product of two bf16 values is exact, and rounding an fp32 sum to
// bf16 equals rounding the exact sum once (fp32 carries more than 2*8+2
// significand bits, so the double rounding is innocuous) — outside the
// subnormal range, which activations of this path do not reach.
//
// Reductions use one fixed tree, the one the reference's compiled tl.sum uses
// for a row of 8 warps with 8 elements per thread (rows of 2048 columns or
// more): each thread adds its values in order, chunk by chunk, then an xor
// butterfly (16, 8, 4, 2, 1) inside each warp and an xor butterfly (4, 2, 1)
// over the warp sums (block_sum). The CPU oracle restates the same tree.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace lr {

// Device-side status bits. Kernels OR error bits into a status word instead of
// trapping; the host reads and clears it with lr_device_status().
enum : unsigned int {
  kDevErrTableIndex = 1u << 0,  // an adaLN index pointed outside the table
  kDevErrWaitTimeout = 1u << 1, // a bounded mbarrier wait gave up
  kDevErrRowIndex = 1u << 2,    // a gather/restore row index pointed outside its source
};

// ------------------------------------------------------- scalar bf16 helpers
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

// ------------------------------------------------------- packed bf16x2 helpers
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t w) {
  return *reinterpret_cast<__nv_bfloat162*>(&w);
}
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}
// Round two fp32 values to bf16 (nearest even) and pack them (lo, hi).
__device__ __forceinline__ uint32_t cvt2(float lo, float hi) {
  return as_u32(__floats2bfloat162_rn(lo, hi));
}
// bf16(a * b) and bf16(a + b), element-wise on two packed values.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  return as_u32(__hmul2_rn(as_bf2(a), as_bf2(b)));
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  return as_u32(__hadd2_rn(as_bf2(a), as_bf2(b)));
}
// Running max of |a| over packed values (acc holds non-negative bf16 values).
__device__ __forceinline__ uint32_t bamax2(uint32_t acc, uint32_t a) {
  return as_u32(__hmax2(as_bf2(acc), as_bf2(a & 0x7fff7fffu)));
}
__device__ __forceinline__ float bamax_final(uint32_t acc) { return fmaxf(bf_lo(acc), bf_hi(acc)); }

constexpr uint32_t kBf2One = 0x3f803f80u;  // (1.0, 1.0) in bf16x2

// Widen both bf16 halves of a word to fp32. With LR_WIDEN_FMA the widening is
// the mixed-precision add.rn.f32.bf16 of each half and -0.0 (exact for every
// value, signed zeros included), an FMA-pipe instruction, instead of a shift
// and a mask on the integer pipe.
#ifndef LR_WIDEN_FMA
#define LR_WIDEN_FMA 1
#endif
__device__ __forceinline__ float2 widen2(uint32_t w) {
#if LR_WIDEN_FMA
  float2 f;
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "add.rn.f32.bf16 %0, l, 0f80000000;\n\tadd.rn.f32.bf16 %1, h, 0f80000000;\n\t}"
      : "=f"(f.x), "=f"(f.y)
      : "r"(w));
  return f;
#else
  return make_float2(bf_lo(w), bf_hi(w));
#endif
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const float2 a = widen2(v.x), b = widen2(v.y), c = widen2(v.z), d = widen2(v.w);
  f[0] = a.x; f[1] = a.y;
  f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y;
  f[6] = d.x; f[7] = d.y;
}
// Round eight fp32 values to bf16 and pack them.
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(cvt2(f[0], f[1]), cvt2(f[2], f[3]), cvt2(f[4], f[5]), cvt2(f[6], f[7]));
}
__device__ __forceinline__ uint4 bmul8(const uint4& a, const uint4& b) {
  return make_uint4(bmul2(a.x, b.x), bmul2(a.y, b.y), bmul2(a.z, b.z), bmul2(a.w, b.w));
}
__device__ __forceinline__ uint4 badd8(const uint4& a, const uint4& b) {
  return make_uint4(badd2(a.x, b.x), badd2(a.y, b.y), badd2(a.z, b.z), badd2(a.w, b.w));
}
__device__ __forceinline__ uint32_t bamax8(uint32_t acc, const uint4& a) {
  acc = bamax2(acc, a.x);
  acc = bamax2(acc, a.y);
  acc = bamax2(acc, a.z);
  return bamax2(acc, a.w);
}

// ------------------------------------------------------------- quantisation
// Division and the RMS reciprocal square root come in two forms, chosen per
// launch (`gpu`):
//   gpu = true   the instructions the reference's Triton kernels compile to on
//                the GPU: fp32 `/` is PTX div.full.f32 and tl.rsqrt is PTX
//                rsqrt.approx.f32 (what the reference computes on a B200);
//   gpu = false  IEEE round-to-nearest (__fdiv_rn, __fsqrt_rn): the
//                reference's PyTorch path and its Triton kernels under the
//                Triton interpreter, which the CPU oracle restates.
__device__ __forceinline__ float div_full(float a, float b) {
  float d;
  asm("div.full.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float rsqrt_approx(float a) {
  float d;
  asm("rsqrt.approx.f32 %0, %1;" : "=f"(d) : "f"(a));
  return d;
}
__device__ __forceinline__ float quotient(float a, float b, bool gpu) {
  return gpu ? div_full(a, b) : __fdiv_rn(a, b);
}
// 1 / sqrt(ss / n + eps)   (model/kernels.py:65,106)
__device__ __forceinline__ float rms_factor(float ss, float n, float eps, bool gpu) {
  if (gpu) return rsqrt_approx(__fadd_rn(div_full(ss, n), eps));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, n), eps)));
}

// Row scale from a row absmax: max(absmax, 1e-8) / 127 (model/kernels.py:13,121-122).
__device__ __forceinline__ float row_scale_from_absmax(float absmax, bool gpu) {
  return quotient(fmaxf(absmax, 1.0e-8f), 127.0f, gpu);
}

// Scalar reference form: RNE(clamp(v / s, -127, 127)) (model/kernels.py:14,126).
__device__ __forceinline__ int quant_i8(float v, float s, bool gpu) {
  float q = quotient(v, s, gpu);
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return __float2int_rn(q);
}

// Eight bf16 values -> eight int8 (packed in a uint2), exactly
// RNE(clamp(v / s, -127, 127)) for the quotient v / s of the chosen
// arithmetic: IEEE division, or (`gpu`) div.full.f32, which the compiled
// reference uses.
//   * s >= absmax/127 of the row, so |v / s| < 127.5 and the clamp never binds
//     for finite values (div.full.f32 is within 2 ulp of v / s);
//   * q0 = v * (1/s) (both IEEE-rounded) lies within 2^-16 of v / s for
//     |v / s| < 128, and so does either quotient (IEEE: exactly rounded;
//     div.full.f32: within 2 ulp, at most 2^-16 below 128), so all three round
//     to the same integer unless q0 is within 2^-14 of a half-integer; those
//     (rare) chunks redo the quotient itself;
//   * rounding to an integer is the float add of 1.5*2^23 (exact RNE for
//     |q| < 2^22), whose low mantissa byte is the two's-complement int8.
#ifndef LR_QUANT_FAST_GPU
#define LR_QUANT_FAST_GPU 1  // 0: div.full.f32 on every element in the gpu arithmetic (tuning knob)
#endif
__device__ __forceinline__ uint2 pack_q8(const uint32_t (&b)[8]) {
  const uint32_t lo = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
  const uint32_t hi = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
  return make_uint2(lo, hi);
}
// The quotients themselves: RNE(v / s) in the chosen arithmetic.
__device__ __forceinline__ uint2 quant8_exact(const uint4& v, float s, bool gpu) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float f[8];
  unpack8(v, f);
  uint32_t b[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) b[e] = __float_as_uint(__fadd_rn(gpu ? div_full(f[e], s) : __fdiv_rn(f[e], s), kMagic));
  return pack_q8(b);
}
// The reciprocal form alone: the bytes of RNE(v * (1/s)), with `near_tie`
// set if any of them lies within 2^-14 of a rounding tie (then the chunk must
// be redone by quant8_exact). Lets a kernel branch once for several chunks.
__device__ __forceinline__ uint2 quant8_fast(const uint4& v, float inv, bool& near_tie) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float f[8];
  unpack8(v, f);
  uint32_t b[8];
  const float2 inv2 = make_float2(inv, inv);
  const float2 magic2 = make_float2(kMagic, kMagic);
  const float2 nmagic2 = make_float2(-kMagic, -kMagic);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float2 q0 = __fmul2_rn(make_float2(f[e], f[e + 1]), inv2);
    const float2 t = __fadd2_rn(q0, magic2);
    const float2 r = __fadd2_rn(t, nmagic2);
    const float2 d = __fadd2_rn(q0, make_float2(-r.x, -r.y));
    near_tie |= (fabsf(d.x) > 0.49993896484375f) | (fabsf(d.y) > 0.49993896484375f);  // 0.5 - 2^-14
    b[e] = __float_as_uint(t.x);
    b[e + 1] = __float_as_uint(t.y);
  }
  return pack_q8(b);
}
__device__ __forceinline__ uint2 quant8(const uint4& v, float s, float inv, bool gpu) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float f[8];
  unpack8(v, f);
  uint32_t b[8];
  if (gpu && !LR_QUANT_FAST_GPU) {
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = __float_as_uint(__fadd_rn(div_full(f[e], s), kMagic));
    return pack_q8(b);
  }
  bool near_tie = false;
  const float2 inv2 = make_float2(inv, inv);
  const float2 magic2 = make_float2(kMagic, kMagic);
  const float2 nmagic2 = make_float2(-kMagic, -kMagic);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float2 q0 = __fmul2_rn(make_float2(f[e], f[e + 1]), inv2);
    const float2 t = __fadd2_rn(q0, magic2);
    const float2 r = __fadd2_rn(t, nmagic2);
    const float2 d = __fadd2_rn(q0, make_float2(-r.x, -r.y));
    near_tie |= (fabsf(d.x) > 0.49993896484375f) | (fabsf(d.y) > 0.49993896484375f);  // 0.5 - 2^-14
    b[e] = __float_as_uint(t.x);
    b[e + 1] = __float_as_uint(t.y);
  }
  if (near_tie) {
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = __float_as_uint(__fadd_rn(gpu ? div_full(f[e], s) : __fdiv_rn(f[e], s), kMagic));
  }
  return pack_q8(b);
}

// Read-only streaming loads (bypass L1 allocation for one-touch data).
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
  // xor butterfly over the warp sums, as warp 0's lanes would run it:
  // s[w] += s[w ^ off] for off = NWARPS/2, ..., 1; the result is s[0]
#pragma unroll
  for (int off = NWARPS / 2; off > 0; off >>= 1) {
#pragma unroll
    for (int w = 0; w < off; ++w) s[w] = __fadd_rn(s[w], s[w + off]);
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
