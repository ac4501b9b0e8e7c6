// HBM-bound row kernels of the W8A8 projection path (sm_100a):
//   K1 quantize_rows, K2 int8_epilogue, K3/K4/K8 RMSNorm+adaLN(+quant)(+residual),
//   K5 gated residual, K6/K7 SwiGLU(+quant).
//
// Layout: one 256-thread CTA per row. Thread t owns the 8-column chunks that
// start at columns (c*256 + t)*8 for c = 0..C-1, so a warp reads 512
// contiguous bytes of bf16 per chunk with 16-byte loads. A row is read from
// HBM once and kept in registers as packed bf16 between the reduction passes
// (every intermediate of these kernels is bf16-representable).
#include <initializer_list>
#include <mutex>
#include <unordered_map>

#include "lr_common.cuh"
#include "lr_host.h"

// Minimum resident CTAs per SM requested for the one-row RMSNorm kernel on
// rows of up to 4 chunks per thread (a register cap when nonzero). With the
// reference's summation order the compiler's own allocation is faster
// (12240 x 6144: K4 81.2 -> 78.4 us, K3 58.5 -> 56.4 us against a cap of 4, 64
// registers). Tuning knob.
#ifndef LR_RMS_MINB
#define LR_RMS_MINB 0
#endif
// The same caps for the two-row residual RMSNorm kernel on rows of up to 3
// chunks per thread (K8: 3 -> 80 registers, 3 CTAs per SM; 123 -> 108 us at
// 12240 x 6144 with the 16-column sum order), for the quantiser on rows of
// more than 4 chunks per thread (K1 on
// FFN widths: 4 -> 64 registers; 185 -> 140 us at 12240 x 24576, ~ the HBM copy
// rate) and for the SwiGLU kernels (4: 292 -> 270 us at 12240 x 2 x 14336).
#ifndef LR_RMS2_MINB
#define LR_RMS2_MINB 3
#endif
#ifndef LR_QUANT_WIDE_MINB
#define LR_QUANT_WIDE_MINB 4
#endif
#ifndef LR_SWIGLU_MINB
#define LR_SWIGLU_MINB 4
#endif
// Caps for the quantiser on rows of up to 4 chunks per thread (0: a cap of 5
// measured slower) and for the per-token Q/K RMSNorm + RoPE kernel (4 -> 64
// registers: 148 -> 124 us at 12240 tokens x 48 heads).
#ifndef LR_QUANT_MINB
#define LR_QUANT_MINB 0
#endif
#ifndef LR_QK_MINB
#define LR_QK_MINB 4
#endif

namespace lr {

static __device__ unsigned int g_device_status = 0;

// Arithmetic of divisions and the RMS reciprocal square root for every kernel
// of this file (see quotient() in lr_common.cuh): 1 = as the reference's
// compiled Triton kernels on the GPU (the default), 0 = IEEE, as its PyTorch
// path and the CPU oracle. One value per device, set by lr_set_arithmetic.
__constant__ int c_arith_gpu = 1;
__device__ __forceinline__ bool arith_gpu() { return c_arith_gpu != 0; }

__device__ __forceinline__ void flag_error(unsigned int bits) { atomicOr(&g_device_status, bits); }

}  // namespace lr

#include "lr_rows.cuh"

namespace lr {
using rows::load_chunk;
using rows::store_chunk;
using rows::store_q8;
using rows::splat8;
using rows::RmsArgs;
using rows::table_row_ptr;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSpan = kThreads * 8;  // columns covered by one chunk sweep

using bf16 = __nv_bfloat16;

// Load the C chunks of one row owned by this thread.
template <int C, bool VEC, bool STREAM>
__device__ __forceinline__ void load_row(uint4 (&dst)[C], const bf16* row, int64_t width) {
#pragma unroll
  for (int c = 0; c < C; ++c)
    dst[c] = load_chunk<VEC, STREAM>(row, ((int64_t)c * kThreads + threadIdx.x) * 8, width);
}

// Persistent row loop: CTA b handles rows b, b + gridDim.x, ...; for narrow
// rows (C <= 4) the next row's chunks are loaded into registers before the
// current row is reduced, so each CTA keeps one row of loads in flight while
// it computes. Wider rows already issue C >= 6 loads per thread per row.
template <int C>
struct Prefetch {
  static constexpr bool kOn = C <= 4;
  static constexpr int kN = kOn ? C : 1;
};

// --------------------------------------------------------------------- K1
template <int C, bool VEC>
__global__ void __launch_bounds__(kThreads, (C > 4 ? LR_QUANT_WIDE_MINB : LR_QUANT_MINB)) quantize_rows_kernel(const bf16* __restrict__ x,
                                                                  int64_t row_stride, int width,
                                                                  int8_t* __restrict__ q,
                                                                  float* __restrict__ scales,
                                                                  int64_t rows, int arith) {
  __shared__ float red[kWarps];
  int64_t row = blockIdx.x;
  // arith < 0: the device's mode (lr_set_arithmetic); LR_ARITH_TORCH_CUDA: the
  // scale is absmax times the float reciprocal of 127 (how PyTorch divides a
  // CUDA tensor by a scalar), the quotient IEEE
  const bool gpu = arith < 0 ? arith_gpu() : arith == LR_ARITH_REFERENCE_GPU;
  const bool by_reciprocal = arith == LR_ARITH_TORCH_CUDA;
  if (row >= rows) return;
  uint4 raw[C];
  load_row<C, VEC, true>(raw, x + row * row_stride, width);
  while (true) {
    const int64_t next = row + gridDim.x;
    uint4 nxt[Prefetch<C>::kN];
    if (Prefetch<C>::kOn && next < rows)
      load_row<Prefetch<C>::kN, VEC, true>(nxt, x + next * row_stride, width);
    uint32_t amax2 = 0u;
#pragma unroll
    for (int c = 0; c < C; ++c) amax2 = bamax8(amax2, raw[c]);
    const float amax = block_max<kWarps>(bamax_final(amax2), red);
    const float s = by_reciprocal ? __fmul_rn(fmaxf(amax, 1.0e-8f), 1.0f / 127.0f)
                                  : row_scale_from_absmax(amax, gpu);
    const float inv = __frcp_rn(s);
    int8_t* dst = q + row * (int64_t)width;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      store_q8<VEC>(dst, col, width, quant8(raw[c], s, inv, gpu));
    }
    if (threadIdx.x == 0) scales[row] = s;
    if (next >= rows) break;
    if (Prefetch<C>::kOn) {
#pragma unroll
      for (int c = 0; c < C; ++c) raw[c] = nxt[Prefetch<C>::kOn ? c : 0];
    } else {
      load_row<C, VEC, true>(raw, x + next * row_stride, width);
    }
    row = next;
  }
}

// --------------------------------------------------------------- K3/K4/K8
// Sums of squares in the reference's compiled order. Its bf16-output kernel
// lays a row out with 8 columns per thread, like the chunks here, and each
// thread adds its squares in column order. Its int8-output kernels lay it out
// with 16 columns per thread (the 16-byte int8 stores): thread t' adds columns
// 4096 r + 16 t' + [0, 16) for r = 0, 1, ... . Here thread t holds the 8-column
// chunks c*256 + t, so the 16-column thread j + 128 p (j = t >> 1, p = 0, 1) is
// the chain over chunks c = p, p + 2, ... alternating between the lanes 2j
// and 2j + 1: the running sum crosses the lane pair by shuffles. The 256
// chains go through `stage` to the thread with their index, so block_sum then
// reduces them in the reference's butterflies. Squares of bf16 values are
// exact in fp32, so each fused multiply-add equals the separate multiply and add.
// Running max of magnitudes over packed bf16 values: max.xorsign.abs keeps
// max(|acc|, |a|) per lane (the sign bit it sets is discarded at the end).
__device__ __forceinline__ uint32_t bmaxabs2(uint32_t acc, uint32_t a) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(a));
  return d;
}
__device__ __forceinline__ float bmaxabs_final(uint32_t acc) { return fmaxf(fabsf(bf_lo(acc)), fabsf(bf_hi(acc))); }

// acc + lo(u)^2, then + hi(u)^2: the mixed-precision fma.rn.f32.bf16 of
// sm_100 multiplies the bf16 halves exactly and rounds the sum once, as the
// fp32 fma of the widened values does, without unpacking them first.
__device__ __forceinline__ float sumsq_word(float acc, uint32_t u) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\t"
      "fma.rn.f32.bf16 %0, l, l, %0;\n\tfma.rn.f32.bf16 %0, h, h, %0;\n\t}"
      : "+f"(acc)
      : "r"(u));
  return acc;
}

template <int C>
__device__ __forceinline__ float sumsq_part8(const uint4 (&v)[C]) {
  float part = 0.0f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    part = sumsq_word(part, v[c].x);
    part = sumsq_word(part, v[c].y);
    part = sumsq_word(part, v[c].z);
    part = sumsq_word(part, v[c].w);
  }
  return part;
}

template <int C>
__device__ __forceinline__ float sumsq_part16(const uint4 (&v)[C], float* stage) {
  const int lane = threadIdx.x & 31;
  float acc[2] = {0.0f, 0.0f};
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float f[8];
    unpack8(v[c], f);
    float a = acc[c & 1];  // the even lane continues the chain with its chunk
#pragma unroll
    for (int e = 0; e < 8; ++e) a = __fmaf_rn(f[e], f[e], a);
    float b = __shfl_sync(0xffffffffu, a, lane & ~1);  // then the odd lane with its own
#pragma unroll
    for (int e = 0; e < 8; ++e) b = __fmaf_rn(f[e], f[e], b);
    acc[c & 1] = __shfl_sync(0xffffffffu, b, lane | 1);
  }
  stage[(threadIdx.x >> 1) + 128 * (threadIdx.x & 1)] = acc[threadIdx.x & 1];
  __syncthreads();
  return stage[threadIdx.x];
}

// Both rows of the two-row kernel at once (.x row 0, .y row 1).
template <int C>
__device__ __forceinline__ float2 sumsq_part16x2(const uint4 (&v0)[C], const uint4 (&v1)[C], float2* stage) {
  const int lane = threadIdx.x & 31;
  float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float f0[8], f1[8];
    unpack8(v0[c], f0);
    unpack8(v1[c], f1);
    float2 a = acc[c & 1];
#pragma unroll
    for (int e = 0; e < 8; ++e) a = __ffma2_rn(make_float2(f0[e], f1[e]), make_float2(f0[e], f1[e]), a);
    float2 b = make_float2(__shfl_sync(0xffffffffu, a.x, lane & ~1), __shfl_sync(0xffffffffu, a.y, lane & ~1));
#pragma unroll
    for (int e = 0; e < 8; ++e) b = __ffma2_rn(make_float2(f0[e], f1[e]), make_float2(f0[e], f1[e]), b);
    acc[c & 1] = make_float2(__shfl_sync(0xffffffffu, b.x, lane | 1), __shfl_sync(0xffffffffu, b.y, lane | 1));
  }
  stage[(threadIdx.x >> 1) + 128 * (threadIdx.x & 1)] = acc[threadIdx.x & 1];
  __syncthreads();
  return stage[threadIdx.x];
}

template <int C, bool VEC, bool RESID, bool MOD, bool QUANT>
__device__ __forceinline__ void rms_mod_row(const RmsArgs& a, int64_t row, uint4 (&v)[C],
                                            const uint4 (&d)[C], float* red, float* stage) {
  const int hidden = a.hidden;
  bool bad;
  const bf16* trow = table_row_ptr(a.table, a.table_rows, a.table_width, a.indices, a.sequence,
                                   row, bad);
  if (bad && threadIdx.x == 0) flag_error(kDevErrTableIndex);
  const bool have_table = trow != nullptr;

  if (RESID) {
    // v = bf16(x + bf16(gate * update))   (model/kernels.py:101-105)
    const uint4 gate_default = splat8(a.table == nullptr ? kBf2One : 0u);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      const uint4 gt = have_table
                           ? load_chunk<VEC, false>(trow + (int64_t)a.gate_slot * hidden, col, hidden)
                           : gate_default;
      v[c] = badd8(v[c], bmul8(gt, d[c]));
      store_chunk<VEC>(a.residual_out + row * (int64_t)hidden, col, hidden, v[c]);
    }
  }

  // sum of squares in the order of the reference's kernel for this output
  const float part = (QUANT && C >= 2) ? sumsq_part16<C>(v, stage) : sumsq_part8<C>(v);
  const float ss = block_sum<kWarps>(part, red);
  // r = 1 / sqrt(ss / hidden + eps)   (model/kernels.py:65,106)
  const bool gpu = arith_gpu();
  const float r = rms_factor(ss, (float)hidden, a.eps, gpu);

  uint32_t amax2 = 0u;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
    float f[8], w[8];
    unpack8(v[c], f);
    unpack8(load_chunk<VEC, false>(a.weight, col, hidden), w);
    // n = bf16((x * r) * w)   (model/kernels.py:65-68,106-108)
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 n2 = __fmul2_rn(__fmul2_rn(make_float2(f[e], f[e + 1]), r2), make_float2(w[e], w[e + 1]));
      f[e] = n2.x;
      f[e + 1] = n2.y;
    }
    uint4 m = pack8(f);
    if (MOD && have_table) {
      // m = bf16(bf16(n * bf16(1 + scale)) + shift)   (model/kernels.py:77-78,117-120)
      const uint4 sc = load_chunk<VEC, false>(trow + (int64_t)a.scale_slot * hidden, col, hidden);
      const uint4 sh = load_chunk<VEC, false>(trow + (int64_t)a.shift_slot * hidden, col, hidden);
      m = badd8(bmul8(m, badd8(splat8(kBf2One), sc)), sh);
    }
    if (QUANT) amax2 = bamax8(amax2, m);
    v[c] = m;
  }

  if (QUANT) {
    const float amax = block_max<kWarps>(bamax_final(amax2), red);
    const float s = row_scale_from_absmax(amax, gpu);
    const float inv = __frcp_rn(s);
    int8_t* dst = a.q + row * (int64_t)hidden;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      store_q8<VEC>(dst, col, hidden, quant8(v[c], s, inv, gpu));
    }
    if (threadIdx.x == 0) a.scales[row] = s;
  } else {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      store_chunk<VEC>(a.out + row * (int64_t)hidden, col, hidden, v[c]);
    }
  }
}

template <int C, bool VEC, bool RESID, bool MOD, bool QUANT>
__global__ void __launch_bounds__(kThreads, (C <= 4 ? LR_RMS_MINB : 0)) rms_mod_kernel(const RmsArgs a) {
  __shared__ float red[kWarps];
  __shared__ float stage[(QUANT && C >= 2) ? kThreads : 1];
  constexpr bool kPre = Prefetch<C>::kOn;
  constexpr int kN = Prefetch<C>::kN;
  constexpr int kD = RESID ? C : 1;
  int64_t row = blockIdx.x;
  if (row >= a.rows) return;
  uint4 v[C], d[kD];
  load_row<C, VEC, true>(v, a.x + row * (int64_t)a.hidden, a.hidden);
  if (RESID) load_row<kD, VEC, true>(d, a.update + row * (int64_t)a.hidden, a.hidden);
  while (true) {
    const int64_t next = row + gridDim.x;
    uint4 nv[kN], nd[RESID ? kN : 1];
    if (kPre && next < a.rows) {
      load_row<kN, VEC, true>(nv, a.x + next * (int64_t)a.hidden, a.hidden);
      if (RESID) load_row<RESID ? kN : 1, VEC, true>(nd, a.update + next * (int64_t)a.hidden, a.hidden);
    }
    uint4 dd[C];
#pragma unroll
    for (int c = 0; c < C; ++c) dd[c] = d[RESID ? c : 0];
    rms_mod_row<C, VEC, RESID, MOD, QUANT>(a, row, v, dd, red, stage);
    if (next >= a.rows) break;
    if (kPre) {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        v[c] = nv[kPre ? c : 0];
        if (RESID) d[RESID ? c : 0] = nd[(RESID && kPre) ? c : 0];
      }
    } else {
      load_row<C, VEC, true>(v, a.x + next * (int64_t)a.hidden, a.hidden);
      if (RESID) load_row<kD, VEC, true>(d, a.update + next * (int64_t)a.hidden, a.hidden);
    }
    row = next;
  }
}

// ------------------------------------------------- K4/K8 in the 16-column layout
// The int8-output RMSNorm kernels of the reference lay a row out over 256
// threads with 16 columns each: reference thread t' sums the squares of
// columns 4096 r + 16 t' + [0, 16), r = 0, 1, ..., in order, then the row sum
// is an xor butterfly inside each of its 8 warps and across the warps. Here a
// 128-thread CTA owns a row and thread t stands in for reference threads t
// and t + 128 (reference warps g and g + 4 of warp g), so every chain lives in
// one thread: no lane-pair shuffles and no transpose through shared memory.
// Group k of a thread is (t' = t + 128 (k / R), r = k % R); each group is one
// 32-byte load (sm_100 256-bit vector access), a warp reads 1 KB contiguous.
// The first cross-warp step of the reference's butterfly (w + 4 into w) is the
// sum of a thread's two chains' warp sums; the last two go through shared
// memory. Results are identical to rms_mod_kernel. Rows of 2048 to 8192
// columns, a multiple of 16.
constexpr int kQ16Threads = 128;

struct Bf16x16 {
  uint32_t w[8];
};

__device__ __forceinline__ Bf16x16 ld256_stream(const void* p) {
  Bf16x16 v;
  asm volatile("ld.global.cs.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
__device__ __forceinline__ Bf16x16 ld256_keep(const void* p) {
  Bf16x16 v;
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st256(void* p, const Bf16x16& v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
               "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
               : "memory");
}
__device__ __forceinline__ Bf16x16 splat16(uint32_t w) {
  Bf16x16 v;
#pragma unroll
  for (int i = 0; i < 8; ++i) v.w[i] = w;
  return v;
}

// The per-row work of the 16-column K4/K8 kernels, from the row's groups in
// registers: residual (K8), sums of squares, RMS factor, normalise +
// modulate, absmax, quantise, stores. Two block barriers; every thread of the
// CTA calls it for the same row. FULL: every group of every thread lies
// inside the row (hidden = 2048 NG), so no group needs a bounds test, and the
// quantiser branches once per 16-column group to its exact path (values
// within 2^-14 of a rounding tie, rare) instead of once per 8 columns
// (measured at 12240 x 6144: 51.3 -> 50.3 us; at 5376 columns, where groups
// are partial, the per-8-column form stays faster).
template <int NG, int R, bool RESID, bool MOD, bool FULL>
__device__ __forceinline__ void q16_row(const RmsArgs& a, int64_t row, const int (&col)[NG], const bool (&ok)[NG],
                                        Bf16x16 (&v)[NG], const Bf16x16 (&d)[RESID ? NG : 1], float* red_sum,
                                        float* red_max, const bf16* trow) {
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int hidden = a.hidden;
  const bool have_table = trow != nullptr;
  if (RESID) {
    // v = bf16(x + bf16(gate * update))   (model/kernels.py:101-105)
    const uint32_t gate_default = a.table == nullptr ? kBf2One : 0u;
#pragma unroll
    for (int k = 0; k < NG; ++k) {
      if (!FULL && !ok[k]) continue;
      const Bf16x16 g = have_table ? ld256_keep(trow + (int64_t)a.gate_slot * hidden + col[k]) : splat16(gate_default);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[k].w[i] = badd2(v[k].w[i], bmul2(g.w[i], d[RESID ? k : 0].w[i]));
      st256(a.residual_out + row * (int64_t)hidden + col[k], v[k]);
    }
  }
  // chains: .x over the groups of t' = t, .y over those of t' = t + 128
  // (columns past the row are zeros and add exactly nothing)
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < NG; ++k) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (k < R) acc.x = sumsq_word(acc.x, v[k].w[i]);
      else acc.y = sumsq_word(acc.y, v[k].w[i]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc.x = __fadd_rn(acc.x, __shfl_xor_sync(0xffffffffu, acc.x, off));
    acc.y = __fadd_rn(acc.y, __shfl_xor_sync(0xffffffffu, acc.y, off));
  }
  if (lane == 0) red_sum[warp] = __fadd_rn(acc.x, acc.y);  // s[w] + s[w + 4]
  __syncthreads();
  const float4 rsum = *reinterpret_cast<const float4*>(red_sum);
  const float ss = __fadd_rn(__fadd_rn(rsum.x, rsum.z), __fadd_rn(rsum.y, rsum.w));
  const bool gpu = arith_gpu();
  // r = 1 / sqrt(ss / hidden + eps)   (model/kernels.py:65,106)
  const float rs = rms_factor(ss, (float)hidden, a.eps, gpu);
  const float2 r2 = make_float2(rs, rs);
  uint32_t amax2 = 0u;
#pragma unroll
  for (int k = 0; k < NG; ++k) {
    if (!FULL && !ok[k]) continue;
    const Bf16x16 w = ld256_keep(a.weight + col[k]);
    // n = bf16((x * r) * w)   (model/kernels.py:65-68,106-108)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 n = __fmul2_rn(__fmul2_rn(widen2(v[k].w[i]), r2), widen2(w.w[i]));
      v[k].w[i] = cvt2(n.x, n.y);
    }
    if (MOD && have_table) {
      // m = bf16(bf16(n * bf16(1 + scale)) + shift)   (model/kernels.py:117-120)
      const Bf16x16 sc = ld256_keep(trow + (int64_t)a.scale_slot * hidden + col[k]);
      const Bf16x16 sh = ld256_keep(trow + (int64_t)a.shift_slot * hidden + col[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[k].w[i] = badd2(bmul2(v[k].w[i], badd2(kBf2One, sc.w[i])), sh.w[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax2 = bmaxabs2(amax2, v[k].w[i]);
  }
  float amax = bmaxabs_final(amax2);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if (lane == 0) red_max[warp] = amax;
  __syncthreads();
  const float4 rmax = *reinterpret_cast<const float4*>(red_max);
  amax = fmaxf(fmaxf(rmax.x, rmax.y), fmaxf(rmax.z, rmax.w));
  const float s = row_scale_from_absmax(amax, gpu);
  const float inv = __frcp_rn(s);
  int8_t* dst = a.q + row * (int64_t)hidden;
#pragma unroll
  for (int k = 0; k < NG; ++k) {
    if (!FULL && !ok[k]) continue;
    const uint4 v0 = make_uint4(v[k].w[0], v[k].w[1], v[k].w[2], v[k].w[3]);
    const uint4 v1 = make_uint4(v[k].w[4], v[k].w[5], v[k].w[6], v[k].w[7]);
    uint2 lo, hi;
    if (FULL) {
      bool near_tie = gpu && !LR_QUANT_FAST_GPU;
      lo = quant8_fast(v0, inv, near_tie);
      hi = quant8_fast(v1, inv, near_tie);
      if (near_tie) {
        // a value of the group is within 2^-14 of a rounding tie (rare): the quotients
        lo = quant8_exact(v0, s, gpu);
        hi = quant8_exact(v1, s, gpu);
      }
    } else {
      lo = quant8(v0, s, inv, gpu);
      hi = quant8(v1, s, inv, gpu);
    }
    *reinterpret_cast<uint4*>(dst + col[k]) = make_uint4(lo.x, lo.y, hi.x, hi.y);
  }
  if (t == 0) a.scales[row] = s;
}

template <int NG, int R>
__device__ __forceinline__ void q16_columns(int (&col)[NG], bool (&ok)[NG], int hidden) {
#pragma unroll
  for (int k = 0; k < NG; ++k) {
    col[k] = 4096 * (k % R) + 16 * ((int)threadIdx.x + kQ16Threads * (k / R));
    ok[k] = col[k] < hidden;
  }
}

// One row per CTA of the same layout, for a grid of all rows: rows in flight
// are CTAs, not registers (a persistent form that prefetched the next row in
// registers held 4 CTAs per SM and ran 74 us at 12240 x 6144; staging the next
// rows, or the weights and modulation, in shared memory by cp.async was
// slower still).
#ifndef LR_Q16R_MINB
#define LR_Q16R_MINB 8
#endif
template <int NG, int R, bool RESID, bool MOD, bool FULL>
__global__ void __launch_bounds__(kQ16Threads, LR_Q16R_MINB) rms_quant16_row_kernel(const RmsArgs a) {
  __shared__ __align__(16) float red_sum[kQ16Threads / 32];
  __shared__ __align__(16) float red_max[kQ16Threads / 32];
  const int64_t row = blockIdx.x;
  int col[NG];
  bool ok[NG];
  q16_columns<NG, R>(col, ok, a.hidden);
  Bf16x16 v[NG], d[RESID ? NG : 1];
#pragma unroll
  for (int k = 0; k < NG; ++k) {
    if (FULL) {
      v[k] = ld256_stream(a.x + row * (int64_t)a.hidden + col[k]);
      if (RESID) d[RESID ? k : 0] = ld256_stream(a.update + row * (int64_t)a.hidden + col[k]);
    } else {
      v[k] = ok[k] ? ld256_stream(a.x + row * (int64_t)a.hidden + col[k]) : splat16(0u);
      if (RESID) d[RESID ? k : 0] = ok[k] ? ld256_stream(a.update + row * (int64_t)a.hidden + col[k]) : splat16(0u);
    }
  }
  bool bad;
  const bf16* trow = table_row_ptr(a.table, a.table_rows, a.table_width, a.indices, a.sequence, row, bad);
  if (bad && threadIdx.x == 0) flag_error(kDevErrTableIndex);
  q16_row<NG, R, RESID, MOD, FULL>(a, row, col, ok, v, d, red_sum, red_max, trow);
}

// --------------------------------------------------- K3 in the 8-column layout
// The reference's bf16-output RMSNorm kernel lays a row out over 256 threads
// with 8 columns each: reference thread t' sums the squares of columns
// 2048 c + 8 t' + [0, 8), c = 0, 1, ..., in order, then the same butterflies
// as the int8-output kernels. As in rms_quant16_row_kernel, a 128-thread CTA
// owns a row and thread t stands in for reference threads t and t + 128, so
// the chains need no exchange; chunk j of a thread is (t' = t + 128 (j % 2),
// c = j / 2), one 16-byte access. Results are identical to rms_mod_kernel.
#ifndef LR_K3R_MINB
#define LR_K3R_MINB 8
#endif
template <int C, bool MOD>
__global__ void __launch_bounds__(kQ16Threads, LR_K3R_MINB) rms_bf16_row_kernel(const RmsArgs a) {
  __shared__ float red_sum[kQ16Threads / 32];
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int hidden = a.hidden;
  const int64_t row = blockIdx.x;
  int col[2 * C];
#pragma unroll
  for (int j = 0; j < 2 * C; ++j) col[j] = 2048 * (j / 2) + 8 * (t + kQ16Threads * (j % 2));
  uint4 v[2 * C];
  const bf16* xrow = a.x + row * (int64_t)hidden;
#pragma unroll
  for (int j = 0; j < 2 * C; ++j) v[j] = load_chunk<true, true>(xrow, col[j], hidden);
  bool bad;
  const bf16* trow = table_row_ptr(a.table, a.table_rows, a.table_width, a.indices, a.sequence, row, bad);
  if (bad && t == 0) flag_error(kDevErrTableIndex);
  float2 acc = make_float2(0.0f, 0.0f);  // .x: t' = t, .y: t' = t + 128
#pragma unroll
  for (int j = 0; j < 2 * C; ++j) {
    float& c = (j % 2) ? acc.y : acc.x;
    c = sumsq_word(c, v[j].x);
    c = sumsq_word(c, v[j].y);
    c = sumsq_word(c, v[j].z);
    c = sumsq_word(c, v[j].w);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc.x = __fadd_rn(acc.x, __shfl_xor_sync(0xffffffffu, acc.x, off));
    acc.y = __fadd_rn(acc.y, __shfl_xor_sync(0xffffffffu, acc.y, off));
  }
  if (lane == 0) red_sum[warp] = __fadd_rn(acc.x, acc.y);  // s[w] + s[w + 4]
  __syncthreads();
  const float ss = __fadd_rn(__fadd_rn(red_sum[0], red_sum[2]), __fadd_rn(red_sum[1], red_sum[3]));
  // r = 1 / sqrt(ss / hidden + eps)   (model/kernels.py:65)
  const float rs = rms_factor(ss, (float)hidden, a.eps, arith_gpu());
  const float2 r2 = make_float2(rs, rs);
  bf16* orow = a.out + row * (int64_t)hidden;
#pragma unroll
  for (int j = 0; j < 2 * C; ++j) {
    if (col[j] >= hidden) continue;
    const uint4 w = load_chunk<true, false>(a.weight, col[j], hidden);
    const uint32_t xw[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t m[4];
    // n = bf16((x * r) * w)   (model/kernels.py:65-68)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 n = __fmul2_rn(__fmul2_rn(widen2(xw[i]), r2), widen2(ww[i]));
      m[i] = cvt2(n.x, n.y);
    }
    if (MOD && trow != nullptr) {
      // out = bf16(bf16(n * bf16(1 + scale)) + shift)   (model/kernels.py:77-78)
      const uint4 sc = load_chunk<true, false>(trow + (int64_t)a.scale_slot * hidden, col[j], hidden);
      const uint4 sh = load_chunk<true, false>(trow + (int64_t)a.shift_slot * hidden, col[j], hidden);
      m[0] = badd2(bmul2(m[0], badd2(kBf2One, sc.x)), sh.x);
      m[1] = badd2(bmul2(m[1], badd2(kBf2One, sc.y)), sh.y);
      m[2] = badd2(bmul2(m[2], badd2(kBf2One, sc.z)), sh.z);
      m[3] = badd2(bmul2(m[3], badd2(kBf2One, sc.w)), sh.w);
    }
    *reinterpret_cast<uint4*>(orow + col[j]) = make_uint4(m[0], m[1], m[2], m[3]);
  }
}

// Two rows per CTA: both rows' partial sums (and then absmaxes) go through one
// block reduction, halving the barriers per row and giving each thread two
// independent rows of work between them. Each row's reduction tree is exactly
// the single-row tree (block_sum2 / block_max2 reduce the two components
// separately in the same order), so results are identical to rms_mod_kernel.
template <int NWARPS>
__device__ __forceinline__ float2 block_sum2(float2 v, float2* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    v.x = __fadd_rn(v.x, __shfl_xor_sync(0xffffffffu, v.x, off));
    v.y = __fadd_rn(v.y, __shfl_xor_sync(0xffffffffu, v.y, off));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float2 s[NWARPS];
#pragma unroll
  for (int w = 0; w < NWARPS; ++w) s[w] = scratch[w];
#pragma unroll
  for (int off = NWARPS / 2; off > 0; off >>= 1) {
#pragma unroll
    for (int w = 0; w < off; ++w) s[w] = make_float2(__fadd_rn(s[w].x, s[w + off].x), __fadd_rn(s[w].y, s[w + off].y));
  }
  __syncthreads();
  return s[0];
}

template <int NWARPS>
__device__ __forceinline__ float2 block_max2(float2 v, float2* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    v.x = fmaxf(v.x, __shfl_xor_sync(0xffffffffu, v.x, off));
    v.y = fmaxf(v.y, __shfl_xor_sync(0xffffffffu, v.y, off));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float2 m = scratch[0];
#pragma unroll
  for (int w = 1; w < NWARPS; ++w) m = make_float2(fmaxf(m.x, scratch[w].x), fmaxf(m.y, scratch[w].y));
  __syncthreads();
  return m;
}

template <int C, bool VEC, bool RESID, bool MOD, bool QUANT>
__global__ void __launch_bounds__(kThreads, (C <= 3 ? LR_RMS2_MINB : 0)) rms_mod2_kernel(const RmsArgs a) {
  __shared__ float2 red[kWarps];
  __shared__ float2 stage[(QUANT && C >= 2) ? kThreads : 1];
  const int hidden = a.hidden;
  const int64_t row0 = 2 * (int64_t)blockIdx.x;
  const bool has1 = row0 + 1 < a.rows;
  const int64_t rows2[2] = {row0, has1 ? row0 + 1 : row0};
  uint4 v[2][C];
  const bf16* trow[2];
  bool have_table[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    bool bad;
    trow[j] = table_row_ptr(a.table, a.table_rows, a.table_width, a.indices, a.sequence, rows2[j], bad);
    if (bad && threadIdx.x == 0) flag_error(kDevErrTableIndex);
    have_table[j] = trow[j] != nullptr;
#pragma unroll
    for (int c = 0; c < C; ++c)
      v[j][c] = load_chunk<VEC, true>(a.x + rows2[j] * (int64_t)hidden,
                                      ((int64_t)c * kThreads + threadIdx.x) * 8, hidden);
  }
  if (RESID) {
    // v = bf16(x + bf16(gate * update))   (model/kernels.py:101-105)
    const uint4 gate_default = splat8(a.table == nullptr ? kBf2One : 0u);
    uint4 d[2][C];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < C; ++c)
        d[j][c] = load_chunk<VEC, true>(a.update + rows2[j] * (int64_t)hidden,
                                        ((int64_t)c * kThreads + threadIdx.x) * 8, hidden);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
        const uint4 gt = have_table[j]
                             ? load_chunk<VEC, false>(trow[j] + (int64_t)a.gate_slot * hidden, col, hidden)
                             : gate_default;
        v[j][c] = badd8(v[j][c], bmul8(gt, d[j][c]));
        if (j == 0 || has1) store_chunk<VEC>(a.residual_out + rows2[j] * (int64_t)hidden, col, hidden, v[j][c]);
      }
  }
  // sums of squares of both rows (.x row 0, .y row 1) in the order of the
  // reference's kernel for this output
  float2 part;
  if (QUANT && C >= 2) {
    part = sumsq_part16x2<C>(v[0], v[1], stage);
  } else {
    part = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      float f0[8], f1[8];
      unpack8(v[0][c], f0);
      unpack8(v[1][c], f1);
#pragma unroll
      for (int e = 0; e < 8; ++e) part = __ffma2_rn(make_float2(f0[e], f1[e]), make_float2(f0[e], f1[e]), part);
    }
  }
  const float2 ss = block_sum2<kWarps>(part, red);
  // r = 1 / sqrt(ss / hidden + eps)   (model/kernels.py:65,106)
  const bool gpu = arith_gpu();
  const float rr[2] = {rms_factor(ss.x, (float)hidden, a.eps, gpu), rms_factor(ss.y, (float)hidden, a.eps, gpu)};
  uint32_t amax2[2] = {0u, 0u};
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
    float w[8];
    unpack8(load_chunk<VEC, false>(a.weight, col, hidden), w);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float f[8];
      unpack8(v[j][c], f);
      const float2 r2 = make_float2(rr[j], rr[j]);
      // n = bf16((x * r) * w)   (model/kernels.py:65-68,106-108)
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 n2 = __fmul2_rn(__fmul2_rn(make_float2(f[e], f[e + 1]), r2), make_float2(w[e], w[e + 1]));
        f[e] = n2.x;
        f[e + 1] = n2.y;
      }
      uint4 m = pack8(f);
      if (MOD && have_table[j]) {
        // m = bf16(bf16(n * bf16(1 + scale)) + shift)   (model/kernels.py:77-78,117-120)
        const uint4 sc = load_chunk<VEC, false>(trow[j] + (int64_t)a.scale_slot * hidden, col, hidden);
        const uint4 sh = load_chunk<VEC, false>(trow[j] + (int64_t)a.shift_slot * hidden, col, hidden);
        m = badd8(bmul8(m, badd8(splat8(kBf2One), sc)), sh);
      }
      if (QUANT) amax2[j] = bamax8(amax2[j], m);
      v[j][c] = m;
    }
  }
  if (QUANT) {
    const float2 amax = block_max2<kWarps>(make_float2(bamax_final(amax2[0]), bamax_final(amax2[1])), red);
    const float am[2] = {amax.x, amax.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (j == 1 && !has1) break;
      const float s = row_scale_from_absmax(am[j], gpu);
      const float inv = __frcp_rn(s);
      int8_t* dst = a.q + rows2[j] * (int64_t)hidden;
#pragma unroll
      for (int c = 0; c < C; ++c)
        store_q8<VEC>(dst, ((int64_t)c * kThreads + threadIdx.x) * 8, hidden, quant8(v[j][c], s, inv, gpu));
      if (threadIdx.x == 0) a.scales[rows2[j]] = s;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (j == 1 && !has1) break;
#pragma unroll
      for (int c = 0; c < C; ++c)
        store_chunk<VEC>(a.out + rows2[j] * (int64_t)hidden, ((int64_t)c * kThreads + threadIdx.x) * 8, hidden,
                         v[j][c]);
    }
  }
}

// --------------------------------------------------------------------- K5
template <int C, bool VEC>
__global__ void __launch_bounds__(kThreads) gated_residual_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ y, const bf16* __restrict__ table,
    int64_t table_rows, int64_t table_width, const int64_t* __restrict__ indices,
    int64_t sequence, int hidden, int gate_slot, bf16* __restrict__ out, int64_t rows) {
  constexpr bool kPre = Prefetch<C>::kOn;
  constexpr int kN = Prefetch<C>::kN;
  const uint4 gate_default = splat8(table == nullptr ? kBf2One : 0u);
  int64_t row = blockIdx.x;
  if (row >= rows) return;
  uint4 xv[C], yv[C];
  load_row<C, VEC, true>(xv, x + row * (int64_t)hidden, hidden);
  load_row<C, VEC, true>(yv, y + row * (int64_t)hidden, hidden);
  while (true) {
    const int64_t next = row + gridDim.x;
    uint4 nx[kN], ny[kN];
    if (kPre && next < rows) {
      load_row<kN, VEC, true>(nx, x + next * (int64_t)hidden, hidden);
      load_row<kN, VEC, true>(ny, y + next * (int64_t)hidden, hidden);
    }
    bool bad;
    const bf16* trow = table_row_ptr(table, table_rows, table_width, indices, sequence, row, bad);
    if (bad && threadIdx.x == 0) flag_error(kDevErrTableIndex);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      const uint4 gt = trow != nullptr
                           ? load_chunk<VEC, false>(trow + (int64_t)gate_slot * hidden, col, hidden)
                           : gate_default;
      // out = bf16(x + bf16(gate * y))   (model/kernels.py:146-153)
      store_chunk<VEC>(out + row * (int64_t)hidden, col, hidden, badd8(xv[c], bmul8(gt, yv[c])));
    }
    if (next >= rows) break;
    if (kPre) {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        xv[c] = nx[kPre ? c : 0];
        yv[c] = ny[kPre ? c : 0];
      }
    } else {
      load_row<C, VEC, true>(xv, x + next * (int64_t)hidden, hidden);
      load_row<C, VEC, true>(yv, y + next * (int64_t)hidden, hidden);
    }
    row = next;
  }
}

// ------------------------------------------------------------------ K6/K7
// 1: the sigmoid of SwiGLU uses the fast hardware exponential and division
// (__expf, __fdividef), as the reference's compiled Triton kernel does
// (tl.sigmoid lowers to ex2.approx and div.full); 0: expf and IEEE division.
// Both reproduce the reference's golden SwiGLU outputs exactly; the fast form
// runs the K7 kernel in 162 instead of 270 us at 12240 x 2 x 14336. Tuning knob.
#ifndef LR_SWIGLU_FAST
#define LR_SWIGLU_FAST 1
#endif
__device__ __forceinline__ float silu(float g) {
  // g * sigmoid(g), sigmoid(g) = 1 / (1 + exp(-g))   (model/kernels.py:165,177)
  if (LR_SWIGLU_FAST) return __fmul_rn(g, __fdividef(1.0f, __fadd_rn(1.0f, __expf(-g))));
  return __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
}

template <int C, bool VEC, bool QUANT>
__global__ void __launch_bounds__(kThreads, LR_SWIGLU_MINB) swiglu_kernel(const bf16* __restrict__ projected,
                                                          int inner, bf16* __restrict__ out,
                                                          int8_t* __restrict__ q,
                                                          float* __restrict__ scales,
                                                          int64_t rows) {
  __shared__ float red[kWarps];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const bf16* value = projected + row * 2 * (int64_t)inner;
    const bf16* gate = value + inner;
    uint4 v[C];
    uint32_t amax2 = 0u;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
      float gf[8];
      unpack8(load_chunk<VEC, true>(gate, col, inner), gf);
#pragma unroll
      for (int e = 0; e < 8; ++e) gf[e] = silu(gf[e]);
      // bf16(value * bf16(silu(gate)))
      v[c] = bmul8(load_chunk<VEC, true>(value, col, inner), pack8(gf));
      if (QUANT) amax2 = bamax8(amax2, v[c]);
    }
    if (QUANT) {
      const float amax = block_max<kWarps>(bamax_final(amax2), red);
      const bool gpu = arith_gpu();
      const float s = row_scale_from_absmax(amax, gpu);
      const float inv = __frcp_rn(s);
      int8_t* dst = q + row * (int64_t)inner;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
        store_q8<VEC>(dst, col, inner, quant8(v[c], s, inv, gpu));
      }
      if (threadIdx.x == 0) scales[row] = s;
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int64_t col = ((int64_t)c * kThreads + threadIdx.x) * 8;
        store_chunk<VEC>(out + row * (int64_t)inner, col, inner, v[c]);
      }
    }
  }
}

// -------------------------------------------------------- Q/K RMSNorm + RoPE
// model/kernels.py:188-257 (full rotary) and :345-402 (general), per head row:
//   r = 1 / sqrt(sum(x^2) / head_dim + eps);  n = bf16((x * r) * w)
//   d < rotary_dim: bf16(bf16(n_d * c_d) + bf16(-+n_pair * s_d)), c/s the
//   bf16-rounded cos/sin of the row's token, pair = d +- rotary_dim / 2.
// One sum order for both kernels below: with L = next power of two >=
// ceil(head_dim / 8) lanes per row, lane l holds elements [8l, 8l + 8), sums
// the squares of its even and of its odd elements (left to right), adds the
// two, and the L lanes add by an xor butterfly (L/2, ..., 1).

// Fast form: one CTA per token, heads contiguous (head stride = head_dim),
// 16-byte aligned rows, head_dim = 8L with L a power of two <= 32, rotary_dim
// 0 or 16 * 2^k. Thread t owns chunk position p = t % L of every head it
// touches (256 is a multiple of L), so its weights and cos/sin are loaded once
// per token; the rotary partner chunk is lane p ^ (rotary_dim / 16) of the
// same head. All NI chunk loads of a thread are issued before any compute.
// The sum that threads holding one term each compute with xor butterflies over
// their 32-thread warps and then over the warps, as seen from thread 0 (the
// butterfly leaves that value in every thread): at offset o, thread T adds
// thread T + o. Here lane p holds the terms T = 8p .. 8p+7 in v; the terms
// span n_lanes lanes (a power of two) from this lane group's first lane, which
// returns the total. Offsets 16 and 8 are lanes 2 and 1 away, 4, 2 and 1 are
// inside a lane, and warp w's sum sits in lane 4w.
__device__ __forceinline__ float thread_tree_sum(float (&v)[8], int n_lanes) {
  const int n = n_lanes * 8;
  if (n >= 32) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], __shfl_down_sync(0xffffffffu, v[j], 2));
  }
  if (n >= 16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], __shfl_down_sync(0xffffffffu, v[j], 1));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], v[j + 4]);
  v[0] = __fadd_rn(v[0], v[2]);
  v[1] = __fadd_rn(v[1], v[3]);
  v[0] = __fadd_rn(v[0], v[1]);
  for (int ow = (n >> 5) >> 1; ow > 0; ow >>= 1) v[0] = __fadd_rn(v[0], __shfl_down_sync(0xffffffffu, v[0], 4 * ow));
  return v[0];
}

// Head-row sum of squares of the Q/K kernels in the order of the reference's
// compiled Q/K kernels (4 warps, one term per thread, so exact for head
// dimensions up to 128; thread_tree_sum). `f` are this lane's 8 values (columns 8p .. 8p+7 of
// the head row), `raw` the same as packed bf16; the head's lanes start at
// `base`.
//   * full rotary (paired): terms x_i^2 + x_{i+D/2}^2 for i < D/2
//     (model/kernels.py:217-222), the partner values from lane p + D/16;
//   * otherwise: terms x_i^2 (model/kernels.py:374-375).
// A bf16 value's square is exact in fp32, so a fused multiply-add of one
// equals the separate multiply and add.
__device__ __forceinline__ float qk_sumsq(const float (&f)[8], const uint4& raw, int p, int base, int lanes,
                                          int head_dim, bool paired) {
  float t[8];
  int n_lanes = lanes;
  if (paired) {
    const int h8 = head_dim >> 4;
    const int src = base + (p < h8 ? p + h8 : p - h8);
    const uint4 y = make_uint4(__shfl_sync(0xffffffffu, raw.x, src), __shfl_sync(0xffffffffu, raw.y, src),
                               __shfl_sync(0xffffffffu, raw.z, src), __shfl_sync(0xffffffffu, raw.w, src));
    float g[8];
    unpack8(y, g);
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = p < h8 ? __fmaf_rn(g[e], g[e], __fmul_rn(f[e], f[e])) : 0.0f;
    n_lanes = 1;
    while (n_lanes < h8) n_lanes <<= 1;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = __fmul_rn(f[e], f[e]);
  }
  const float total = thread_tree_sum(t, n_lanes);
  return __shfl_sync(0xffffffffu, total, base);
}

template <int NI>
__global__ void __launch_bounds__(256, LR_QK_MINB) qk_norm_rope_tok_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, int64_t q_ts, int64_t k_ts,
    const bf16* __restrict__ wq, const bf16* __restrict__ wk, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int64_t sequence, int qc, int lanes, int head_dim, int rotary_dim,
    float eps, bf16* __restrict__ q_out, bf16* __restrict__ k_out) {
  const int64_t tok = blockIdx.x;
  const int64_t b = tok / sequence, s = tok - b * sequence;
  const int t = threadIdx.x;
  const int p = t & (lanes - 1);
  uint4 x[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int c = t + 256 * i;
    if (c < 2 * qc) {
      const bool is_k = c >= qc;
      const int cc = is_k ? c - qc : c;
      const bf16* src = is_k ? k + (b * sequence + s) * k_ts : q + (b * sequence + s) * q_ts;
      x[i] = ld_stream(src + (int64_t)cc * 8);
    } else {
      x[i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  float wqf[8], wkf[8];
  unpack8(ld_keep(wq + p * 8), wqf);
  unpack8(ld_keep(wk + p * 8), wkf);
  const bool rotates = p * 8 < rotary_dim;
  const bool lower = p * 8 < rotary_dim / 2;
  const bool paired = rotary_dim == head_dim && head_dim % 16 == 0;
  const int pair = rotary_dim / 16;
  uint4 c2 = make_uint4(0u, 0u, 0u, 0u), s2 = c2;
  if (rotates) {
    const float4* cp = reinterpret_cast<const float4*>(cos_t + s * rotary_dim + p * 8);
    const float4* sp = reinterpret_cast<const float4*>(sin_t + s * rotary_dim + p * 8);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    c2 = make_uint4(cvt2(c0.x, c0.y), cvt2(c0.z, c0.w), cvt2(c1.x, c1.y), cvt2(c1.z, c1.w));
    s2 = make_uint4(cvt2(s0.x, s0.y), cvt2(s0.z, s0.w), cvt2(s1.x, s1.y), cvt2(s1.z, s1.w));
  }
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int c = t + 256 * i;
    const bool is_k = c >= qc;
    float f[8];
    unpack8(x[i], f);
    const float ss = qk_sumsq(f, x[i], p, (t & 31) & ~(lanes - 1), lanes, head_dim, paired);
    const float r = rms_factor(ss, (float)head_dim, eps, arith_gpu());
    const float2 r2 = make_float2(r, r);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 n2 = __fmul2_rn(__fmul2_rn(make_float2(f[e], f[e + 1]), r2),
                                   is_k ? make_float2(wkf[e], wkf[e + 1]) : make_float2(wqf[e], wqf[e + 1]));
      f[e] = n2.x;
      f[e + 1] = n2.y;
    }
    uint4 n = pack8(f);
    if (rotary_dim > 0) {
      uint4 m = make_uint4(__shfl_xor_sync(0xffffffffu, n.x, pair), __shfl_xor_sync(0xffffffffu, n.y, pair),
                           __shfl_xor_sync(0xffffffffu, n.z, pair), __shfl_xor_sync(0xffffffffu, n.w, pair));
      if (rotates) {
        if (lower) m = make_uint4(m.x ^ 0x80008000u, m.y ^ 0x80008000u, m.z ^ 0x80008000u, m.w ^ 0x80008000u);
        n = badd8(bmul8(n, c2), bmul8(m, s2));
      }
    }
    if (c < 2 * qc) {
      const int cc = is_k ? c - qc : c;
      *reinterpret_cast<uint4*>((is_k ? k_out : q_out) + tok * (int64_t)qc * 8 + (int64_t)cc * 8) = n;
    }
  }
}

// General form (any head/token strides and alignment, head_dim <= 256, any
// even rotary_dim): one warp per (batch, token, head) row, Q then K, element
// loads; the normalised row is staged in shared memory so each lane can read
// its rotary partner wherever it lies.
__global__ void __launch_bounds__(256) qk_norm_rope_row_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, int64_t q_ts, int64_t q_hs, int64_t k_ts,
    int64_t k_hs, const bf16* __restrict__ wq, const bf16* __restrict__ wk,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int64_t rows, int64_t sequence,
    int heads, int head_dim, int lanes, int rotary_dim, float eps, bf16* __restrict__ q_out,
    bf16* __restrict__ k_out) {
  __shared__ float buf[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = rotary_dim / 2;
  const bool paired = rotary_dim == head_dim && head_dim % 16 == 0;
  const uint16_t* wbits[2] = {reinterpret_cast<const uint16_t*>(wq), reinterpret_cast<const uint16_t*>(wk)};
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += (int64_t)gridDim.x * 8) {
    const int64_t token = (row / heads) % sequence;
    const int64_t head = row % heads;
    const int64_t batch = row / (sequence * heads);
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const int64_t ts = which ? k_ts : q_ts, hs = which ? k_hs : q_hs;
      const uint16_t* src = reinterpret_cast<const uint16_t*>(which ? k : q) + batch * sequence * ts +
                            token * ts + head * hs;
      uint16_t* dst = reinterpret_cast<uint16_t*>(which ? k_out : q_out) + row * (int64_t)head_dim;
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        x[e] = d < head_dim ? bf_bits(src[d]) : 0.0f;
      }
      const uint4 raw = pack8(x);  // exact: the values are bf16
      const float ss = qk_sumsq(x, raw, lane, 0, lanes, head_dim, paired);
      const float r = rms_factor(ss, (float)head_dim, eps, arith_gpu());
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        if (d < head_dim) {
          x[e] = bf16r(__fmul_rn(__fmul_rn(x[e], r), bf_bits(wbits[which][d])));
          buf[warp][d] = x[e];
        }
      }
      __syncwarp();
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        if (d >= head_dim) continue;
        float o = x[e];
        if (d < rotary_dim) {
          const float c = bf16r(cos_t[token * rotary_dim + d]);
          const float sn = bf16r(sin_t[token * rotary_dim + d]);
          const float pv = d < half ? -buf[warp][d + half] : buf[warp][d - half];
          o = bf16r(__fadd_rn(bf16r(__fmul_rn(x[e], c)), bf16r(__fmul_rn(pv, sn))));
        }
        dst[d] = f2bf_bits(o);
      }
      __syncwarp();
    }
  }
}

// --------------------------------------------------------------------- K2
// One CTA per row; 4 int32 accumulators per thread step.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) int8_epilogue_kernel(
    const int32_t* __restrict__ acc, int64_t cols, const float* __restrict__ row_scale,
    const float* __restrict__ col_scale, const bf16* __restrict__ bias, bf16* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const float rs = row_scale[row];
  const int32_t* ar = acc + row * cols;
  uint16_t* orow = reinterpret_cast<uint16_t*>(out + row * cols);
  const uint16_t* bb = reinterpret_cast<const uint16_t*>(bias);
  for (int64_t col = (int64_t)threadIdx.x * 4; col < cols; col += (int64_t)kThreads * 4) {
    int32_t a4[4];
    if (VEC) {
      const int4 t = __ldcs(reinterpret_cast<const int4*>(ar + col));
      a4[0] = t.x; a4[1] = t.y; a4[2] = t.z; a4[3] = t.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) a4[e] = (col + e < cols) ? ar[col + e] : 0;
    }
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t n = (col + e < cols) ? col + e : col;
      // (float(acc) * row_scale) * col_scale + bias   (model/kernels.py:33-38)
      d[e] = __fmul_rn(__fmul_rn(__int2float_rn(a4[e]), rs), col_scale[n]);
      if (bias != nullptr) d[e] = __fadd_rn(d[e], bf_bits(bb[n]));
    }
    if (VEC) {
      *reinterpret_cast<uint2*>(orow + col) = make_uint2(cvt2(d[0], d[1]), cvt2(d[2], d[3]));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (col + e < cols) orow[col + e] = f2bf_bits(d[e]);
    }
  }
}

// Smallest supported chunk count covering `width` columns, or -1.
int pick_chunks(int64_t width) {
  const int64_t need = (width + kSpan - 1) / kSpan;
  const int options[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int c : options)
    if (c >= need) return c;
  return -1;
}

#define LR_CHUNK_DISPATCH(C, ...)                   \
  switch (C) {                                      \
    case 1: { constexpr int kC = 1; __VA_ARGS__; } break;   \
    case 2: { constexpr int kC = 2; __VA_ARGS__; } break;   \
    case 3: { constexpr int kC = 3; __VA_ARGS__; } break;   \
    case 4: { constexpr int kC = 4; __VA_ARGS__; } break;   \
    case 6: { constexpr int kC = 6; __VA_ARGS__; } break;   \
    case 8: { constexpr int kC = 8; __VA_ARGS__; } break;   \
    case 12: { constexpr int kC = 12; __VA_ARGS__; } break; \
    default: { constexpr int kC = 16; __VA_ARGS__; } break; \
  }

constexpr int64_t kMaxRows = 0x7fffffff;

// Grid of a persistent row kernel: every CTA that fits at once on the GPU
// (occupancy of this instantiation x SM count), capped by the row count.
template <typename Kernel>
unsigned persistent_grid(Kernel kernel, int64_t rows, bool persistent = true, int threads = kThreads,
                         size_t smem = 0) {
  if (!persistent) return (unsigned)rows;  // one row per CTA
  static std::mutex mu;
  static std::unordered_map<const void*, int> per_sm;
  int n = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = per_sm.find(reinterpret_cast<const void*>(kernel));
    if (it != per_sm.end()) {
      n = it->second;
    } else {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
      }
      per_sm.emplace(reinterpret_cast<const void*>(kernel), n);
    }
  }
  const int64_t g = (int64_t)n * sm_count();
  return (unsigned)(rows < g ? rows : g);
}

}  // namespace

int read_status_elementwise(unsigned int* bits, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess)
    return launch_status("reading the device status");
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess)
      return launch_status("clearing the device status");
  }
  *bits |= v;
  return LR_OK;
}

}  // namespace lr

using lr::bf16;
using lr::kMaxRows;
using lr::pick_chunks;

extern "C" int lr_set_arithmetic(int mode) {
  LR_REQUIRE(mode == LR_ARITH_IEEE || mode == LR_ARITH_REFERENCE_GPU, "set_arithmetic: unknown mode %d", mode);
  if (cudaMemcpyToSymbol(lr::c_arith_gpu, &mode, sizeof(mode)) != cudaSuccess)
    return lr::launch_status("setting the arithmetic mode");
  return LR_OK;
}

extern "C" int lr_get_arithmetic(int* mode) {
  LR_REQUIRE(mode != nullptr, "get_arithmetic: null pointer");
  if (cudaMemcpyFromSymbol(mode, lr::c_arith_gpu, sizeof(int)) != cudaSuccess)
    return lr::launch_status("reading the arithmetic mode");
  return LR_OK;
}

static int quantize_rows_launch(const void* x, int64_t rows, int64_t width, int64_t row_stride, int8_t* q,
                                float* scales, int arith, void* stream) {
  LR_REQUIRE(rows >= 0 && width > 0, "quantize_rows: invalid shape [%lld, %lld]", (long long)rows,
             (long long)width);
  LR_REQUIRE(row_stride >= width, "quantize_rows: row stride %lld < width %lld",
             (long long)row_stride, (long long)width);
  if (rows == 0) return LR_OK;
  LR_REQUIRE(x && q && scales, "quantize_rows: null pointer");
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "quantize_rows: too many rows");
  const int C = pick_chunks(width);
  if (C < 0) return lr::set_error(LR_ERR_UNSUPPORTED, "quantize_rows: width %lld > 32768", (long long)width);
  const bool vec = width % 8 == 0 && row_stride % 8 == 0 && lr::aligned(x, 16) && lr::aligned(q, 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bf16* xp = static_cast<const bf16*>(x);
  LR_CHUNK_DISPATCH(C, {
    if (vec)
      lr::quantize_rows_kernel<kC, true><<<lr::persistent_grid(lr::quantize_rows_kernel<kC, true>, rows, lr::Prefetch<kC>::kOn), lr::kThreads, 0, s>>>(xp, row_stride, (int)width, q, scales, rows, arith);
    else
      lr::quantize_rows_kernel<kC, false><<<lr::persistent_grid(lr::quantize_rows_kernel<kC, false>, rows, lr::Prefetch<kC>::kOn), lr::kThreads, 0, s>>>(xp, row_stride, (int)width, q, scales, rows, arith);
  });
  return lr::launch_status("quantize_rows");
}

extern "C" int lr_quantize_rows(const void* x, int64_t rows, int64_t width, int64_t row_stride,
                                int8_t* q, float* scales, void* stream) {
  return quantize_rows_launch(x, rows, width, row_stride, q, scales, -1, stream);
}

extern "C" int lr_quantize_rows_arith(const void* x, int64_t rows, int64_t width, int64_t row_stride,
                                      int8_t* q, float* scales, int arithmetic, void* stream) {
  LR_REQUIRE(arithmetic == LR_ARITH_IEEE || arithmetic == LR_ARITH_REFERENCE_GPU ||
             arithmetic == LR_ARITH_TORCH_CUDA, "quantize_rows: unknown arithmetic %d", arithmetic);
  return quantize_rows_launch(x, rows, width, row_stride, q, scales, arithmetic, stream);
}

extern "C" int lr_int8_epilogue(const int32_t* acc, int64_t rows, int64_t cols,
                                const float* row_scale, const float* col_scale, const void* bias,
                                void* out, void* stream) {
  LR_REQUIRE(rows >= 0 && cols > 0, "int8_epilogue: invalid shape");
  if (rows == 0) return LR_OK;
  LR_REQUIRE(acc && row_scale && col_scale && out, "int8_epilogue: null pointer");
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "int8_epilogue: too many rows");
  const bool vec = cols % 4 == 0 && lr::aligned(acc, 16) && lr::aligned(out, 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    lr::int8_epilogue_kernel<true><<<(unsigned)rows, lr::kThreads, 0, s>>>(
        acc, cols, row_scale, col_scale, static_cast<const bf16*>(bias), static_cast<bf16*>(out));
  else
    lr::int8_epilogue_kernel<false><<<(unsigned)rows, lr::kThreads, 0, s>>>(
        acc, cols, row_scale, col_scale, static_cast<const bf16*>(bias), static_cast<bf16*>(out));
  return lr::launch_status("int8_epilogue");
}

namespace {

int check_table(const char* who, const void* table, int64_t table_rows, int64_t table_width,
                const int64_t* indices, int64_t sequence, int64_t hidden, int slot_a, int slot_b,
                int slot_c) {
  LR_REQUIRE(sequence > 0, "%s: sequence must be positive", who);
  if (table == nullptr) return LR_OK;
  LR_REQUIRE(indices != nullptr, "%s: indices are required with a table", who);
  LR_REQUIRE(table_rows > 0, "%s: empty adaLN table", who);
  const int hi = slot_a > slot_b ? (slot_a > slot_c ? slot_a : slot_c) : (slot_b > slot_c ? slot_b : slot_c);
  const int lo = slot_a < slot_b ? (slot_a < slot_c ? slot_a : slot_c) : (slot_b < slot_c ? slot_b : slot_c);
  LR_REQUIRE(lo >= 0 && (int64_t)(hi + 1) * hidden <= table_width,
             "%s: slot %d does not fit a table row of width %lld (hidden %lld)", who, hi,
             (long long)table_width, (long long)hidden);
  return LR_OK;
}

bool vec_ok(int64_t hidden, std::initializer_list<const void*> ptrs) {
  if (hidden % 8) return false;
  for (const void* p : ptrs)
    if (p && !lr::aligned(p, 16)) return false;
  return true;
}

}  // namespace

// The gated residual (K5) and the bf16-output RMSNorm (K3) run one row per CTA
// (grid = rows) instead of the persistent prefetching grid: 70.8 -> 66.8 us
// and 60.0 -> 58.5 us at 12240 x 6144. Tuning knobs.
#ifndef LR_K5_ONE
#define LR_K5_ONE 1
#endif
#ifndef LR_K3_ONE
#define LR_K3_ONE 1
#endif
#ifndef LR_RMS2_OFF
#define LR_RMS2_OFF 0  // 1: the residual variant runs the one-row kernel too (tuning knob)
#endif

#ifndef LR_Q16_OFF
#define LR_Q16_OFF 0  // 1: K4/K8 run the 8-column-chunk kernels (tuning knob)
#endif
// K4/K8 in the reference's 16-column layout (rms_quant16_row_kernel): rows of
// 2048 to 8192 columns, a multiple of 16, with 32-byte aligned bf16 operands
// and 16-byte aligned int8 rows.
static bool q16_ok(const lr::RmsArgs& a) {
  if (LR_Q16_OFF || a.hidden < 2048 || a.hidden > 8192 || a.hidden % 16) return false;
  for (const void* p : {(const void*)a.x, (const void*)a.update, (const void*)a.weight, (const void*)a.table,
                        (const void*)a.residual_out})
    if (p && !lr::aligned(p, 32)) return false;
  return lr::aligned(a.q, 16) && (a.table == nullptr || a.table_width % 16 == 0);
}

template <int NG, int R, bool RESID, bool MOD>
static void q16_row_launch(const lr::RmsArgs& a, int64_t rows, cudaStream_t s) {
  // every group inside the row: 2048 columns per group
  if (a.hidden == 2048 * NG)
    lr::rms_quant16_row_kernel<NG, R, RESID, MOD, true><<<(unsigned)rows, lr::kQ16Threads, 0, s>>>(a);
  else
    lr::rms_quant16_row_kernel<NG, R, RESID, MOD, false><<<(unsigned)rows, lr::kQ16Threads, 0, s>>>(a);
}

template <int NG, int R>
static void q16_launch(const lr::RmsArgs& a, int64_t rows, bool resid, bool mod, cudaStream_t s) {
  if (resid) {
    if (mod) q16_row_launch<NG, R, true, true>(a, rows, s); else q16_row_launch<NG, R, true, false>(a, rows, s);
  } else {
    if (mod) q16_row_launch<NG, R, false, true>(a, rows, s); else q16_row_launch<NG, R, false, false>(a, rows, s);
  }
}

#ifndef LR_K3R_OFF
#define LR_K3R_OFF 0  // 1: K3 runs the 256-thread chunk kernel (tuning knob)
#endif

static int rms_launch(const lr::RmsArgs& a, int64_t rows, bool resid, bool mod, bool quant, bool vec,
                      cudaStream_t s) {
  if (quant && q16_ok(a)) {
    if (a.hidden <= 4096) q16_launch<2, 1>(a, rows, resid, mod, s);
    else if (a.hidden <= 6144) q16_launch<3, 2>(a, rows, resid, mod, s);
    else q16_launch<4, 2>(a, rows, resid, mod, s);
    return lr::launch_status("rms_adaln");
  }
  if (!quant && !resid && vec && !LR_K3R_OFF && a.hidden >= 2048 && a.hidden <= 8192 && a.hidden % 8 == 0) {
    // K3 in the 8-column layout, one 128-thread CTA per row
    const int c = (a.hidden + 2047) / 2048;
    const unsigned grid = (unsigned)rows;
#define LR_K3R(CC)                                                                                     \
  if (mod) lr::rms_bf16_row_kernel<CC, true><<<grid, lr::kQ16Threads, 0, s>>>(a);                   \
  else lr::rms_bf16_row_kernel<CC, false><<<grid, lr::kQ16Threads, 0, s>>>(a)
    if (c <= 1) { LR_K3R(1); } else if (c == 2) { LR_K3R(2); } else if (c == 3) { LR_K3R(3); } else { LR_K3R(4); }
#undef LR_K3R
    return lr::launch_status("rms_adaln");
  }
  const int C = pick_chunks(a.hidden);
  if (C < 0) return lr::set_error(LR_ERR_UNSUPPORTED, "rms_adaln: hidden %d > 32768", a.hidden);
// The residual variant (K8) of rows of up to 4 chunks per thread runs two rows
// per CTA (measured faster); every other case the persistent one-row kernel.
// Both reduce each row in the same tree, so their results are identical.
#define LR_RMS(V, R, M, Q)                                                                        \
  if (R && kC <= 4 && !LR_RMS2_OFF)                                                               \
    lr::rms_mod2_kernel<(kC <= 4 ? kC : 4), V, R, M, Q><<<(unsigned)((rows + 1) / 2), lr::kThreads, 0, s>>>(a); \
  else                                                                                            \
    lr::rms_mod_kernel<kC, V, R, M, Q><<<lr::persistent_grid(lr::rms_mod_kernel<kC, V, R, M, Q>, rows, lr::Prefetch<kC>::kOn && !(LR_K3_ONE && !Q)), lr::kThreads, 0, s>>>(a)
#define LR_RMS_Q(V, R, M)  \
  if (quant) { LR_RMS(V, R, M, true); } else { LR_RMS(V, R, M, false); }
#define LR_RMS_M(V, R)     \
  if (mod) { LR_RMS_Q(V, R, true); } else { LR_RMS_Q(V, R, false); }
#define LR_RMS_R(V)        \
  if (resid) { LR_RMS_M(V, true); } else { LR_RMS_M(V, false); }
  LR_CHUNK_DISPATCH(C, {
    if (vec) { LR_RMS_R(true); } else { LR_RMS_R(false); }
  });
#undef LR_RMS_R
#undef LR_RMS_M
#undef LR_RMS_Q
#undef LR_RMS
  return lr::launch_status("rms_adaln");
}

extern "C" int lr_rms_adaln(const void* x, const void* norm_weight, float eps, const void* table,
                            int64_t table_rows, int64_t table_width, const int64_t* indices,
                            int64_t sequence, int64_t rows, int64_t hidden, int shift_slot,
                            int scale_slot, void* out, void* stream) {
  LR_REQUIRE(rows >= 0 && hidden > 0, "rms_adaln: invalid shape");
  if (rows == 0) return LR_OK;
  LR_REQUIRE(x && norm_weight && out, "rms_adaln: null pointer");
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "rms_adaln: too many rows");
  int st = check_table("rms_adaln", table, table_rows, table_width, indices, sequence, hidden,
                       shift_slot, scale_slot, shift_slot);
  if (st) return st;
  lr::RmsArgs a{};
  a.x = static_cast<const bf16*>(x);
  a.weight = static_cast<const bf16*>(norm_weight);
  a.eps = eps;
  a.table = static_cast<const bf16*>(table);
  a.table_rows = table_rows;
  a.table_width = table_width;
  a.indices = indices;
  a.sequence = sequence;
  a.hidden = (int)hidden;
  a.shift_slot = shift_slot;
  a.scale_slot = scale_slot;
  a.out = static_cast<bf16*>(out);
  a.rows = rows;
  const bool vec = vec_ok(hidden, {x, norm_weight, table, out}) && table_width % 8 == 0;
  return rms_launch(a, rows, false, table != nullptr, false, vec, static_cast<cudaStream_t>(stream));
}

extern "C" int lr_rms_adaln_quant_int8(const void* x, const void* norm_weight, float eps,
                                       const void* table, int64_t table_rows, int64_t table_width,
                                       const int64_t* indices, int64_t sequence, int64_t rows,
                                       int64_t hidden, int shift_slot, int scale_slot,
                                       const void* update, int gate_slot, void* residual_out,
                                       int8_t* q, float* scales, void* stream) {
  LR_REQUIRE(rows >= 0 && hidden > 0, "rms_adaln_quant_int8: invalid shape");
  if (rows == 0) return LR_OK;
  LR_REQUIRE(x && norm_weight && q && scales, "rms_adaln_quant_int8: null pointer");
  LR_REQUIRE(update == nullptr || residual_out != nullptr,
             "rms_adaln_quant_int8: residual_out is required with update");
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "rms_adaln_quant_int8: too many rows");
  int st = check_table("rms_adaln_quant_int8", table, table_rows, table_width, indices, sequence,
                       hidden, shift_slot, scale_slot, update ? gate_slot : shift_slot);
  if (st) return st;
  lr::RmsArgs a{};
  a.x = static_cast<const bf16*>(x);
  a.update = static_cast<const bf16*>(update);
  a.weight = static_cast<const bf16*>(norm_weight);
  a.eps = eps;
  a.table = static_cast<const bf16*>(table);
  a.table_rows = table_rows;
  a.table_width = table_width;
  a.indices = indices;
  a.sequence = sequence;
  a.hidden = (int)hidden;
  a.shift_slot = shift_slot;
  a.scale_slot = scale_slot;
  a.gate_slot = gate_slot;
  a.residual_out = static_cast<bf16*>(residual_out);
  a.q = q;
  a.scales = scales;
  a.rows = rows;
  const bool vec = vec_ok(hidden, {x, norm_weight, table, update, residual_out}) &&
                   (table == nullptr || table_width % 8 == 0) && lr::aligned(q, 8);
  return rms_launch(a, rows, update != nullptr, table != nullptr, true, vec,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int lr_gated_residual(const void* x, const void* y, const void* table,
                                 int64_t table_rows, int64_t table_width, const int64_t* indices,
                                 int64_t sequence, int64_t rows, int64_t hidden, int gate_slot,
                                 void* out, void* stream) {
  LR_REQUIRE(rows >= 0 && hidden > 0, "gated_residual: invalid shape");
  if (rows == 0) return LR_OK;
  LR_REQUIRE(x && y && out, "gated_residual: null pointer");
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "gated_residual: too many rows");
  int st = check_table("gated_residual", table, table_rows, table_width, indices, sequence, hidden,
                       gate_slot, gate_slot, gate_slot);
  if (st) return st;
  const int C = pick_chunks(hidden);
  if (C < 0) return lr::set_error(LR_ERR_UNSUPPORTED, "gated_residual: hidden > 32768");
  const bool vec = vec_ok(hidden, {x, y, table, out}) && (table == nullptr || table_width % 8 == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bf16 *xp = static_cast<const bf16*>(x), *yp = static_cast<const bf16*>(y),
             *tp = static_cast<const bf16*>(table);
  bf16* op = static_cast<bf16*>(out);
  LR_CHUNK_DISPATCH(C, {
    if (vec)
      lr::gated_residual_kernel<kC, true><<<lr::persistent_grid(lr::gated_residual_kernel<kC, true>, rows, lr::Prefetch<kC>::kOn && !LR_K5_ONE), lr::kThreads, 0, s>>>(
          xp, yp, tp, table_rows, table_width, indices, sequence, (int)hidden, gate_slot, op, rows);
    else
      lr::gated_residual_kernel<kC, false><<<lr::persistent_grid(lr::gated_residual_kernel<kC, false>, rows, lr::Prefetch<kC>::kOn && !LR_K5_ONE), lr::kThreads, 0, s>>>(
          xp, yp, tp, table_rows, table_width, indices, sequence, (int)hidden, gate_slot, op, rows);
  });
  return lr::launch_status("gated_residual");
}

static int swiglu_common(const char* who, const void* projected, int64_t rows, int64_t inner,
                         void* out, int8_t* q, float* scales, void* stream) {
  LR_REQUIRE(rows >= 0 && inner > 0, "%s: invalid shape", who);
  if (rows == 0) return LR_OK;
  LR_REQUIRE(projected != nullptr, "%s: null pointer", who);
  if (rows > kMaxRows) return lr::set_error(LR_ERR_UNSUPPORTED, "%s: too many rows", who);
  const int C = pick_chunks(inner);
  if (C < 0) return lr::set_error(LR_ERR_UNSUPPORTED, "%s: inner width > 32768", who);
  const bool quant = q != nullptr;
  const bool vec = vec_ok(inner, {projected, out}) && (!quant || lr::aligned(q, 8));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bf16* p = static_cast<const bf16*>(projected);
  bf16* o = static_cast<bf16*>(out);
  LR_CHUNK_DISPATCH(C, {
    if (vec) {
      if (quant) lr::swiglu_kernel<kC, true, true><<<lr::persistent_grid(lr::swiglu_kernel<kC, true, true>, rows, false), lr::kThreads, 0, s>>>(p, (int)inner, o, q, scales, rows);
      else lr::swiglu_kernel<kC, true, false><<<lr::persistent_grid(lr::swiglu_kernel<kC, true, false>, rows, false), lr::kThreads, 0, s>>>(p, (int)inner, o, q, scales, rows);
    } else {
      if (quant) lr::swiglu_kernel<kC, false, true><<<lr::persistent_grid(lr::swiglu_kernel<kC, false, true>, rows, false), lr::kThreads, 0, s>>>(p, (int)inner, o, q, scales, rows);
      else lr::swiglu_kernel<kC, false, false><<<lr::persistent_grid(lr::swiglu_kernel<kC, false, false>, rows, false), lr::kThreads, 0, s>>>(p, (int)inner, o, q, scales, rows);
    }
  });
  return lr::launch_status(who);
}

extern "C" int lr_swiglu(const void* projected, int64_t rows, int64_t inner, void* out,
                         void* stream) {
  if (rows > 0 && out == nullptr) return lr::set_error(LR_ERR_INVALID_ARGUMENT, "swiglu: null output");
  return swiglu_common("swiglu", projected, rows, inner, out, nullptr, nullptr, stream);
}

extern "C" int lr_swiglu_quant_int8(const void* projected, int64_t rows, int64_t inner, int8_t* q,
                                    float* scales, void* stream) {
  if (rows > 0 && (q == nullptr || scales == nullptr))
    return lr::set_error(LR_ERR_INVALID_ARGUMENT, "swiglu_quant_int8: null output");
  return swiglu_common("swiglu_quant_int8", projected, rows, inner, nullptr, q, scales, stream);
}

extern "C" int lr_qk_norm_rope(const void* query, const void* key, int64_t q_token_stride,
                               int64_t q_head_stride, int64_t k_token_stride, int64_t k_head_stride,
                               const void* q_weight, const void* k_weight, const float* cos,
                               const float* sin, int64_t batch, int64_t sequence, int64_t heads,
                               int64_t head_dim, int64_t rotary_dim, float eps, void* q_out,
                               void* k_out, void* stream) {
  LR_REQUIRE(batch >= 0 && sequence >= 0 && heads > 0 && head_dim > 0, "qk_norm_rope: invalid shape");
  LR_REQUIRE(head_dim <= 256, "qk_norm_rope: head_dim %lld > 256", (long long)head_dim);
  LR_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
             "rotary dimensions must be even and fit the attention head");
  const int64_t rows = batch * sequence * heads;
  if (rows == 0) return LR_OK;
  LR_REQUIRE(query && key && q_weight && k_weight && q_out && k_out && (rotary_dim == 0 || (cos && sin)),
             "qk_norm_rope: null pointer");
  int lanes = 1;
  while (lanes * 8 < head_dim) lanes *= 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bf16 *qp = static_cast<const bf16*>(query), *kp = static_cast<const bf16*>(key);
  const bf16 *wq = static_cast<const bf16*>(q_weight), *wk = static_cast<const bf16*>(k_weight);
  bf16 *qo = static_cast<bf16*>(q_out), *ko = static_cast<bf16*>(k_out);
  const int64_t qc = heads * head_dim / 8;  // 16-byte chunks of one token's Q heads
  const int64_t ni = (2 * qc + 255) / 256;
  const bool rot_ok = rotary_dim == 0 || (rotary_dim % 16 == 0 && ((rotary_dim / 16) & (rotary_dim / 16 - 1)) == 0);
  const bool fast = lanes * 8 == head_dim && q_head_stride == head_dim && k_head_stride == head_dim && rot_ok &&
                    ni <= 16 && (q_token_stride * 2) % 16 == 0 && (k_token_stride * 2) % 16 == 0 &&
                    lr::aligned(query, 16) && lr::aligned(key, 16) && lr::aligned(q_weight, 16) &&
                    lr::aligned(k_weight, 16) && lr::aligned(q_out, 16) && lr::aligned(k_out, 16) &&
                    (rotary_dim == 0 || (lr::aligned(cos, 16) && lr::aligned(sin, 16)));
  if (fast) {
    const unsigned grid = (unsigned)(batch * sequence);
#define LR_QK(NN)                                                                                      \
  lr::qk_norm_rope_tok_kernel<NN><<<grid, 256, 0, s>>>(qp, kp, q_token_stride, k_token_stride, wq, wk, cos, \
                                                       sin, sequence, (int)qc, lanes, (int)head_dim,        \
                                                       (int)rotary_dim, eps, qo, ko)
    if (ni <= 1) LR_QK(1);
    else if (ni <= 2) LR_QK(2);
    else if (ni <= 3) LR_QK(3);
    else if (ni <= 4) LR_QK(4);
    else if (ni <= 6) LR_QK(6);
    else if (ni <= 8) LR_QK(8);
    else if (ni <= 12) LR_QK(12);
    else LR_QK(16);
#undef LR_QK
  } else {
    const int64_t ctas = (rows + 7) / 8;
    const int64_t cap = 8ll * lr::sm_count();
    lr::qk_norm_rope_row_kernel<<<(unsigned)(ctas < cap ? ctas : cap), 256, 0, s>>>(
        qp, kp, q_token_stride, q_head_stride, k_token_stride, k_head_stride, wq, wk, cos, sin, rows, sequence,
        (int)heads, (int)head_dim, lanes, (int)rotary_dim, eps, qo, ko);
  }
  return lr::launch_status("qk_norm_rope");
}
