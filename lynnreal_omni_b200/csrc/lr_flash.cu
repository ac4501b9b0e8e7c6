// Flash token compression (model/flash.py) on sm_100a:
//   * gather_rows_kernel   — the index_select of the compressed blocks' inputs
//                            (hidden rows, adaLN indices, rotary rows, mask
//                            columns; model/flash.py:71-79);
//   * restore_kernel       — the residual restore before the first suffix
//                            block, fused into one pass (model/flash.py:81-84):
//                              out[b,t] = bf16(full[b,t] + bf16(bf16(x[b,k] - in[b,k]) * gain)),
//                              k = inverse[t];
//   * nearest_anchor_kernel — the dropped-row -> same-time anchor search of
//                            spatial_layout (model/flash.py:27-32).
// All three are HBM- or latency-bound index work: one warp per output row,
// 16-byte vector accesses, a grid of a few CTAs per SM striding over rows.
#include <mutex>

#include "lr_common.cuh"
#include "lr_host.h"

namespace lr {

static __device__ unsigned int g_flash_status = 0;

namespace {

using bf16 = __nv_bfloat16;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void flag_flash(unsigned int bits) { atomicOr(&g_flash_status, bits); }

unsigned grid_for(int64_t warps_needed, int ctas_per_sm) {
  const int64_t ctas = (warps_needed + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)ctas_per_sm * sm_count();
  return (unsigned)(ctas < cap ? (ctas > 0 ? ctas : 1) : cap);
}

// ------------------------------------------------------------------ gather
// out[o, i, :] = src[o, index[i], :] for o < outer, i < n_index; a row is
// `vecs` elements of type V. Wide rows: one warp per output row, U vectors per
// lane in flight. Narrow rows (fewer than 32 vectors): one thread per vector.
template <typename V, int U, bool WIDE>
__global__ void __launch_bounds__(kThreads) gather_rows_kernel(const char* __restrict__ src,
                                                               int64_t src_outer_stride, int64_t src_rows,
                                                               int64_t vecs, const int64_t* __restrict__ index,
                                                               int64_t n_index, char* __restrict__ out,
                                                               int64_t out_outer_stride, int64_t total_rows) {
  if (WIDE) {
    const int lane = threadIdx.x & 31;
    const int64_t step = (int64_t)gridDim.x * kWarps;
    for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < total_rows; r += step) {
      const int64_t o = r / n_index, i = r - o * n_index;
      const int64_t s = index[i];
      V* dst = reinterpret_cast<V*>(out + o * out_outer_stride) + i * vecs;
      const bool ok = s >= 0 && s < src_rows;
      if (!ok && lane == 0) flag_flash(kDevErrRowIndex);
      const V* row = reinterpret_cast<const V*>(src + o * src_outer_stride) + (ok ? s : 0) * vecs;
      for (int64_t j = lane; j < vecs; j += 32 * U) {
        V buf[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = j + 32 * u;
          if (c < vecs) buf[u] = ok ? row[c] : V{};
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = j + 32 * u;
          if (c < vecs) dst[c] = buf[u];
        }
      }
    }
  } else {
    const int64_t total = total_rows * vecs;
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t g = (int64_t)blockIdx.x * kThreads + threadIdx.x; g < total; g += step) {
      const int64_t r = g / vecs, c = g - r * vecs;
      const int64_t o = r / n_index, i = r - o * n_index;
      const int64_t s = index[i];
      const bool ok = s >= 0 && s < src_rows;
      if (!ok) flag_flash(kDevErrRowIndex);
      reinterpret_cast<V*>(out + o * out_outer_stride)[i * vecs + c] =
          ok ? reinterpret_cast<const V*>(src + o * src_outer_stride)[s * vecs + c] : V{};
    }
  }
}

struct alignas(16) Vec16 { uint4 v; };
struct alignas(8) Vec8 { uint2 v; };

template <typename V>
int launch_gather(const void* src, int64_t outer, int64_t src_outer_stride, int64_t src_rows,
                  int64_t row_bytes, const int64_t* index, int64_t n_index, void* out,
                  int64_t out_outer_stride, cudaStream_t s) {
  const int64_t vecs = row_bytes / (int64_t)sizeof(V);
  const int64_t rows = outer * n_index;
  const char* sp = static_cast<const char*>(src);
  char* op = static_cast<char*>(out);
  if (vecs >= 32) {
    gather_rows_kernel<V, 4, true><<<grid_for(rows, 8), kThreads, 0, s>>>(
        sp, src_outer_stride, src_rows, vecs, index, n_index, op, out_outer_stride, rows);
  } else {
    gather_rows_kernel<V, 1, false><<<grid_for((rows * vecs + 31) / 32, 8), kThreads, 0, s>>>(
        sp, src_outer_stride, src_rows, vecs, index, n_index, op, out_outer_stride, rows);
  }
  return launch_status("gather_rows");
}

// ----------------------------------------------------------------- restore
__device__ __forceinline__ uint32_t bneg2(uint32_t a) { return a ^ 0x80008000u; }

// bf16(bf16(c - i) * gain) + full, on 8 packed values. c - i and the final sum
// are single bf16 roundings of exact fp32 results (packed add.rn.bf16x2 of a
// negated operand); the gain product is fp32 then rounded, like the
// reference's bf16-tensor-times-Python-float multiply. gain == 1 is exact and
// skipped.
template <bool UNIT>
__device__ __forceinline__ uint4 restore8(const uint4& f, const uint4& c, const uint4& i, float gain) {
  uint4 d = make_uint4(badd2(c.x, bneg2(i.x)), badd2(c.y, bneg2(i.y)), badd2(c.z, bneg2(i.z)),
                       badd2(c.w, bneg2(i.w)));
  if (!UNIT) {
    float v[8];
    unpack8(d, v);
    const float2 g2 = make_float2(gain, gain);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 p = __fmul2_rn(make_float2(v[e], v[e + 1]), g2);
      v[e] = p.x;
      v[e + 1] = p.y;
    }
    d = pack8(v);
  }
  return badd8(f, d);
}

__device__ __forceinline__ float restore1(float f, float c, float i, float gain, bool unit) {
  float d = bf16r(__fsub_rn(c, i));
  if (!unit) d = bf16r(__fmul_rn(d, gain));
  return bf16r(__fadd_rn(f, d));
}

// One warp per (batch, sequence) row. VEC: hidden % 8 == 0 and 16-byte aligned
// rows; otherwise one element per lane step.
template <bool VEC, bool UNIT, int U>
__global__ void __launch_bounds__(kThreads) restore_kernel(const bf16* __restrict__ full,
                                                           const bf16* __restrict__ comp,
                                                           const bf16* __restrict__ input,
                                                           const int64_t* __restrict__ inverse, int64_t batch,
                                                           int64_t rows, int64_t kept, int64_t hidden, float gain,
                                                           bf16* out) {
  const int lane = threadIdx.x & 31;
  const int64_t total = batch * rows;
  const int64_t step = (int64_t)gridDim.x * kWarps;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < total; r += step) {
    const int64_t b = r / rows, t = r - b * rows;
    const int64_t k = inverse[t];
    const bool ok = k >= 0 && k < kept;
    if (!ok && lane == 0) flag_flash(kDevErrRowIndex);
    const int64_t src = (b * kept + (ok ? k : 0)) * hidden;
    const int64_t dst = r * hidden;
    if (VEC) {
      const int64_t chunks = hidden / 8;
      const uint4* fp = reinterpret_cast<const uint4*>(full + dst);
      const uint4* cp = reinterpret_cast<const uint4*>(comp + src);
      const uint4* ip = reinterpret_cast<const uint4*>(input + src);
      uint4* op = reinterpret_cast<uint4*>(out + dst);
      for (int64_t j = lane; j < chunks; j += 32 * U) {
        uint4 f[U], c[U], in[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t q = j + 32 * u;
          if (q < chunks) {
            f[u] = __ldcs(fp + q);
            c[u] = ok ? __ldg(cp + q) : make_uint4(0u, 0u, 0u, 0u);
            in[u] = ok ? __ldg(ip + q) : make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t q = j + 32 * u;
          if (q < chunks) __stcs(op + q, restore8<UNIT>(f[u], c[u], in[u], gain));
        }
      }
    } else {
      const uint16_t* fp = reinterpret_cast<const uint16_t*>(full) + dst;
      const uint16_t* cp = reinterpret_cast<const uint16_t*>(comp) + src;
      const uint16_t* ip = reinterpret_cast<const uint16_t*>(input) + src;
      uint16_t* op = reinterpret_cast<uint16_t*>(out) + dst;
      for (int64_t j = lane; j < hidden; j += 32) {
        const float c = ok ? bf_bits(cp[j]) : 0.0f, in = ok ? bf_bits(ip[j]) : 0.0f;
        op[j] = f2bf_bits(restore1(bf_bits(fp[j]), c, in, gain, UNIT));
      }
    }
  }
}

// ---------------------------------------------------------- nearest anchor
// For dropped row src: among anchors a with positions[a,0] == positions[src,0],
// the one with the smallest Euclidean distance over axes 1-2, ties to the
// lowest anchor position in `anchors`; no same-time anchor -> anchor 0 (the
// argmin of an all-infinite row). The distance is compared as the fp32
// square root of the squared distance (computed exactly in fp64, rounded to
// fp32): equal to the reference's fp32 cdist wherever that is exact (integer
// coordinates below 2^11), including the ties its rounding creates.
// inverse[src] = inverse[anchors[best]].
__global__ void __launch_bounds__(kThreads) nearest_anchor_kernel(const float* __restrict__ pos,
                                                                  const int64_t* __restrict__ dropped,
                                                                  int64_t n_dropped,
                                                                  const int64_t* __restrict__ anchors,
                                                                  int64_t n_anchors, int64_t* inverse) {
  const int lane = threadIdx.x & 31;
  const int64_t step = (int64_t)gridDim.x * kWarps;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < n_dropped; r += step) {
    const int64_t src = dropped[r];
    const float t0 = pos[src * 3], h0 = pos[src * 3 + 1], w0 = pos[src * 3 + 2];
    float best = __int_as_float(0x7f800000);  // +inf
    int64_t bj = n_anchors;                    // none finite yet
    for (int64_t j = lane; j < n_anchors; j += 32) {
      const int64_t a = anchors[j];
      if (pos[a * 3] != t0) continue;
      const double dh = __dsub_rn((double)h0, (double)pos[a * 3 + 1]);
      const double dw = __dsub_rn((double)w0, (double)pos[a * 3 + 2]);
      const float d = __fsqrt_rn(__double2float_rn(__dadd_rn(__dmul_rn(dh, dh), __dmul_rn(dw, dw))));
      if (d < best) {  // strict: the first (lowest j) of equal distances stays
        best = d;
        bj = j;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int64_t oj = __shfl_xor_sync(0xffffffffu, bj, off);
      if (ob < best || (ob == best && oj < bj)) {
        best = ob;
        bj = oj;
      }
    }
    if (lane == 0) {
      if (bj >= n_anchors) bj = 0;
      inverse[src] = inverse[anchors[bj]];
    }
  }
}

}  // namespace

int read_status_flash(unsigned int* bits, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_flash_status, sizeof(v)) != cudaSuccess)
    return launch_status("reading the device status");
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_flash_status, &zero, sizeof(zero)) != cudaSuccess)
      return launch_status("clearing the device status");
  }
  *bits |= v;
  return LR_OK;
}

}  // namespace lr

extern "C" int lr_gather_rows(const void* src, int64_t outer, int64_t src_outer_stride, int64_t src_rows,
                              int64_t row_bytes, const int64_t* index, int64_t n_index, void* out,
                              int64_t out_outer_stride, void* stream) {
  LR_REQUIRE(outer >= 0 && src_rows >= 0 && n_index >= 0 && row_bytes >= 0,
             "gather_rows: negative size");
  if (outer == 0 || n_index == 0 || row_bytes == 0) return LR_OK;
  LR_REQUIRE(src != nullptr && index != nullptr && out != nullptr, "gather_rows: null pointer");
  LR_REQUIRE(src_rows > 0, "gather_rows: index into an empty dimension");
  LR_REQUIRE(src_outer_stride >= src_rows * row_bytes && out_outer_stride >= n_index * row_bytes,
             "gather_rows: outer strides overlap rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto fits = [&](uintptr_t v) {
    return row_bytes % (int64_t)v == 0 && src_outer_stride % (int64_t)v == 0 &&
           out_outer_stride % (int64_t)v == 0 && lr::aligned(src, v) && lr::aligned(out, v);
  };
  if (fits(16))
    return lr::launch_gather<lr::Vec16>(src, outer, src_outer_stride, src_rows, row_bytes, index, n_index, out,
                                        out_outer_stride, s);
  if (fits(8))
    return lr::launch_gather<lr::Vec8>(src, outer, src_outer_stride, src_rows, row_bytes, index, n_index, out,
                                       out_outer_stride, s);
  if (fits(4))
    return lr::launch_gather<uint32_t>(src, outer, src_outer_stride, src_rows, row_bytes, index, n_index, out,
                                       out_outer_stride, s);
  if (fits(2))
    return lr::launch_gather<uint16_t>(src, outer, src_outer_stride, src_rows, row_bytes, index, n_index, out,
                                       out_outer_stride, s);
  return lr::launch_gather<uint8_t>(src, outer, src_outer_stride, src_rows, row_bytes, index, n_index, out,
                                    out_outer_stride, s);
}

extern "C" int lr_flash_restore(const void* full, const void* compressed, const void* input,
                                const int64_t* inverse, int64_t batch, int64_t sequence, int64_t kept,
                                int64_t hidden, float gain, void* out, void* stream) {
  LR_REQUIRE(batch >= 0 && sequence >= 0 && kept >= 0 && hidden >= 0, "flash_restore: negative size");
  if (batch == 0 || sequence == 0 || hidden == 0) return LR_OK;
  LR_REQUIRE(full && compressed && input && inverse && out, "flash_restore: null pointer");
  LR_REQUIRE(kept > 0, "flash_restore: empty compressed sequence");
  using lr::bf16;
  const bf16* f = static_cast<const bf16*>(full);
  const bf16* c = static_cast<const bf16*>(compressed);
  const bf16* i = static_cast<const bf16*>(input);
  bf16* o = static_cast<bf16*>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = hidden % 8 == 0 && lr::aligned(full, 16) && lr::aligned(compressed, 16) &&
                   lr::aligned(input, 16) && lr::aligned(out, 16);
  const bool unit = gain == 1.0f;
  const unsigned grid = lr::grid_for(batch * sequence, 8);
#define LR_RESTORE(V, UN) \
  lr::restore_kernel<V, UN, 2><<<grid, lr::kThreads, 0, s>>>(f, c, i, inverse, batch, sequence, kept, hidden, gain, o)
  if (vec && unit) LR_RESTORE(true, true);
  else if (vec) LR_RESTORE(true, false);
  else if (unit) LR_RESTORE(false, true);
  else LR_RESTORE(false, false);
#undef LR_RESTORE
  return lr::launch_status("flash_restore");
}

extern "C" int lr_flash_nearest_anchor(const float* positions, int64_t sequence, const int64_t* dropped,
                                       int64_t n_dropped, const int64_t* anchors, int64_t n_anchors,
                                       int64_t* inverse, void* stream) {
  LR_REQUIRE(sequence >= 0 && n_dropped >= 0 && n_anchors >= 0, "flash_nearest_anchor: negative size");
  if (n_dropped == 0) return LR_OK;
  LR_REQUIRE(n_anchors > 0, "flash_nearest_anchor: dropped rows but no anchors");
  LR_REQUIRE(positions && dropped && anchors && inverse, "flash_nearest_anchor: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  lr::nearest_anchor_kernel<<<lr::grid_for(n_dropped, 8), lr::kThreads, 0, s>>>(positions, dropped, n_dropped,
                                                                                anchors, n_anchors, inverse);
  return lr::launch_status("flash_nearest_anchor");
}
