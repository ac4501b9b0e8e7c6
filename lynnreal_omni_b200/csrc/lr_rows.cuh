// Row-kernel helpers shared by the row kernels' translation units: chunked
// 16-byte loads/stores of bf16 rows, int8 chunk stores, the adaLN table lookup
// and the argument block of the RMSNorm kernels. A translation unit includes
// this after defining `flag_error(unsigned)` (its device status word).
#pragma once

#include "lr_common.cuh"

namespace lr {
namespace rows {

using bf16 = __nv_bfloat16;

// Load the 8-column chunk starting at `col` of a row (zeros past `width`).
// VEC: the chunk is 16-byte aligned and either fully inside or fully outside.
template <bool VEC, bool STREAM>
__device__ __forceinline__ uint4 load_chunk(const bf16* row, int64_t col, int64_t width) {
  if (VEC) {
    if (col < width) return STREAM ? ld_stream(row + col) : ld_keep(row + col);
    return make_uint4(0u, 0u, 0u, 0u);
  } else {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(row);
    uint32_t h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = (col + e < width) ? p[col + e] : 0u;
    return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                      h[6] | (h[7] << 16));
  }
}

template <bool VEC>
__device__ __forceinline__ void store_chunk(bf16* row, int64_t col, int64_t width, const uint4& v) {
  if (VEC) {
    if (col < width) *reinterpret_cast<uint4*>(row + col) = v;
  } else {
    uint16_t* p = reinterpret_cast<uint16_t*>(row);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (col + e < width) p[col + e] = (uint16_t)(w[e >> 1] >> ((e & 1) * 16));
  }
}

// Store eight int8 values (packed in a uint2) at q[col..col+7].
template <bool VEC>
__device__ __forceinline__ void store_q8(int8_t* q, int64_t col, int64_t width, const uint2& w) {
  if (VEC) {
    if (col < width) *reinterpret_cast<uint2*>(q + col) = w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (col + e < width) q[col + e] = (int8_t)((e < 4 ? w.x : w.y) >> (8 * (e & 3)));
  }
}

__device__ __forceinline__ uint4 splat8(uint32_t w) { return make_uint4(w, w, w, w); }

struct RmsArgs {
  const bf16* x;
  const bf16* update;  // K8 residual branch (may be null)
  const bf16* weight;
  float eps;
  const bf16* table;  // may be null: no modulation, gate 1
  int64_t table_rows, table_width;
  const int64_t* indices;
  int64_t sequence;
  int hidden;
  int shift_slot, scale_slot, gate_slot;
  bf16* residual_out;
  int8_t* q;
  float* scales;
  bf16* out;
  int64_t rows;
};

// Resolve the adaLN table row of flattened row `row`; null if the table is
// absent, or (with the status bit raised) if the index is out of range.
__device__ __forceinline__ const bf16* table_row_ptr(const bf16* table, int64_t table_rows,
                                                     int64_t table_width, const int64_t* indices,
                                                     int64_t sequence, int64_t row, bool& bad) {
  bad = false;
  if (table == nullptr) return nullptr;
  // row % sequence without the 64-bit division routine in the common cases
  // (one batch: row < sequence; both below 2^31: a 32-bit remainder)
  const int64_t pos = row < sequence ? row
                      : ((row | sequence) >> 31) == 0 ? (int64_t)((uint32_t)row % (uint32_t)sequence)
                                                      : row % sequence;
  const int64_t tr = indices[pos];
  if (tr < 0 || tr >= table_rows) {
    bad = true;
    return nullptr;
  }
  return table + tr * table_width;
}

}  // namespace rows
}  // namespace lr
