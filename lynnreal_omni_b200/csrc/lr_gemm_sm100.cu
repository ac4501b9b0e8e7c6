// INT8 GEMM with int32 accumulation and a fused bf16 epilogue on sm_100a.
//
// Tensor-core path (K10 of the reference, model/int8_gemm.py:13-46, rebuilt
// for Blackwell rather than translated):
//   * persistent kernel, one CTA per SM, grouped-M tile raster;
//   * 128x256 output tiles, K staged 128 bytes at a time through a 4-deep
//     shared-memory ring filled by TMA (128-byte swizzle, zero fill past the
//     matrix edges — this is how ragged M/N/K tails are handled);
//   * warp 0 issues TMA, one thread of warp 1 issues tcgen05.mma.kind::i8
//     (M=128, N=256, K=32 per instruction) into a TMEM int32 accumulator;
//   * two accumulators (2 x 256 TMEM columns) so warps 2-5 run the epilogue of
//     tile i (tcgen05.ld -> fp32 scale/bias/GELU/gated residual -> bf16 stores)
//     while the tensor core computes tile i+1;
//   * every mbarrier wait is bounded (globaltimer); on timeout the kernel raises
//     a device status bit, drains its own copies and MMAs, frees TMEM, returns.
// No TMA multicast is used anywhere (the kernel may run on any GPU of a node).
//
// CUDA-core path: a shared-memory tiled kernel for operand layouts TMA cannot
// address (non-K-major weights, unaligned strides). Integer accumulation is
// exact in any order, so both paths produce identical bits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "lr_common.cuh"
#include "lr_host.h"

// Compile-time tuning knobs of the pair kernel (defaults are the measured best).
#ifndef LR_GEMM_STAGES2
#define LR_GEMM_STAGES2 6
#endif
#ifndef LR_GEMM_L2_HINTS  // 0: default policy; 1: A panel evict-last; 2: also B evict-first
#define LR_GEMM_L2_HINTS 1
#endif
#ifndef LR_GEMM_STREAM_STORES  // 1: evict-first (st.global.cs) output stores
#define LR_GEMM_STREAM_STORES 0
#endif
#ifndef LR_GEMM_TMA_OUT  // 1: the pair kernel stores bf16 outputs with bulk tensor stores
#define LR_GEMM_TMA_OUT 1
#endif
#ifndef LR_GEMM_OUT_EVICT_FIRST  // L2 policy of those stores: 1 evict-first, 0 normal
#define LR_GEMM_OUT_EVICT_FIRST 1
#endif

namespace lr {

static __device__ unsigned int g_gemm_status = 0;
// Limit of every mbarrier wait of the tensor-core kernels (lr_gemm_test_wait
// shortens it) and a one-shot request to drop one TMA load (tests of the
// bounded waits; see lr_gemm_test_wait).
static __device__ unsigned long long g_gemm_wait_limit_ns = 2000000000ull;
static __device__ unsigned int g_gemm_drop_load = 0;

namespace gemm {

using bf16 = __nv_bfloat16;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes of K per stage (= int8 elements)
constexpr int UK = 32;   // K per tcgen05.mma.kind::i8
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;
constexpr int B_STAGE = BN * BK;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512
constexpr int NUM_EPI_WARPS = 4;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int BAR_BYTES = 256;
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * (A_STAGE + B_STAGE) + BAR_BYTES;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s, the default wait limit

// kS32: store raw int32 accumulators ([M, N], row stride N); kS32Part: store a
// K slice's partial accumulators into its own [M, N] plane of the split-K
// workspace (plane = work item's slice).
enum Epi : int { kNone = 0, kGelu = 1, kGated = 2, kS32 = 3, kS32Part = 4 };

struct EpiArgs {
  const float* row_scale;
  const float* col_scale;
  const bf16* bias;
  bf16* out;
  int64_t ldo;
  const bf16* resid;
  int64_t ldr;
  const bf16* table;
  int64_t table_rows, table_width;
  const int64_t* indices;
  int64_t sequence;
  int gate_slot;
  int32_t* acc_out;  // kS32: row stride N
};

// ------------------------------------------------------------ epilogue math
__device__ __forceinline__ float dequant(int32_t acc, float rs, float cs) {
  // (float(acc) * row_scale) * col_scale   (model/int8_gemm.py:41-42,89)
  return __fmul_rn(__fmul_rn(__int2float_rn(acc), rs), cs);
}

// tanh-approximated GELU of a bf16 value, evaluated in fp32:
//   0.5 * x * (1 + tanh(u)),  u = sqrt(2/pi) * (x + 0.044715 * x^3),
// computed as the identical x / (1 + exp(-2u)), which needs one exponential
// and no cancellation in the negative tail (where 1 + tanh(u) loses all its
// significant bits).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float kTwoBeta = 1.5957691216057308f;  // 2 * sqrt(2/pi)
  const float kKappa = 0.044715f;
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float two_u = __fmul_rn(kTwoBeta, __fadd_rn(x, __fmul_rn(kKappa, x3)));
  return __fdividef(x, __fadd_rn(1.0f, __expf(-two_u)));
}

// The same for two values with packed fp32 arithmetic (each lane rounds
// exactly as the scalar form does, so the results are identical).
__device__ __forceinline__ float2 gelu_tanh2(float2 x) {
  const float2 beta2 = make_float2(1.5957691216057308f, 1.5957691216057308f);
  const float2 kappa = make_float2(0.044715f, 0.044715f);
  const float2 x3 = __fmul2_rn(__fmul2_rn(x, x), x);
  const float2 two_u = __fmul2_rn(beta2, __fadd2_rn(x, __fmul2_rn(kappa, x3)));
  const float2 den = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(__expf(-two_u.x), __expf(-two_u.y)));
  return make_float2(__fdividef(x.x, den.x), __fdividef(x.y, den.y));
}

// Final bf16 value of one output element. `d` already holds the dequantised
// fp32 value including bias; `resid`/`gate` are used by kGated only.
template <int EPI>
__device__ __forceinline__ float finish(float d, float resid, float gate) {
  if (EPI == kGelu) return gelu_tanh(bf16r(d));
  if (EPI == kGated) return __fadd_rn(resid, bf16r(__fmul_rn(gate, bf16r(d))));
  return d;
}

__device__ __forceinline__ const bf16* gate_row(const EpiArgs& ep, int64_t row, bool& bad) {
  bad = false;
  if (ep.table == nullptr) return nullptr;
  const int64_t tr = ep.indices[row % ep.sequence];
  if (tr < 0 || tr >= ep.table_rows) {
    bad = true;
    return nullptr;
  }
  return ep.table + tr * ep.table_width;  // the caller adds the gate slot offset
}

// ------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Arrive on the mbarrier at the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(bar), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of `bar` with parity `parity` to complete. Gives up when
// another role has aborted, or after kWaitLimitNs (raising the status bit).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity,
                                             volatile uint32_t* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  const unsigned long long limit = g_gemm_wait_limit_ns;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1u;
      atomicOr(&g_gemm_status, (unsigned)kDevErrWaitTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields: start address>>4 [0,14), leading byte offset>>4 [16,30) (unused
// for swizzled K-major, 1), stride byte offset>>4 [32,46), descriptor version
// 1 at [46,48), swizzle mode 2 (128B) at [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) |
         ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor for kind::i8: s32 accumulator [4,6)=2, signed A
// [7,10)=1, signed B [10,13)=1, both K-major, N>>3 at [17,23), M>>4 at [24,29).
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Load 32 consecutive int32 TMEM columns of this thread's lane and wait for
// them in the same asm block, so no consumer can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// ------------------------------------------------ CTA-pair (cta_group::2) PTX
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  return remote;
}
// All threads of both CTAs; orders shared-memory writes (barrier init, TMEM
// address) before any peer access, and keeps a CTA's shared memory alive
// until its peer no longer reads it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_bounded_cluster(uint32_t bar, uint32_t parity,
                                                     volatile uint32_t* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  const unsigned long long limit = g_gemm_wait_limit_ns;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1u;
      atomicOr(&g_gemm_status, (unsigned)kDevErrWaitTimeout);
      return false;
    }
  }
}
// TMA load into this CTA's shared memory whose completion is signalled on an
// mbarrier of either CTA of the pair (`bar` is a shared::cluster address).
// No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// L2 eviction policies for the operand streams (LR_GEMM_L2_HINTS): the A panel
// of a raster group is re-read for every N block.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Instruction descriptor of the pair MMA: M = 256 (128 rows per CTA), N = 256.
constexpr uint32_t kIdescPair = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)(256 >> 4) << 24);
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdescPair), "r"(accumulate)
      : "memory");
}
// Arrive (once the pair's prior MMAs complete) on the mbarrier at offset `bar`
// in every CTA of `cta_mask`.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// Grouped raster: `group` consecutive M-blocks are swept across all N-blocks
// before the next group starts, so the group's A panel stays L2-resident while
// B streams through once per group.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group, int& mb,
                                            int& nb) {
  const int span = group * num_n;
  const int g = t / span;
  const int first = g * group;
  const int gsize = min(num_m - first, group);
  const int r = t - g * span;
  mb = first + r % gsize;
  nb = r / gsize;
}

// Epilogue of one W-column chunk of one row (W a multiple of 8), vectorised
// (all W columns valid).
template <int EPI, int W = 32>
__device__ __forceinline__ void chunk_values(const EpiArgs& ep, const uint32_t (&acc)[W], int64_t row,
                                             int col0, float rs, const bf16* gate_ptr, bool have_gate,
                                             const uint4* resid_pre, uint4 (&out)[W / 8]) {
  static_assert(W % 8 == 0, "chunk width");
  const float4* cs4 = reinterpret_cast<const float4*>(ep.col_scale + col0);
  float d[W];
  const float2 rs2 = make_float2(rs, rs);
#pragma unroll
  for (int q = 0; q < W / 4; ++q) {
    // (float(acc) * row_scale) * col_scale, two columns per packed multiply
    // (each lane rounds as dequant() does)
    const float4 c = __ldg(cs4 + q);
    const float2 lo = __fmul2_rn(__fmul2_rn(make_float2(__int2float_rn((int32_t)acc[4 * q + 0]),
                                                        __int2float_rn((int32_t)acc[4 * q + 1])), rs2),
                                 make_float2(c.x, c.y));
    const float2 hi = __fmul2_rn(__fmul2_rn(make_float2(__int2float_rn((int32_t)acc[4 * q + 2]),
                                                        __int2float_rn((int32_t)acc[4 * q + 3])), rs2),
                                 make_float2(c.z, c.w));
    d[4 * q + 0] = lo.x;
    d[4 * q + 1] = lo.y;
    d[4 * q + 2] = hi.x;
    d[4 * q + 3] = hi.y;
  }
  if (ep.bias != nullptr) {
    const uint4* b4 = reinterpret_cast<const uint4*>(ep.bias + col0);
#pragma unroll
    for (int q = 0; q < W / 8; ++q) {
      float b[8];
      unpack8(__ldg(b4 + q), b);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 s2 = __fadd2_rn(make_float2(d[8 * q + e], d[8 * q + e + 1]), make_float2(b[e], b[e + 1]));
        d[8 * q + e] = s2.x;
        d[8 * q + e + 1] = s2.y;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < W / 8; ++q) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = d[8 * q + e];
    uint4 y = pack8(o);  // bf16(dequant)
    if (EPI == kGelu) {
      unpack8(y, o);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 g2 = gelu_tanh2(make_float2(o[e], o[e + 1]));
        o[e] = g2.x;
        o[e + 1] = g2.y;
      }
      y = pack8(o);
    } else if (EPI == kGated) {
      // bf16(x + bf16(gate * bf16(dequant)))   (model/kernels.py:146-153)
      const uint4 x = resid_pre != nullptr ? resid_pre[q]
                                            : *reinterpret_cast<const uint4*>(ep.resid + row * ep.ldr + col0 + 8 * q);
      const uint32_t gd = (ep.table == nullptr) ? kBf2One : 0u;
      const uint4 g = have_gate ? __ldg(reinterpret_cast<const uint4*>(gate_ptr + col0 + 8 * q))
                                : make_uint4(gd, gd, gd, gd);
      y = badd8(x, bmul8(g, y));
    }
    out[q] = y;
  }
}

template <int EPI, int W = 32>
__device__ __forceinline__ void store_chunk_vec(const EpiArgs& ep, const uint32_t (&acc)[W],
                                                int64_t row, int col0, float rs,
                                                const bf16* gate_ptr, bool have_gate,
                                                const uint4* resid_pre = nullptr) {
  uint4 y[W / 8];
  chunk_values<EPI, W>(ep, acc, row, col0, rs, gate_ptr, have_gate, resid_pre, y);
  uint4* dst = reinterpret_cast<uint4*>(ep.out + row * ep.ldo + col0);
#pragma unroll
  for (int q = 0; q < W / 8; ++q) {
    if (LR_GEMM_STREAM_STORES)
      __stcs(dst + q, y[q]);  // evict-first output stores
    else
      dst[q] = y[q];
  }
}

// Same, with per-column bounds (ragged N tail) and scalar accesses.
template <int EPI>
__device__ __forceinline__ void store_chunk_tail(const EpiArgs& ep, const uint32_t (&acc)[32],
                                                 int64_t row, int col0, int N, float rs,
                                                 const bf16* gate_ptr, bool have_gate) {
  const uint16_t* bias = reinterpret_cast<const uint16_t*>(ep.bias);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int col = col0 + j;
    if (col >= N) break;
    if (EPI == kS32 || EPI == kS32Part) {
      ep.acc_out[row * (int64_t)N + col] = (int32_t)acc[j];
      continue;
    }

    float d = dequant((int32_t)acc[j], rs, ep.col_scale[col]);
    if (bias != nullptr) d = __fadd_rn(d, bf_bits(bias[col]));
    float x = 0.0f, g = 0.0f;
    if (EPI == kGated) {
      x = bf_bits(reinterpret_cast<const uint16_t*>(ep.resid)[row * ep.ldr + col]);
      g = have_gate ? bf_bits(reinterpret_cast<const uint16_t*>(gate_ptr)[col])
                    : ((ep.table == nullptr) ? 1.0f : 0.0f);
    }
    reinterpret_cast<uint16_t*>(ep.out)[row * ep.ldo + col] = f2bf_bits(finish<EPI>(d, x, g));
  }
}

// ------------------------------------------------- TMA-store epilogue
// Output destinations of the bulk-tensor-store epilogue: bf16 matrices of M
// rows x N columns (each map's base is already offset to the GEMM's first
// row), box 32 columns x 32 rows, 64-byte swizzle. One destination is the
// plain output; several are the same rows in every rank's copy of a gathered
// tensor (peer memory mapped over NVLink), so the epilogue is also the
// all-gather. Plain TMA stores, no multicast.
constexpr int kMaxDst = 8;
struct OutMaps {
  CUtensorMap map[kMaxDst];
  int count;
};
constexpr int kOutChunk = 32 * 32 * 2;               // one warp's 32 rows x 32 columns of bf16
constexpr int kOutStage = NUM_EPI_WARPS * 2 * kOutChunk;  // double-buffered per epilogue warp

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y,
                                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most one committed group still reads shared memory
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// wait until every committed group has completed its writes
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Drain one accumulator as drain_accumulator does, but store each 32-column
// chunk through shared memory with bulk tensor stores: the 32 lanes write
// their rows into this warp's staging buffer (64-byte swizzle, so the 16-byte
// writes are bank-conflict free), then lane 0 stores the 32 x 32 box to every
// destination. Rows past M are clipped by the tensor maps. Requires N a
// multiple of 32. `chunk` counts this warp's chunks (staging buffer parity).
template <int EPI>
__device__ __forceinline__ void drain_accumulator_tma(const EpiArgs& ep, const OutMaps& outs, int M, int N,
                                                      uint32_t tbase, int64_t row0, int col_base, int lane,
                                                      uint32_t release_bar, uint8_t* staging, uint32_t& chunk,
                                                      uint64_t policy) {
  const int64_t row = row0 + lane;
  const bool row_ok = row < M;
  float rs = 0.0f;
  const bf16* gptr = nullptr;
  bool have_gate = false;
  if (row_ok) {
    rs = ep.row_scale[row];
    if (EPI == kGated && ep.table != nullptr) {
      bool bad;
      const bf16* g = gate_row(ep, row, bad);
      if (bad) atomicOr(&g_gemm_status, (unsigned)kDevErrTableIndex);
      if (g != nullptr) {
        gptr = g + (int64_t)ep.gate_slot * N;
        have_gate = true;
      }
    }
  }
  uint4 xr[4] = {}, xn[4] = {};
  auto load_resid = [&](int c, uint4 (&dst)[4]) {
    if (row_ok) {
      const uint4* src = reinterpret_cast<const uint4*>(ep.resid + row * ep.ldr + col_base + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = src[q];
    }
  };
  if (EPI == kGated) load_resid(0, xr);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    if (EPI == kGated && c + 1 < BN / 32) load_resid(c + 1, xn);
    uint32_t r[32];
    tmem_ld32(tbase + (uint32_t)(c * 32), r);
    if (c == BN / 32 - 1) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(release_bar, 0u);
    }
    const int col0 = col_base + c * 32;
    if (col0 >= N) continue;
    uint4 y[4];
    chunk_values<EPI>(ep, r, row, col0, rs, gptr, have_gate, EPI == kGated ? xr : nullptr, y);
    uint8_t* buf = staging + (chunk & 1u) * kOutChunk;
    if (lane == 0) bulk_wait_read1();  // the store that last used this buffer has read it
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = y[q];
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      const uint32_t src = smem_u32(buf);
      for (int d = 0; d < outs.count; ++d) tma_store_2d(&outs.map[d], src, col0, (int)row0, policy);
      bulk_commit();
    }
    ++chunk;
    if (EPI == kGated) {
#pragma unroll
      for (int q = 0; q < 4; ++q) xr[q] = xn[q];
    }
  }
}

// Drain one 128-row x 256-column accumulator of this warp's TMEM lanes:
// tcgen05.ld 32 columns at a time, release the accumulator (arrive on
// `release_bar`, in CTA `release_rank` of the cluster) once every column is
// in registers, then run the epilogue and store.
template <int EPI>
__device__ __forceinline__ void drain_accumulator(const EpiArgs& ep, int M, int N, uint32_t tbase,
                                                  int64_t row, int col_base, int lane,
                                                  uint32_t release_bar, int release_rank,
                                                  bool remote) {
  const bool row_ok = row < M;
  float rs = 0.0f;
  const bf16* gptr = nullptr;
  bool have_gate = false;
  if (row_ok) {
    if (EPI != kS32 && EPI != kS32Part) rs = ep.row_scale[row];
    if (EPI == kGated && ep.table != nullptr) {
      bool bad;
      const bf16* g = gate_row(ep, row, bad);
      if (bad) atomicOr(&g_gemm_status, (unsigned)kDevErrTableIndex);
      if (g != nullptr) {
        gptr = g + (int64_t)ep.gate_slot * N;
        have_gate = true;
      }
    }
  }
  // Gated residual: each chunk's residual row segment is loaded one chunk
  // ahead, so its memory latency overlaps the previous chunk's epilogue.
  uint4 xr[4] = {}, xn[4] = {};
  auto load_resid = [&](int c, uint4 (&dst)[4]) {
    const int col = col_base + c * 32;
    if (row_ok && col + 32 <= N) {
      const uint4* src = reinterpret_cast<const uint4*>(ep.resid + row * ep.ldr + col);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = src[q];
    }
  };
  if (EPI == kGated) load_resid(0, xr);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    if (EPI == kGated && c + 1 < BN / 32) load_resid(c + 1, xn);
    uint32_t r[32];
    tmem_ld32(tbase + (uint32_t)(c * 32), r);
    if (c == BN / 32 - 1) {
      // All columns of this accumulator are in registers: hand it back.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (remote)
          mbar_arrive_cluster(release_bar, (uint32_t)release_rank);
        else
          mbar_arrive(release_bar);
      }
    }
    const int col0 = col_base + c * 32;
    if (!row_ok || col0 >= N) continue;
    if (EPI == kS32 || EPI == kS32Part) {
      if (col0 + 32 <= N && (N % 4) == 0) {
        int4* dst = reinterpret_cast<int4*>(ep.acc_out + row * (int64_t)N + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]);
      } else {
        store_chunk_tail<EPI>(ep, r, row, col0, N, rs, gptr, have_gate);
      }
    } else if (col0 + 32 <= N) {
      store_chunk_vec<EPI>(ep, r, row, col0, rs, gptr, have_gate, EPI == kGated ? xr : nullptr);
    } else {
      store_chunk_tail<EPI>(ep, r, row, col0, N, rs, gptr, have_gate);
    }
    if (EPI == kGated) {
#pragma unroll
      for (int q = 0; q < 4; ++q) xr[q] = xn[q];
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b, int M, int N, int K, int group_m,
                   const EpiArgs ep) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sa = smem;                               // STAGES x [128 rows x 128 B]
  uint8_t* sb = smem + STAGES * A_STAGE;            // STAGES x [256 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + STAGES * B_STAGE);
  uint64_t* full = bars;                            // TMA landed       (count 1 + tx)
  uint64_t* empty = bars + STAGES;                  // MMA done reading (count 1)
  uint64_t* tfull = bars + 2 * STAGES;              // accumulator ready (count 1)
  uint64_t* tempty = bars + 2 * STAGES + NUM_ACC;   // accumulator drained (count 128)
  uint64_t* drain = bars + 2 * STAGES + 2 * NUM_ACC;  // abort-path MMA drain (count 1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), NUM_EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&map_a);
    prefetch_map(&map_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, A_STAGE + B_STAGE);
          tma_load_2d(smem_u32(sa + stage * A_STAGE), &map_a, fb, kb * BK, mb * BM);
          tma_load_2d(smem_u32(sb + stage * B_STAGE), &map_b, fb, kb * BK, nb * BN);
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Abort: let every copy this thread issued land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) {
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(smem_u32(&full[s]), issued_phase[s]) &&
                   globaltimer() - t0 < g_gemm_wait_limit_ns / 4) {
            }
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
        if (!wait_bounded(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + stage * A_STAGE);
          const uint32_t b0 = smem_u32(sb + stage * B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / UK; ++kk)
            mma_i8(d_tmem, sw128_desc(a0 + kk * UK), sw128_desc(b0 + kk * UK),
                   (kb | kk) != 0 ? 1u : 0u);
          mma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit(smem_u32(&tfull[acc]));
      }
      if (!ok) {
        // Abort: wait for the MMAs already issued before TMEM is released.
        mma_commit(smem_u32(drain));
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0u) && globaltimer() - t0 < g_gemm_wait_limit_ns / 4) {
        }
      }
    }
  } else {
    // -------------------------------------------------- epilogue warps
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32) belong to this warp
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
      // One lane polls; the warp reconverges before the .sync.aligned TMEM loads.
      int ok = 1;
      if (lane == 0) ok = wait_bounded(smem_u32(&tfull[acc]), acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(t, num_m, num_n, group_m, mb, nb);
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      drain_accumulator<EPI>(ep, M, N, tbase, (int64_t)mb * BM + quad * 32 + lane, nb * BN, lane,
                             smem_u32(&tempty[acc]), 0, false);
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------ CTA-pair tensor-core kernel
// A cluster of two CTAs computes one 256x256 output tile: each CTA loads 128
// rows of A and 128 rows (one N half) of B per 128-byte K step, the leader
// (cluster rank 0) issues tcgen05.mma.cta_group::2 (M=256, N=256), and each CTA
// drains its own 128-row accumulator from its TMEM. Per CTA a stage is 32 KB,
// so six stages (192 KB) fit where the single-CTA kernel holds four.
constexpr int STAGES2 = LR_GEMM_STAGES2;
constexpr int A2_STAGE = 128 * BK;
constexpr int B2_STAGE = 128 * BK;
constexpr size_t SMEM2_BYTES = 1024 + (size_t)STAGES2 * (A2_STAGE + B2_STAGE) + BAR_BYTES;
// with the bulk-tensor-store epilogue: the staging buffers start 1 KB past the
// barriers (1024-aligned, as the 64-byte swizzle pattern needs 512)
constexpr size_t SMEM2_OUT_BYTES = 1024 + (size_t)STAGES2 * (A2_STAGE + B2_STAGE) + 1024 + kOutStage;

template <int EPI, bool TMA_OUT = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap map_a,
                    const __grid_constant__ CUtensorMap map_b, int M, int N, int K, int group_m,
                    int splits, const EpiArgs ep, const __grid_constant__ OutMaps outs) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sa = smem;                       // STAGES2 x [128 rows x 128 B]
  uint8_t* sb = smem + STAGES2 * A2_STAGE;  // STAGES2 x [128 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + STAGES2 * B2_STAGE);
  uint64_t* full = bars;                              // leader: both CTAs' copies landed
  uint64_t* empty = bars + STAGES2;                   // pair MMA done reading (multicast)
  uint64_t* tfull = bars + 2 * STAGES2;               // accumulator ready (multicast)
  uint64_t* tempty = bars + 2 * STAGES2 + NUM_ACC;    // leader: both CTAs drained
  uint64_t* drain = bars + 2 * STAGES2 + 2 * NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  // TMA_OUT: per-epilogue-warp double-buffered output staging, 1024-aligned
  uint8_t* out_stage = reinterpret_cast<uint8_t*>(bars) + 1024;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int num_m = (M + 255) / 256;
  const int num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;
  // Split-K: work item w covers tile w / splits and K blocks
  // [(w % splits) * kper, min(+kper, kblocks)); the host picks `splits` so
  // that no slice is empty. With splits == 1 a work item is a whole tile.
  const int kper = (kblocks + splits - 1) / splits;
  const int work = tiles * splits;
  const int cluster_id = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 2 * NUM_EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&map_a);
    prefetch_map(&map_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------ TMA producer (both CTAs)
      const uint64_t pol_a = LR_GEMM_L2_HINTS >= 1 ? l2_policy_evict_last() : l2_policy_evict_normal();
      const uint64_t pol_b = LR_GEMM_L2_HINTS >= 2 ? l2_policy_evict_first() : l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      // test of the bounded waits: the leader of cluster 0 skips one A load,
      // so that stage's barrier never completes (one launch only)
      bool drop = leader && cluster_id == 0 && atomicExch(&g_gemm_drop_load, 0u) != 0u;
      for (int w = cluster_id; w < work && ok; w += clusters) {
        const int t = w / splits;
        const int kb0 = (w - t * splits) * kper;
        const int kb1 = min(kb0 + kper, kblocks);
        int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          if (leader) mbar_expect_tx(fb, 2 * (A2_STAGE + B2_STAGE));
          const uint32_t fb_leader = map_to_rank(fb, 0);
          if (drop)
            drop = false;
          else
            tma_load_2d_pair(smem_u32(sa + stage * A2_STAGE), &map_a, fb_leader, kb * BK,
                             mb * 256 + (int)rank * 128, pol_a);
          tma_load_2d_pair(smem_u32(sb + stage * B2_STAGE), &map_b, fb_leader, kb * BK,
                           nb * BN + (int)rank * 128, pol_b);
          issued_any = true;
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && issued_any) {
        // Abort: copies signal the leader's barrier, so give the ones in flight
        // a fixed grace period to land before this CTA can exit.
        const unsigned long long t0 = globaltimer();
        while (globaltimer() - t0 < 100000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------ MMA issuer (leader only)
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int w = cluster_id; w < work && ok; w += clusters, ++local) {
        const int t = w / splits;
        const int kb0 = (w - t * splits) * kper;
        const int kb1 = min(kb0 + kper, kblocks);
        const int acc = local & 1;
        const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
        if (!wait_bounded_cluster(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + stage * A2_STAGE);
          const uint32_t b0 = smem_u32(sb + stage * B2_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / UK; ++kk)
            mma_i8_pair(d_tmem, sw128_desc(a0 + kk * UK), sw128_desc(b0 + kk * UK),
                        (kb != kb0 || kk != 0) ? 1u : 0u);
          mma_commit_pair(smem_u32(&empty[stage]), (uint16_t)0x3);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit_pair(smem_u32(&tfull[acc]), (uint16_t)0x3);
      }
      if (!ok) {
        mma_commit_pair(smem_u32(drain), (uint16_t)0x1);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(drain), 0u) && globaltimer() - t0 < g_gemm_wait_limit_ns / 4) {
        }
      }
    }
  } else {
    // -------------------------------------------- epilogue warps (both CTAs)
    const int quad = warp & 3;
    uint8_t* staging = out_stage + (warp - 2) * 2 * kOutChunk;
    uint32_t chunk = 0;
    const uint64_t out_policy = LR_GEMM_OUT_EVICT_FIRST ? l2_policy_evict_first() : l2_policy_evict_normal();
    int local = 0;
    for (int w = cluster_id; w < work; w += clusters, ++local) {
      const int t = w / splits;
      const int acc = local & 1;
      const uint32_t acc_phase = (uint32_t)(local >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_bounded(smem_u32(&tfull[acc]), acc_phase, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(t, num_m, num_n, group_m, mb, nb);
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (TMA_OUT) {
        drain_accumulator_tma<EPI>(ep, outs, M, N, tbase, (int64_t)mb * 256 + rank * 128 + quad * 32, nb * BN, lane,
                                   smem_u32(&tempty[acc]), staging, chunk, out_policy);
      } else {
        EpiArgs epw = ep;
        if (EPI == kS32Part) epw.acc_out = ep.acc_out + (int64_t)(w - t * splits) * M * N;
        drain_accumulator<EPI>(epw, M, N, tbase, (int64_t)mb * 256 + rank * 128 + quad * 32 + lane,
                               nb * BN, lane, smem_u32(&tempty[acc]), 0, true);
      }
    }
    if (TMA_OUT && lane == 0) {
      // every bulk store of this warp has written its destinations (local or
      // peer memory) before the kernel can complete
      bulk_wait_all();
      __threadfence_system();
    }
  }

  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------- split-K finishing
// Dequantise the summed int32 split-K workspace [M, N] and apply the epilogue
// (the same epilogue code as the tensor-core kernels, so the bits are the
// same). Split-K is only taken for outputs that allow 16-byte accesses (N a
// multiple of 8, aligned workspace): a thread per 8 consecutive columns of
// one row, so each warp reads 1 KB contiguous runs of every slice's plane.
template <int EPI>
__global__ void __launch_bounds__(256) splitk_epilogue_kernel(const int32_t* __restrict__ ws, int M,
                                                              int N, int splits, const EpiArgs ep) {
  const int64_t row = blockIdx.x;
  const int col0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (col0 >= N) return;
  const float rs = ep.row_scale[row];
  const bf16* gptr = nullptr;
  bool have_gate = false;
  if (EPI == kGated && ep.table != nullptr) {
    bool bad;
    const bf16* g = gate_row(ep, row, bad);
    if (bad && col0 == 0) atomicOr(&g_gemm_status, (unsigned)kDevErrTableIndex);
    if (g != nullptr) {
      gptr = g + (int64_t)ep.gate_slot * N;
      have_gate = true;
    }
  }
  const int64_t plane4 = (int64_t)M * N / 4;  // one slice's plane, in int4 units
  const int4* src = reinterpret_cast<const int4*>(ws + row * (int64_t)N + col0);
  // sum the K slices' partial accumulators, slice 0 first (exact int32 adds)
  int4 lo = __ldcs(src), hi = __ldcs(src + 1);
#pragma unroll 4
  for (int sp = 1; sp < splits; ++sp) {
    const int4 a = __ldcs(src + sp * plane4), b = __ldcs(src + sp * plane4 + 1);
    lo.x += a.x; lo.y += a.y; lo.z += a.z; lo.w += a.w;
    hi.x += b.x; hi.y += b.y; hi.z += b.z; hi.w += b.w;
  }
  const uint32_t acc[8] = {(uint32_t)lo.x, (uint32_t)lo.y, (uint32_t)lo.z, (uint32_t)lo.w,
                           (uint32_t)hi.x, (uint32_t)hi.y, (uint32_t)hi.z, (uint32_t)hi.w};
  store_chunk_vec<EPI, 8>(ep, acc, row, col0, rs, gptr, have_gate);
}

// ---------------------------------------------------------- CUDA-core path
constexpr int ST_M = 64, ST_N = 64, ST_K = 32;

template <int EPI>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const int8_t* __restrict__ a, int64_t lda,
                                                       const int8_t* __restrict__ b,
                                                       int64_t bsk, int64_t bsn, int M, int N,
                                                       int K, const EpiArgs ep) {
  __shared__ int32_t As[ST_K][ST_M + 1];
  __shared__ int32_t Bs[ST_K][ST_N + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * ST_M, n0 = (int64_t)blockIdx.x * ST_N;
  int32_t acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += ST_K) {
    for (int i = threadIdx.x; i < ST_M * ST_K; i += 256) {
      const int mm = i / ST_K, kk = i % ST_K;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? (int32_t)a[gm * lda + gk] : 0;
    }
    for (int i = threadIdx.x; i < ST_N * ST_K; i += 256) {
      const int nn = i / ST_K, kk = i % ST_K;
      const int64_t gn = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < N && gk < K) ? (int32_t)b[gk * bsk + gn * bsn] : 0;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < ST_K; ++kk)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += As[kk][ty * 4 + i] * Bs[kk][tx * 4 + j];
    __syncthreads();
  }
  const uint16_t* bias = reinterpret_cast<const uint16_t*>(ep.bias);
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= M) continue;
    const bf16* gptr = nullptr;
    bool have_gate = false;
    if (EPI == kGated && ep.table != nullptr) {
      bool bad;
      const bf16* g = gate_row(ep, row, bad);
      if (bad) atomicOr(&g_gemm_status, (unsigned)kDevErrTableIndex);
      if (g != nullptr) gptr = g + (int64_t)ep.gate_slot * N, have_gate = true;
    }
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col >= N) continue;
      if (EPI == kS32) {
        ep.acc_out[row * (int64_t)N + col] = acc[i][j];
        continue;
      }
      float d = dequant(acc[i][j], ep.row_scale[row], ep.col_scale[col]);
      if (bias != nullptr) d = __fadd_rn(d, bf_bits(bias[col]));
      float x = 0.0f, g = 0.0f;
      if (EPI == kGated) {
        x = bf_bits(reinterpret_cast<const uint16_t*>(ep.resid)[row * ep.ldr + col]);
        g = have_gate ? bf_bits(reinterpret_cast<const uint16_t*>(gptr)[col])
                      : ((ep.table == nullptr) ? 1.0f : 0.0f);
      }
      reinterpret_cast<uint16_t*>(ep.out)[row * ep.ldo + col] = f2bf_bits(finish<EPI>(d, x, g));
    }
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D uint8 tensor map: `outer` rows of `inner` bytes, rows `stride` bytes
// apart, box of box_outer rows x 128 bytes, 128-byte swizzle, zero fill.
int make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t stride,
             uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LR_OK;
}

// bf16 destination map of the bulk-store epilogue: M rows x N columns from
// `base`, rows `ld` elements apart, box 32 columns x 32 rows, 64-byte swizzle.
int make_out_map(CUtensorMap* map, const void* base, int64_t M, int64_t N, int64_t ld) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return LR_OK;
}

// Where the bulk-store epilogue writes: `count` bf16 matrices (leading
// dimension `ld`), the GEMM's row m landing on row row_offset + m of each.
struct Destinations {
  void* const* ptrs;
  int count;
  int64_t ld;
  int64_t row_offset;
};

// M-blocks per raster group: as many as keep the group's A panel (rows x K
// bytes) within LR_GEMM_PANEL_MB, so the weights stream from HBM about once
// per group.
// L2 budget of a raster group's A panel. With the A panel evict-last and the
// output stores evict-first, 24 MB keeps the panel resident across the group's
// N sweeps (FFN-up 12240x6144->24576: 1.14 GB of DRAM traffic per launch
// against 1.60 GB at 48 MB with the default policies; a 64-80 MB panel, the
// whole A matrix, thrashed: 2.4 GB).
#ifndef LR_GEMM_PANEL_MB
#define LR_GEMM_PANEL_MB 24
#endif
int raster_group(int block_rows, int num_m, int K) {
  const int64_t budget = (int64_t)LR_GEMM_PANEL_MB << 20;
  int64_t g = budget / ((int64_t)block_rows * (K > 0 ? K : 1));
  if (g < 1) g = 1;
  return (int)(g < num_m ? g : num_m);
}

template <typename Kernel>
int configure_smem(Kernel kernel, size_t bytes, bool (&done)[64]) {
  // Once per device and kernel, from any host thread.
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return LR_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return launch_status("gemm: configuring shared memory");
  if (dev >= 0 && dev < 64) done[dev] = true;
  return LR_OK;
}

// Single-CTA tensor-core kernel: 128x256 tiles (used when M <= 128).
template <int EPI>
int launch_tc(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int M, int N, int K,
              const EpiArgs& ep, cudaStream_t stream) {
  CUtensorMap ma, mb;
  int st = make_map(&ma, a, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BM);
  if (st) return st;
  st = make_map(&mb, b, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BN);
  if (st) return st;
  static bool done[64] = {};
  st = configure_smem(gemm_tc_kernel<EPI>, SMEM_BYTES, done);
  if (st) return st;
  const int num_m = (M + BM - 1) / BM;
  const int tiles = num_m * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  gemm_tc_kernel<EPI><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ma, mb, M, N, K,
                                                                  raster_group(BM, num_m, K), ep);
  return launch_status("int8 gemm (tcgen05)");
}

// CTA-pair tensor-core kernel: 256x256 tiles over clusters of two CTAs. With
// `dst` (or, for the bf16 epilogues, whenever N is a multiple of 32 and the
// output allows 16-byte rows) the epilogue stores through shared memory with
// bulk tensor stores; `dst` may name several destinations (see Destinations).
template <int EPI>
int launch_tc2(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int M, int N, int K,
               const EpiArgs& ep, cudaStream_t stream, const Destinations* dst = nullptr) {
  CUtensorMap ma, mb;
  int st = make_map(&ma, a, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 128);
  if (st) return st;
  st = make_map(&mb, b, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 128);
  if (st) return st;
  const int num_m = (M + 255) / 256;
  const int tiles = num_m * ((N + BN - 1) / BN);
  const int pairs = sm_count() / 2;
  const int clusters = tiles < pairs ? tiles : pairs;
  const int group = raster_group(256, num_m, K);
  if constexpr (EPI == kNone || EPI == kGelu || EPI == kGated) {
    const bool tma = dst != nullptr || (LR_GEMM_TMA_OUT && N % 32 == 0 && ep.ldo % 8 == 0 && aligned(ep.out, 16));
    if (tma) {
      OutMaps outs{};
      if (dst != nullptr) {
        for (int d = 0; d < dst->count; ++d) {
          const bf16* base = static_cast<const bf16*>(dst->ptrs[d]) + dst->row_offset * dst->ld;
          st = make_out_map(&outs.map[d], base, M, N, dst->ld);
          if (st) return st;
        }
        outs.count = dst->count;
      } else {
        st = make_out_map(&outs.map[0], ep.out, M, N, ep.ldo);
        if (st) return st;
        outs.count = 1;
      }
      static bool done_tma[64] = {};
      st = configure_smem(gemm_tc2_kernel<EPI, true>, SMEM2_OUT_BYTES, done_tma);
      if (st) return st;
      gemm_tc2_kernel<EPI, true><<<2 * clusters, NUM_THREADS, SMEM2_OUT_BYTES, stream>>>(ma, mb, M, N, K, group, 1,
                                                                                        ep, outs);
      return launch_status("int8 gemm (tcgen05, CTA pair, bulk-store epilogue)");
    }
  }
  if (dst != nullptr) return set_error(LR_ERR_UNSUPPORTED, "int8 gemm: this epilogue has no multi-destination form");
  static bool done[64] = {};
  st = configure_smem(gemm_tc2_kernel<EPI>, SMEM2_BYTES, done);
  if (st) return st;
  const OutMaps none{};
  gemm_tc2_kernel<EPI><<<2 * clusters, NUM_THREADS, SMEM2_BYTES, stream>>>(ma, mb, M, N, K, group, 1, ep, none);
  return launch_status("int8 gemm (tcgen05, CTA pair)");
}

// Number of K slices for a shape whose tiles cannot fill the GPU's CTA pairs
// (1: no split). Each slice keeps at least 4 K blocks of 128.
int splitk_slices(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
  const int64_t pairs = sm_count() / 2;
  const int64_t kblocks = (K + BK - 1) / BK;
  if (tiles * 2 > pairs || kblocks < 8) return 1;
  int64_t s = pairs / tiles;
  if (s > kblocks / 4) s = kblocks / 4;
  if (s > 16) s = 16;
  if (s < 2) return 1;
  const int64_t kper = (kblocks + s - 1) / s;
  return (int)((kblocks + kper - 1) / kper);  // every slice non-empty
}

// Split-K on the CTA-pair kernel: each K slice stores its partial int32
// accumulators into its own [M, N] plane of the workspace; the epilogue kernel
// adds the planes in slice order and applies the epilogue.
template <int EPI>
int launch_tc2_splitk(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, int M, int N,
                      int K, int splits, int32_t* ws, const EpiArgs& ep, bool vec,
                      cudaStream_t stream) {
  // the finishing kernel's 16-byte accesses: checked before anything launches
  if (!vec || N % 8 != 0 || !aligned(ws, 16))
    return set_error(LR_ERR_UNSUPPORTED, "int8 gemm split-K: output not vectorisable");
  CUtensorMap ma, mb;
  int st = make_map(&ma, a, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 128);
  if (st) return st;
  st = make_map(&mb, b, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 128);
  if (st) return st;
  static bool done[64] = {};
  st = configure_smem(gemm_tc2_kernel<kS32Part>, SMEM2_BYTES, done);
  if (st) return st;
  EpiArgs acc = {};
  acc.acc_out = ws;
  const int num_m = (M + 255) / 256;
  const int work = num_m * ((N + BN - 1) / BN) * splits;
  const int pairs = sm_count() / 2;
  const int clusters = work < pairs ? work : pairs;
  const OutMaps none{};
  gemm_tc2_kernel<kS32Part><<<2 * clusters, NUM_THREADS, SMEM2_BYTES, stream>>>(
      ma, mb, M, N, K, raster_group(256, num_m, K), splits, acc, none);
  st = launch_status("int8 gemm (tcgen05, CTA pair, split-K)");
  if (st) return st;
  const dim3 grid((unsigned)M, (unsigned)((N / 8 + 255) / 256));
  splitk_epilogue_kernel<EPI><<<grid, 256, 0, stream>>>(ws, M, N, splits, ep);
  return launch_status("int8 gemm split-K epilogue");
}

template <int EPI>
int launch_simt(const int8_t* a, int64_t lda, const int8_t* b, int64_t bsk, int64_t bsn, int M,
                int N, int K, const EpiArgs& ep, cudaStream_t stream) {
  dim3 grid((N + ST_N - 1) / ST_N, (M + ST_M - 1) / ST_M);
  if (grid.y > 65535) return set_error(LR_ERR_UNSUPPORTED, "gemm: too many rows for the CUDA-core path");
  gemm_simt_kernel<EPI><<<grid, 256, 0, stream>>>(a, lda, b, bsk, bsn, M, N, K, ep);
  return launch_status("int8 gemm (cuda cores)");
}

template <int EPI>
int run(const int8_t* a, int64_t lda, const int8_t* b, int64_t bsk, int64_t bsn, int64_t M,
        int64_t N, int64_t K, const EpiArgs& ep, bool out_vec_ok, cudaStream_t stream,
        int32_t* ws = nullptr, int64_t ws_bytes = 0, const Destinations* dst = nullptr) {
  const bool tc = bsk == 1 && K > 0 && lda % 16 == 0 && bsn % 16 == 0 && aligned(a, 16) &&
                  aligned(b, 16) && out_vec_ok;
  if (dst != nullptr) {
    if (!tc || M <= BM || N % 32 != 0)
      return set_error(LR_ERR_UNSUPPORTED,
                       "int8 gemm to several destinations needs the CTA-pair tensor-core path "
                       "(K-major 16-byte operands, M > %d, N a multiple of 32)", BM);
    return launch_tc2<EPI>(a, lda, b, bsn, (int)M, (int)N, (int)K, ep, stream, dst);
  }
  if constexpr (EPI != kS32) {
    if (tc && ws != nullptr) {
      const int splits = splitk_slices(M, N, K);
      if (splits > 1 && ws_bytes >= splits * M * N * (int64_t)sizeof(int32_t) && aligned(ws, 16))
        return launch_tc2_splitk<EPI>(a, lda, b, bsn, (int)M, (int)N, (int)K, splits, ws, ep,
                                      out_vec_ok, stream);
    }
  }
  if (tc && M > BM) return launch_tc2<EPI>(a, lda, b, bsn, (int)M, (int)N, (int)K, ep, stream);
  if (tc) return launch_tc<EPI>(a, lda, b, bsn, (int)M, (int)N, (int)K, ep, stream);
  return launch_simt<EPI>(a, lda, b, bsk, bsn, (int)M, (int)N, (int)K, ep, stream);
}

}  // namespace gemm

int read_status_gemm(unsigned int* bits, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess)
    return launch_status("reading the gemm status");
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(zero)) != cudaSuccess)
      return launch_status("clearing the gemm status");
  }
  *bits |= v;
  return LR_OK;
}

}  // namespace lr

namespace {

int check_gemm_shape(const char* who, const int8_t* a, int64_t lda, const int8_t* b,
                     int64_t bsk, int64_t bsn, int64_t M, int64_t N, int64_t K) {
  LR_REQUIRE(M >= 0 && N > 0 && K >= 0, "%s: invalid shape M=%lld N=%lld K=%lld", who,
             (long long)M, (long long)N, (long long)K);
  LR_REQUIRE(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "%s: dimension too large", who);
  LR_REQUIRE(lda >= K, "%s: lda %lld < K %lld", who, (long long)lda, (long long)K);
  LR_REQUIRE(bsk >= 0 && bsn >= 0, "%s: negative weight strides", who);
  LR_REQUIRE(M == 0 || (a != nullptr && b != nullptr), "%s: null operand", who);
  return LR_OK;
}

}  // namespace

static int gemm_entry(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                      int64_t b_stride_n, int64_t M, int64_t N, int64_t K, const float* row_scale,
                      const float* col_scale, const void* bias, int epilogue, const void* resid,
                      int64_t ldr, const void* table, int64_t table_rows, int64_t table_width,
                      const int64_t* indices, int64_t sequence, int gate_slot, void* out,
                      int64_t ldo, void* workspace, int64_t workspace_bytes, void* stream,
                      const lr::gemm::Destinations* dst = nullptr) {
  using namespace lr::gemm;
  int st = check_gemm_shape("int8_gemm", a, lda, b, b_stride_k, b_stride_n, M, N, K);
  if (st) return st;
  if (M == 0) return LR_OK;
  LR_REQUIRE(row_scale && col_scale && out, "int8_gemm: null scale or output pointer");
  LR_REQUIRE(ldo >= N, "int8_gemm: ldo %lld < N %lld", (long long)ldo, (long long)N);
  LR_REQUIRE(epilogue >= LR_EPI_NONE && epilogue <= LR_EPI_GATED_RESIDUAL,
             "int8_gemm: unknown epilogue %d", epilogue);
  EpiArgs ep{};
  ep.row_scale = row_scale;
  ep.col_scale = col_scale;
  ep.bias = static_cast<const bf16*>(bias);
  ep.out = static_cast<bf16*>(out);
  ep.ldo = ldo;
  // The tensor-core epilogue uses 16-byte accesses of out/bias/col_scale/resid and
  // of the gate row (table + row*table_width + gate_slot*N): all must be aligned.
  bool vec = lr::aligned(out, 16) && ldo % 8 == 0 && N % 8 == 0 && lr::aligned(col_scale, 16) &&
             (bias == nullptr || lr::aligned(bias, 16));
  if (epilogue == LR_EPI_GATED_RESIDUAL) {
    LR_REQUIRE(resid != nullptr && ldr >= N, "int8_gemm: gated residual needs resid with ldr >= N");
    LR_REQUIRE(sequence > 0, "int8_gemm: sequence must be positive");
    if (table != nullptr) {
      LR_REQUIRE(indices != nullptr && table_rows > 0, "int8_gemm: table needs indices and rows");
      LR_REQUIRE(gate_slot >= 0 && (int64_t)(gate_slot + 1) * N <= table_width,
                 "int8_gemm: gate slot %d does not fit table width %lld", gate_slot,
                 (long long)table_width);
    }
    ep.resid = static_cast<const bf16*>(resid);
    ep.ldr = ldr;
    ep.table = static_cast<const bf16*>(table);
    ep.table_rows = table_rows;
    ep.table_width = table_width;
    ep.indices = indices;
    ep.sequence = sequence;
    ep.gate_slot = gate_slot;
    vec = vec && lr::aligned(resid, 16) && ldr % 8 == 0 &&
          (table == nullptr || (lr::aligned(table, 16) && table_width % 8 == 0));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* ws = static_cast<int32_t*>(workspace);
  switch (epilogue) {
    case LR_EPI_GELU_TANH:
      return run<kGelu>(a, lda, b, b_stride_k, b_stride_n, M, N, K, ep, vec, s, ws, workspace_bytes, dst);
    case LR_EPI_GATED_RESIDUAL:
      return run<kGated>(a, lda, b, b_stride_k, b_stride_n, M, N, K, ep, vec, s, ws, workspace_bytes, dst);
    default:
      return run<kNone>(a, lda, b, b_stride_k, b_stride_n, M, N, K, ep, vec, s, ws, workspace_bytes, dst);
  }
}

extern "C" int lr_int8_gemm_rows_to(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                                    int64_t b_stride_n, int64_t M, int64_t N, int64_t K,
                                    const float* row_scale, const float* col_scale, const void* bias,
                                    int epilogue, const void* resid, int64_t ldr, const void* table,
                                    int64_t table_rows, int64_t table_width, const int64_t* indices,
                                    int64_t sequence, int gate_slot, void* const* destinations,
                                    int num_destinations, int64_t ld_destination, int64_t row_offset,
                                    void* stream) {
  LR_REQUIRE(num_destinations >= 1 && num_destinations <= lr::gemm::kMaxDst,
             "int8_gemm_rows_to: %d destinations (1 to %d)", num_destinations, lr::gemm::kMaxDst);
  LR_REQUIRE(destinations != nullptr, "int8_gemm_rows_to: null destination list");
  LR_REQUIRE(ld_destination >= N && ld_destination % 8 == 0 && row_offset >= 0,
             "int8_gemm_rows_to: ld_destination %lld (>= N, a multiple of 8) / row_offset %lld",
             (long long)ld_destination, (long long)row_offset);
  for (int d = 0; d < num_destinations; ++d)
    LR_REQUIRE(destinations[d] != nullptr && lr::aligned(destinations[d], 16),
               "int8_gemm_rows_to: destination %d is null or not 16-byte aligned", d);
  if (M == 0) return LR_OK;
  const lr::gemm::Destinations dst{destinations, num_destinations, ld_destination, row_offset};
  void* first = static_cast<__nv_bfloat16*>(destinations[0]) + row_offset * ld_destination;
  return gemm_entry(a, lda, b, b_stride_k, b_stride_n, M, N, K, row_scale, col_scale, bias, epilogue, resid,
                    ldr, table, table_rows, table_width, indices, sequence, gate_slot, first, ld_destination,
                    nullptr, 0, stream, &dst);
}

extern "C" int lr_int8_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                            int64_t b_stride_n, int64_t M, int64_t N, int64_t K,
                            const float* row_scale, const float* col_scale, const void* bias,
                            int epilogue, const void* resid, int64_t ldr, const void* table,
                            int64_t table_rows, int64_t table_width, const int64_t* indices,
                            int64_t sequence, int gate_slot, void* out, int64_t ldo, void* stream) {
  return gemm_entry(a, lda, b, b_stride_k, b_stride_n, M, N, K, row_scale, col_scale, bias,
                    epilogue, resid, ldr, table, table_rows, table_width, indices, sequence,
                    gate_slot, out, ldo, nullptr, 0, stream);
}

extern "C" int lr_gemm_test_wait(int64_t limit_ns, int drop_first_load) {
  LR_REQUIRE(limit_ns >= 0 && limit_ns <= 60ll * 1000000000ll, "gemm_test_wait: limit %lld ns", (long long)limit_ns);
  const unsigned long long limit = limit_ns > 0 ? (unsigned long long)limit_ns : lr::gemm::kWaitLimitNs;
  const unsigned int drop = drop_first_load ? 1u : 0u;
  if (cudaMemcpyToSymbol(lr::g_gemm_wait_limit_ns, &limit, sizeof(limit)) != cudaSuccess ||
      cudaMemcpyToSymbol(lr::g_gemm_drop_load, &drop, sizeof(drop)) != cudaSuccess)
    return lr::launch_status("gemm_test_wait");
  return LR_OK;
}

extern "C" int64_t lr_int8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || M >= (1ll << 31) || N >= (1ll << 31)) return 0;
  const int splits = lr::gemm::splitk_slices(M, N, K);
  return splits > 1 ? splits * M * N * (int64_t)sizeof(int32_t) : 0;
}

extern "C" int lr_int8_gemm_ws(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                               int64_t b_stride_n, int64_t M, int64_t N, int64_t K,
                               const float* row_scale, const float* col_scale, const void* bias,
                               int epilogue, const void* resid, int64_t ldr, const void* table,
                               int64_t table_rows, int64_t table_width, const int64_t* indices,
                               int64_t sequence, int gate_slot, void* out, int64_t ldo,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_entry(a, lda, b, b_stride_k, b_stride_n, M, N, K, row_scale, col_scale, bias,
                    epilogue, resid, ldr, table, table_rows, table_width, indices, sequence,
                    gate_slot, out, ldo, workspace, workspace_bytes, stream);
}

extern "C" int lr_int8_gemm_s32(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                                int64_t b_stride_n, int64_t M, int64_t N, int64_t K, int32_t* acc,
                                void* stream) {
  using namespace lr::gemm;
  int st = check_gemm_shape("int8_gemm_s32", a, lda, b, b_stride_k, b_stride_n, M, N, K);
  if (st) return st;
  if (M == 0) return LR_OK;
  LR_REQUIRE(acc != nullptr, "int8_gemm_s32: null output");
  EpiArgs ep{};
  ep.acc_out = acc;
  return run<kS32>(a, lda, b, b_stride_k, b_stride_n, M, N, K, ep, lr::aligned(acc, 16),
                   static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------- allocation-free GEMM
// Some callers cannot allocate device memory at the point where they run the
// GEMM: a host that hands this library only the tensors it already owns (a
// plugin or FFI caller with no allocator, a framework whose memory pool is
// frozen during a step). For them lr_int8_gemm_noalloc runs the same GEMM with
// the split-K scratch taken from this fixed array instead of a caller
// workspace. The array is LR_NOALLOC_SCRATCH_BYTES (16 MiB) and lives on every
// GPU that loads the library until the process exits.
static __device__ __align__(256) int32_t g_noalloc_scratch[LR_NOALLOC_SCRATCH_BYTES / sizeof(int32_t)];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device. In host code the
// array's name only stands for the symbol, so the address is looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return lr::launch_status("noalloc scratch: cudaGetDevice");
  if (dev < 0 || dev >= 64)
    return lr::set_error(LR_ERR_UNSUPPORTED, "noalloc scratch: device %d is out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return lr::set_error(LR_ERR_CUDA, "noalloc scratch: cudaGetSymbolAddress failed (%s)",
                           cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LR_OK;
}

}  // namespace

extern "C" int lr_int8_gemm_noalloc(const int8_t* a, int64_t lda, const int8_t* b,
                                    int64_t b_stride_k, int64_t b_stride_n, int64_t M, int64_t N,
                                    int64_t K, const float* row_scale, const float* col_scale,
                                    const void* bias, int epilogue, const void* resid, int64_t ldr,
                                    const void* table, int64_t table_rows, int64_t table_width,
                                    const int64_t* indices, int64_t sequence, int gate_slot,
                                    void* out, int64_t ldo, void* stream) {
  const int64_t need = lr_int8_gemm_workspace_bytes(M, N, K);  // 0: this shape runs unsplit
  if (need > (int64_t)LR_NOALLOC_SCRATCH_BYTES)
    return lr::set_error(LR_ERR_UNSUPPORTED,
                         "int8_gemm_noalloc: M=%lld N=%lld K=%lld needs %lld bytes of split-K "
                         "scratch, more than the %lld-byte static maximum; use lr_int8_gemm_ws "
                         "with a caller-provided workspace",
                         (long long)M, (long long)N, (long long)K, (long long)need,
                         (long long)LR_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    const int st = noalloc_scratch(&scratch);
    if (st) return st;
  }
  return gemm_entry(a, lda, b, b_stride_k, b_stride_n, M, N, K, row_scale, col_scale, bias,
                    epilogue, resid, ldr, table, table_rows, table_width, indices, sequence,
                    gate_slot, out, ldo, scratch, need > 0 ? (int64_t)LR_NOALLOC_SCRATCH_BYTES : 0,
                    stream);
}
