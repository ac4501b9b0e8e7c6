// Attention core of the Flash DiT block on sm_100a:
//   out[b, i, h, :] = sum_j softmax_j(scale * q[b,i,h,:] . k[b,j,h,:]) v[b,j,h,:]
// for bf16 Q, K, V laid out [B, S, H, 128] (heads contiguous within a token,
// any token stride), fp32 scores and online softmax, bf16 output — the role
// of the attention backend behind FusedAttention (model/fusion.py:55-57).
//
// One CTA per (128 queries, head, batch); 10 warps:
//   warp 0     TMA producer: the Q tile once, then 128-key K_j and V_j tiles
//              (128-byte swizzle) into three K and two V slots, K two tiles
//              ahead of V (a K slot frees after Q K^T, a V slot after P V);
//   warp 1     one thread issues tcgen05.mma.kind::f16 (bf16 in, fp32 TMEM):
//              S(0), S(1), then per key tile j: O += P(j) V_j followed by
//              S(j+2) = Q K_{j+2}^T into the score buffer P(j) occupied (MMAs
//              of one thread run in order). Scores are double-buffered, so
//              S(j+1) is computed while the softmax of tile j runs and the
//              softmax never waits on its own tile's MMAs. P is read from
//              TMEM (A operand), V as an MN-major operand from its TMA tile;
//   warps 2-9  softmax: two warps per TMEM lane quadrant, each thread owning a
//              query row (= TMEM lane) and one 64-key half of every score
//              tile. Each half keeps its own running max and sum (fp32, exp2,
//              a sixteenth of each full tile's exponentials on the FMA pipe)
//              and its own O accumulator, so the halves never wait for each
//              other within the key loop; the max moves only when it grows by
//              more than 2^8 (exact, since O and l share it), so O is rescaled
//              in TMEM rarely, after its previous P V has finished. P(j) of a
//              half is written as bf16 pairs over the first 32 of its own score
//              columns. At the end the halves exchange max and sum once through
//              shared memory (bounded mbarrier wait) and each warp writes 64
//              output columns: (O_a 2^(m_a-M) + O_b 2^(m_b-M)) / (l_a 2^(m_a-M)
//              + l_b 2^(m_b-M)) -> bf16 -> global.
// TMEM columns: score buffers at 0 and 128, O_a (keys [0, 64) of every tile)
// at 256, O_b (keys [64, 128)) at 384; 512 allocated.
// Every mbarrier wait is bounded (2 s): on timeout the kernel raises a status
// bit, lets its own copies and MMAs finish, frees TMEM and returns.
// No TMA multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "lr_common.cuh"
#include "lr_host.h"

// Exponentials evaluated on the FMA pipe instead of the MUFU unit: every
// LR_ATTN_EMU-th pair of a full key tile (0: none). Tuning knob.
#ifndef LR_ATTN_EMU
#define LR_ATTN_EMU 16
#endif

namespace lr {

static __device__ unsigned int g_attn_status = 0;

namespace attn {

constexpr int D = 128;             // head dim
constexpr int BQ = 128;            // queries per CTA
constexpr int BKV = 128;           // keys per score tile
constexpr int ATOM = 128 * 128;    // [128 rows x 64 bf16] swizzle-128B box
constexpr int TILE = 2 * ATOM;     // [128 rows x 128 bf16]
constexpr int K_SLOTS = 3;
constexpr int V_SLOTS = 2;
constexpr int SOFTMAX_WARPS = 8;   // two per TMEM lane quadrant (64 keys each)
constexpr int NUM_THREADS = 64 + 32 * SOFTMAX_WARPS;
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = TILE;                        // K slots
constexpr int SMEM_V = SMEM_K + K_SLOTS * TILE;     // V slots
constexpr int SMEM_RED = SMEM_V + V_SLOTS * TILE;   // [max | sum][half][row] fp32
constexpr int SMEM_BAR = SMEM_RED + 2 * 2 * BQ * 4;
constexpr int BAR_BYTES = 512;
constexpr size_t SMEM_BYTES = 1024 + SMEM_BAR + BAR_BYTES;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 256;  // score buffers at 0 and 128, O_a at 256, O_b at 384
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// ------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
// Wait for the phase of `bar` with parity `parity`; false if another role
// aborted or after kWaitLimitNs (then this thread raises the abort).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      *abort_flag = 1u;
      atomicOr(&g_attn_status, (unsigned)kDevErrWaitTimeout);
      return false;
    }
  }
}
// Warp-wide bounded wait: every lane polls the barrier and the warp moves on
// together once any lane has seen the phase complete (phases only move
// forward), so no lane waits in a divergent branch.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag, int lane) {
  if (__any_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (__any_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    int stop = 0;
    if (lane == 0) {
      if (*abort_flag) {
        stop = 1;
      } else if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1u;
        atomicOr(&g_attn_status, (unsigned)kDevErrWaitTimeout);
        stop = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024
// bytes apart (stride byte offset); the leading byte offset is unused.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// MN-major operand, 128-byte swizzle: 64 contiguous MN elements (128 bytes)
// per row, K rows 128 bytes apart; the leading byte offset steps between
// 64-element MN blocks (the two TMA boxes of a V tile, ATOM bytes apart),
// the stride byte offset between 8-row K groups (1024 bytes).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(ATOM >> 4) << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// Instruction descriptors, kind::f16: fp32 accumulator [4,6)=1, A and B bf16
// ([7,10)=1, [10,13)=1), B MN-major bit 16 for P V, N>>3 at [17,23), M>>4 at [24,29).
constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BKV >> 3) << 17) |
                              ((uint32_t)(BQ >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(D >> 3) << 17) |
                              ((uint32_t)(BQ >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D += A B with A read from tensor memory (M lanes x K, two bf16 per column).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// Issue a 32-column TMEM load without waiting; the registers are valid only
// after tmem_wait_ld64 (which takes them as in/out operands, so no use can be
// scheduled before the wait).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld64(uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                 "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]),
                 "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]),
                 "+r"(a[29]), "+r"(a[30]), "+r"(a[31]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]),
                 "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]),
                 "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]),
                 "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]),
                 "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair, on the FMA pipe: x = n + f with n = round(x) (add and
// subtract 1.5 * 2^23) and f in [-1/2, 1/2]; 2^f by a cubic fitted to 2^f on
// that interval (relative error below 7.5e-5, far under the bf16 rounding of
// P); 2^n by adding n to the exponent field. x is clamped to >= -125 so the
// result stays a normal float (2^-125 is negligible against a row sum >= 1).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
  const float2 n = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);  // exact
  float2 p = __ffma2_rn(f, make_float2(0.0551716685f, 0.0551716685f), make_float2(0.2426111400f, 0.2426111400f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// P for 64 consecutive scores of a row: p = 2^(s * scale_log2 - m), stored as
// bf16 pairs into `pk`; the pair sums accumulate into lsum (even, odd keys).
template <int EMU>
__device__ __forceinline__ void softmax_half(const float* s, float2 sc2, float2 nm2, float2& lsum,
                                             uint32_t (&pk)[32]) {
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const float2 x = __ffma2_rn(make_float2(s[2 * q], s[2 * q + 1]), sc2, nm2);
    float2 p;
    if (EMU > 0 && (q % (EMU > 0 ? EMU : 1)) == EMU - 1)
      p = exp2_poly2(x);
    else
      p = make_float2(ex2(x.x), ex2(x.y));
    lsum = __fadd2_rn(lsum, p);
    pk[q] = cvt2(p.x, p.y);
  }
}

struct Shape {
  int seq_q, seq_kv, heads;
  int64_t out_ts;  // output token stride (elements)
  float scale_log2;
};

__global__ void __launch_bounds__(NUM_THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const Shape sh, __nv_bfloat16* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bars;           // Q landed (1 + tx)
  uint64_t* k_full = bars + 1;       // [3] K_j landed (1 + tx)
  uint64_t* k_empty = bars + 4;      // [3] Q K_j^T done (commit)
  uint64_t* v_full = bars + 7;       // [2] V_j landed (1 + tx)
  uint64_t* v_empty = bars + 9;      // [2] P_j V_j done (commit)
  uint64_t* s_full = bars + 11;      // [buffer] S(j) ready (commit)
  // p_full alternates by tile parity: the softmax may finish tile j + 1 before
  // the MMA thread has consumed tile j, and a barrier must never run two
  // phases ahead of its waiter.
  uint64_t* p_full = bars + 13;      // [j & 1] P(j) written, O rescaled (8 warps)
  uint64_t* pv_done = bars + 15;     // P(j) V_j done (commit, every j)
  uint64_t* o_done = bars + 16;      // last P V done (commit)
  uint64_t* drain = bars + 17;       // MMA drain before TMEM is freed
  uint64_t* xbar = bars + 18;        // [quadrant] final max / sum exchange of a row's two halves (2 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);
  static_assert(26 * 8 + 8 <= BAR_BYTES, "barrier region");
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, batch = blockIdx.z;
  const int q0 = blockIdx.x * BQ;
  const int tiles = (sh.seq_kv + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < K_SLOTS; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
    }
    for (int s = 0; s < V_SLOTS; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&p_full[s]), SOFTMAX_WARPS);
    }
    mbar_init(smem_u32(pv_done), 1);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(drain), 1);
    for (int b = 0; b < 4; ++b) mbar_init(smem_u32(&xbar[b]), 2);
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&map_q);
    prefetch_map(&map_k);
    prefetch_map(&map_v);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      // K runs two tiles ahead of V (Q K_{j+2}^T is issued right after P_j V_j):
      // K_0 K_1 K_2 V_0 K_3 V_1 ...
      const int32_t x0 = head * D;
      const uint32_t qb = smem_u32(q_full);
      mbar_expect_tx(qb, TILE);
      tma_load_3d(smem_u32(smem + SMEM_Q), &map_q, qb, x0, q0, batch);
      tma_load_3d(smem_u32(smem + SMEM_Q + ATOM), &map_q, qb, x0 + 64, q0, batch);
      bool issued[K_SLOTS + V_SLOTS] = {};
      uint32_t issued_phase[K_SLOTS + V_SLOTS] = {};
      bool ok = true;
      for (int i = 0; i < tiles + 2 && ok; ++i) {
        for (int kv = 0; kv < 2 && ok; ++kv) {
          const int j = kv == 0 ? i : i - 2;  // K_i, then V_{i-2}
          if (j < 0 || j >= tiles) continue;
          const int nslot = kv == 0 ? K_SLOTS : V_SLOTS;
          const int st = j % nslot;
          const uint32_t ph = (uint32_t)(j / nslot) & 1u;
          if (!wait_bounded(smem_u32(kv == 0 ? &k_empty[st] : &v_empty[st]), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(kv == 0 ? &k_full[st] : &v_full[st]);
          uint8_t* dst = smem + (kv == 0 ? SMEM_K : SMEM_V) + st * TILE;
          const CUtensorMap* map = kv == 0 ? &map_k : &map_v;
          mbar_expect_tx(fb, TILE);
          tma_load_3d(smem_u32(dst), map, fb, x0, j * BKV, batch);
          tma_load_3d(smem_u32(dst + ATOM), map, fb, x0 + 64, j * BKV, batch);
          issued[kv * K_SLOTS + st] = true;
          issued_phase[kv * K_SLOTS + st] = ph;
        }
      }
      // Let every copy issued by this thread land before the CTA can exit.
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(qb, 0u) && globaltimer() - t0 < kWaitLimitNs / 4) {
      }
      if (!ok)
        for (int s = 0; s < K_SLOTS + V_SLOTS; ++s)
          if (issued[s]) {
            const uint32_t fb = smem_u32(s < K_SLOTS ? &k_full[s] : &v_full[s - K_SLOTS]);
            const unsigned long long t1 = globaltimer();
            while (!mbar_try_wait(fb, issued_phase[s]) && globaltimer() - t1 < kWaitLimitNs / 4) {
            }
          }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      bool ok = wait_bounded(smem_u32(q_full), 0u, abort_flag);
      tc_fence_after();
      const uint32_t qa = smem_u32(smem + SMEM_Q);
      // S(j) = Q K_j^T into score buffer j & 1.
      auto issue_qk = [&](int j) {
        const uint32_t ka = smem_u32(smem + SMEM_K + (j % K_SLOTS) * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * ATOM + (kk & 3) * 32);
          mma_f16(tmem + (uint32_t)((j & 1) * BKV), desc_kmajor(qa + off), desc_kmajor(ka + off), kIdescQK,
                  kk != 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(&s_full[j & 1]));
        mma_commit(smem_u32(&k_empty[j % K_SLOTS]));
      };
      for (int j = 0; j < 2 && j < tiles && ok; ++j) {
        if (!wait_bounded(smem_u32(&k_full[j]), 0u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_qk(j);
      }
      for (int j = 0; j < tiles && ok; ++j) {
        const int nx = j + 2;
        if (!wait_bounded(smem_u32(&p_full[j & 1]), (uint32_t)(j >> 1) & 1u, abort_flag) ||
            !wait_bounded(smem_u32(&v_full[j % V_SLOTS]), (uint32_t)(j / V_SLOTS) & 1u, abort_flag) ||
            (nx < tiles &&
             !wait_bounded(smem_u32(&k_full[nx % K_SLOTS]), (uint32_t)(nx / K_SLOTS) & 1u, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // O += P(j) V_j, P(j) read from tensor memory (its score buffer).
        const uint32_t va = smem_u32(smem + SMEM_V + (j % V_SLOTS) * TILE);
        // keys [0, 64) into O_a (P over score columns [0, 32)), keys [64, 128)
        // into O_b (P over score columns [64, 96))
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          mma_f16_ts(tmem + COL_O + (kk >= 4 ? 128u : 0u), tmem + (uint32_t)((j & 1) * BKV + kk * 8 + (kk >= 4 ? 32 : 0)),
                     desc_mnmajor(va + (uint32_t)(kk * 16 * 128)), kIdescPV, (j | (kk & 3)) != 0 ? 1u : 0u);
        mma_commit(smem_u32(pv_done));
        mma_commit(smem_u32(&v_empty[j % V_SLOTS]));
        if (j == tiles - 1) mma_commit(smem_u32(o_done));
        if (nx < tiles) issue_qk(nx);  // into the buffer P(j) V_j just read (same order on the tensor core)
      }
      // Wait for every MMA this thread issued before TMEM can be released.
      mma_commit(smem_u32(drain));
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0u) && globaltimer() - t0 < kWaitLimitNs / 4) {
      }
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int quad = warp & 3;          // TMEM lanes [32 quad, 32 quad + 32)
    const int half = (warp - 2) >> 2;   // keys [64 half, 64 half + 64) of every tile
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t o_own = tmem + lane_off + COL_O + (uint32_t)(half * 128);  // this half's O
    float* red = reinterpret_cast<float*>(smem + SMEM_RED);  // [max | sum][half][row]
    uint64_t* xq = xbar + quad;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < tiles; ++j) {
      const int par = j & 1;
      const uint32_t s_col = tmem + lane_off + (uint32_t)(par * BKV + half * 64);
      // S(j) ready; the same commit covers P(j-2) V_{j-2} (issued before).
      if (!warp_wait(smem_u32(&s_full[par]), (uint32_t)(j >> 1) & 1u, abort_flag, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[64];
      {
        uint32_t ra[32], rb[32];
        tmem_ld32_nowait(s_col, ra);
        tmem_ld32_nowait(s_col + 32u, rb);
        tmem_wait_ld64(ra, rb);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          s[e] = __uint_as_float(ra[e]);
          s[32 + e] = __uint_as_float(rb[e]);
        }
      }
      const int valid = sh.seq_kv - j * BKV - half * 64;
      if (valid < 64) {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          if (e >= valid) s[e] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int e = 4; e < 64; e += 4) {
        mx0 = fmaxf(mx0, s[e]);
        mx1 = fmaxf(mx1, s[e + 1]);
        mx2 = fmaxf(mx2, s[e + 2]);
        mx3 = fmaxf(mx3, s[e + 3]);
      }
      // This half's running max moves only when it grows by more than 2^8:
      // p <= 256, O rescaled rarely, exact.
      const float tile_max = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sh.scale_log2;
      const bool move = tile_max > m_run + 8.0f;
      const float m_use = move ? tile_max : m_run;
      const float alpha = move ? ex2(m_run - m_use) : 1.0f;  // 0 on this half's first valid tile
      const float m_sub = m_use == -INFINITY ? 0.0f : m_use;  // no valid key yet: p = 0
      const float2 sc2 = make_float2(sh.scale_log2, sh.scale_log2);
      const float2 nm2 = make_float2(-m_sub, -m_sub);
      float2 lsum = make_float2(0.0f, 0.0f);
      {
        uint32_t pk[32];
        if (valid >= 64)
          softmax_half<LR_ATTN_EMU>(s, sc2, nm2, lsum, pk);
        else  // masked keys need an exact 0: MUFU only
          softmax_half<0>(s, sc2, nm2, lsum, pk);
        tmem_st32(s_col, pk);  // P(j) of this half over its own first 32 score columns
      }
      l_run = fmaf(l_run, alpha, lsum.x + lsum.y);
      m_run = m_use;
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // O must be stable: wait for P(j-1) V_{j-1} (at most one pending).
        if (!warp_wait(smem_u32(pv_done), (uint32_t)(j - 1) & 1u, abort_flag, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 128; c += 64) {
          uint32_t oa[32], ob[32];
          tmem_ld32_nowait(o_own + (uint32_t)c, oa);
          tmem_ld32_nowait(o_own + (uint32_t)c + 32u, ob);
          tmem_wait_ld64(oa, ob);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            oa[e] = __float_as_uint(__uint_as_float(oa[e]) * alpha);
            ob[e] = __float_as_uint(__uint_as_float(ob[e]) * alpha);
          }
          tmem_st32(o_own + (uint32_t)c, oa);
          tmem_st32(o_own + (uint32_t)c + 32u, ob);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[par]));
    }
    // The halves exchange their running max and sum once; each warp then
    // writes output columns [64 half, +64) from both accumulators:
    // O = (O_a 2^(m_a - M) + O_b 2^(m_b - M)) / (l_a 2^(m_a - M) + l_b 2^(m_b - M)).
    float m_o = -INFINITY, l_o = 0.0f;
    if (ok) {
      red[half * BQ + row] = m_run;
      red[(2 + half) * BQ + row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(xq));
      ok = warp_wait(smem_u32(xq), 0u, abort_flag, lane);
      if (ok) {
        m_o = red[(1 - half) * BQ + row];
        l_o = red[(3 - half) * BQ + row];
      }
    }
    if (ok && warp_wait(smem_u32(o_done), 0u, abort_flag, lane)) {
      tc_fence_after();
      const float m_a = half == 0 ? m_run : m_o, m_b = half == 0 ? m_o : m_run;
      const float l_a = half == 0 ? l_run : l_o, l_b = half == 0 ? l_o : l_run;
      const float m_all = fmaxf(m_a, m_b);  // finite: key 0 is valid and in half 0
      const float f_a = ex2(m_a - m_all), f_b = ex2(m_b - m_all);
      const float inv_l = 1.0f / fmaf(l_a, f_a, l_b * f_b);
      const float g_a = f_a * inv_l, g_b = f_b * inv_l;
      const int qrow = q0 + row;
      const uint32_t oa_col = tmem + lane_off + COL_O + (uint32_t)(half * 64);
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t oa[32], ob[32];
        tmem_ld32_nowait(oa_col + (uint32_t)c, oa);
        tmem_ld32_nowait(oa_col + 128u + (uint32_t)c, ob);
        tmem_wait_ld64(oa, ob);
        if (qrow < sh.seq_q) {
          uint4* d4 = reinterpret_cast<uint4*>(out + ((int64_t)batch * sh.seq_q + qrow) * sh.out_ts +
                                               (int64_t)head * D + half * 64 + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              f[e] = fmaf(__uint_as_float(oa[8 * q + e]), g_a, __uint_as_float(ob[8 * q + e]) * g_b);
            d4[q] = pack8(f);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [batch, seq, heads*128] bf16 with token stride `ts` elements: boxes of
// box_rows tokens x 64 columns, 128-byte swizzle, zero fill past the sequence.
int make_map(CUtensorMap* map, const void* base, int64_t heads, int64_t seq, int64_t batch, int64_t ts,
             uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)(heads * D), (cuuint64_t)seq, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ts * 2), (cuuint64_t)(seq * ts * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LR_OK;
}

}  // namespace attn

int read_status_attention(unsigned int* bits, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(v)) != cudaSuccess)
    return launch_status("reading the device status");
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(zero)) != cudaSuccess)
      return launch_status("clearing the device status");
  }
  *bits |= v;
  return LR_OK;
}

}  // namespace lr

extern "C" int lr_attention_bf16(const void* q, int64_t q_token_stride, const void* k, int64_t k_token_stride,
                                 const void* v, int64_t v_token_stride, int64_t batch, int64_t seq_q,
                                 int64_t seq_kv, int64_t heads, int64_t head_dim, float scale, void* out,
                                 int64_t out_token_stride, void* stream) {
  using namespace lr;
  LR_REQUIRE(batch >= 0 && seq_q >= 0 && seq_kv >= 0 && heads > 0, "attention: invalid shape");
  if (head_dim != attn::D)
    return set_error(LR_ERR_UNSUPPORTED, "attention: head_dim %lld (this kernel handles 128)", (long long)head_dim);
  if (batch == 0 || seq_q == 0) return LR_OK;
  LR_REQUIRE(seq_kv > 0, "attention: empty key sequence");
  LR_REQUIRE(q && k && v && out, "attention: null pointer");
  LR_REQUIRE(q_token_stride >= heads * head_dim && k_token_stride >= heads * head_dim &&
                 v_token_stride >= heads * head_dim && out_token_stride >= heads * head_dim,
             "attention: token strides smaller than heads * head_dim");
  if (q_token_stride % 8 || k_token_stride % 8 || v_token_stride % 8 || out_token_stride % 8 || !aligned(q, 16) ||
      !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
    return set_error(LR_ERR_UNSUPPORTED, "attention: pointers and token strides must be 16-byte aligned");
  LR_REQUIRE(seq_q <= INT32_MAX && seq_kv <= INT32_MAX && heads <= 65535 && batch <= 65535,
             "attention: shape too large");
  CUtensorMap mq, mk, mv;
  int st = attn::make_map(&mq, q, heads, seq_q, batch, q_token_stride, attn::BQ);
  if (st) return st;
  st = attn::make_map(&mk, k, heads, seq_kv, batch, k_token_stride, attn::BKV);
  if (st) return st;
  st = attn::make_map(&mv, v, heads, seq_kv, batch, v_token_stride, attn::BKV);
  if (st) return st;
  {
    // Opt in to the kernel's shared memory once per device (any host thread).
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      if (cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)attn::SMEM_BYTES) != cudaSuccess)
        return launch_status("attention: configuring shared memory");
      if (dev >= 0 && dev < 64) configured[dev] = true;
    }
  }
  attn::Shape sh;
  sh.seq_q = (int)seq_q;
  sh.seq_kv = (int)seq_kv;
  sh.heads = (int)heads;
  sh.out_ts = out_token_stride;
  sh.scale_log2 = (float)((double)scale * 1.4426950408889634);
  const dim3 grid((unsigned)((seq_q + attn::BQ - 1) / attn::BQ), (unsigned)heads, (unsigned)batch);
  attn::attention_kernel<<<grid, attn::NUM_THREADS, attn::SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
      mq, mk, mv, sh, static_cast<__nv_bfloat16*>(out));
  return launch_status("attention");
}
