// Attention core of the Flash DiT block on sm_100a:
//   out[b, i, h, :] = sum_j softmax_j(scale * q[b,i,h,:] . k[b,j,h,:]) v[b,j,h,:]
// for bf16 Q, K, V laid out [B, S, H, 128] (heads contiguous within a token,
// any token stride), fp32 scores and online softmax, bf16 output — the role
// of the attention backend behind FusedAttention (model/fusion.py:55-57).
//
// One CTA per (128-query tile, head, batch); 6 warps:
//   warp 0     TMA producer: the Q tile once, then K_j and V_j tiles (128 keys
//              each, 128-byte swizzle) into a 2-stage ring;
//   warp 1     one thread issues tcgen05.mma.kind::f16 (bf16 in, fp32 TMEM):
//              S_j = Q K_j^T into one of two TMEM score buffers (so S_{j+1} is
//              computed while softmax reads S_j), then O += P_j V_j as soon as
//              softmax has written P_j; V is read as an MN-major operand
//              straight from its TMA tile;
//   warps 2-5  softmax, one thread per query row (= TMEM lane): running max and
//              sum in fp32 with exp2, O rescaled in TMEM when the max grows,
//              P_j written as bf16 to shared memory in the swizzled K-major
//              layout the MMA reads; at the end O / l -> bf16 -> global.
// TMEM columns: S buffers at 0 and 128, O at 256 (512 allocated).
// Every mbarrier wait is bounded (2 s): on timeout the kernel raises a status
// bit, lets its own copies and MMAs finish, frees TMEM and returns.
// No TMA multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "lr_common.cuh"
#include "lr_host.h"

namespace lr {

static __device__ unsigned int g_attn_status = 0;

namespace attn {

constexpr int D = 128;          // head dim
constexpr int BQ = 128;         // queries per CTA
constexpr int BKV = 128;        // keys per tile
constexpr int ATOM = 128 * 128; // one [128 rows x 64 bf16] swizzle-128B box
constexpr int TILE = 2 * ATOM;  // [128 rows x 128 bf16]
constexpr int STAGES = 2;
constexpr int NUM_THREADS = 192;
constexpr int SMEM_Q = 0;
constexpr int SMEM_KV = TILE;                       // stage s: K at +2*TILE*s, V at +TILE
constexpr int SMEM_P = SMEM_KV + STAGES * 2 * TILE;
constexpr int SMEM_BAR = SMEM_P + TILE;
constexpr size_t SMEM_BYTES = 1024 + SMEM_BAR + 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 256;
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
// Warp-wide bounded wait: lane 0 polls, the warp reconverges before any
// .sync.aligned tensor-memory instruction that follows.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag, int lane) {
  int ok = 1;
  if (lane == 0) ok = wait_bounded(bar, parity, abort_flag) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
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
// 64-element MN blocks (the two TMA boxes of a tile, ATOM bytes apart), the
// stride byte offset between 8-row K groups (1024 bytes).
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
  uint64_t* kv_full = bars + 1;      // [2] K_j, V_j landed (1 + tx)
  uint64_t* kv_empty = bars + 3;     // [2] P_j V_j done, stage free (commit)
  uint64_t* s_full = bars + 5;       // [2] S_j ready (commit)
  uint64_t* s_free = bars + 7;       // [2] softmax read S_j (4 warps)
  uint64_t* p_full = bars + 9;       // P_j written, O rescaled (4 warps)
  uint64_t* o_done = bars + 10;      // P_j V_j done (commit)
  uint64_t* drain = bars + 11;       // abort-path MMA drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int q0 = qt * BQ;
  const int tiles = (sh.seq_kv + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&kv_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), 1);
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&s_free[s]), 4);
    }
    mbar_init(smem_u32(p_full), 4);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(drain), 1);
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
      const int32_t x0 = head * D;
      uint32_t qb = smem_u32(q_full);
      mbar_expect_tx(qb, TILE);
      tma_load_3d(smem_u32(smem + SMEM_Q), &map_q, qb, x0, q0, batch);
      tma_load_3d(smem_u32(smem + SMEM_Q + ATOM), &map_q, qb, x0 + 64, q0, batch);
      bool issued[2] = {false, false};
      uint32_t issued_phase[2] = {0u, 0u};
      bool ok = true;
      for (int j = 0; j < tiles && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!wait_bounded(smem_u32(&kv_empty[st]), ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = smem_u32(&kv_full[st]);
        uint8_t* kdst = smem + SMEM_KV + st * 2 * TILE;
        mbar_expect_tx(fb, 2 * TILE);
        tma_load_3d(smem_u32(kdst), &map_k, fb, x0, j * BKV, batch);
        tma_load_3d(smem_u32(kdst + ATOM), &map_k, fb, x0 + 64, j * BKV, batch);
        tma_load_3d(smem_u32(kdst + TILE), &map_v, fb, x0, j * BKV, batch);
        tma_load_3d(smem_u32(kdst + TILE + ATOM), &map_v, fb, x0 + 64, j * BKV, batch);
        issued[st] = true;
        issued_phase[st] = ph;
      }
      // Let every copy issued by this thread land before the CTA can exit.
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(qb, 0u) && globaltimer() - t0 < kWaitLimitNs / 4) {
      }
      if (!ok)
        for (int s = 0; s < 2; ++s)
          if (issued[s]) {
            const unsigned long long t1 = globaltimer();
            while (!mbar_try_wait(smem_u32(&kv_full[s]), issued_phase[s]) && globaltimer() - t1 < kWaitLimitNs / 4) {
            }
          }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      bool ok = wait_bounded(smem_u32(q_full), 0u, abort_flag);
      tc_fence_after();
      const uint32_t qa = smem_u32(smem + SMEM_Q);
      const uint32_t pa = smem_u32(smem + SMEM_P);
      for (int j = 0; j <= tiles && ok; ++j) {
        if (j < tiles) {
          const int st = j & 1;
          const uint32_t ph = (uint32_t)(j >> 1) & 1u;
          if (!wait_bounded(smem_u32(&kv_full[st]), ph, abort_flag) ||
              !wait_bounded(smem_u32(&s_free[st]), ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ka = smem_u32(smem + SMEM_KV + st * 2 * TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (uint32_t)((kk >> 2) * ATOM + (kk & 3) * 32);
            mma_f16(tmem + (uint32_t)(st * BKV), desc_kmajor(qa + off), desc_kmajor(ka + off), kIdescQK,
                    kk != 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(&s_full[st]));
        }
        if (j >= 1) {
          const int jp = j - 1, st = jp & 1;
          if (!wait_bounded(smem_u32(p_full), (uint32_t)jp & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t va = smem_u32(smem + SMEM_KV + st * 2 * TILE + TILE);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint32_t poff = (uint32_t)((kk >> 2) * ATOM + (kk & 3) * 32);
            mma_f16(tmem + COL_O, desc_kmajor(pa + poff), desc_mnmajor(va + (uint32_t)(kk * 16 * 128)), kIdescPV,
                    (jp | kk) != 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(o_done));
          mma_commit(smem_u32(&kv_empty[st]));
        }
      }
      // Wait for every MMA this thread issued before TMEM can be released.
      mma_commit(smem_u32(drain));
      const unsigned long long t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(drain), 0u) && globaltimer() - t0 < kWaitLimitNs / 4) {
      }
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32)
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    uint8_t* p_row = smem + SMEM_P + row * 128;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < tiles; ++j) {
      const int sb = j & 1;
      if (!warp_wait(smem_u32(&s_full[sb]), (uint32_t)(j >> 1) & 1u, abort_flag, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + (uint32_t)(sb * BKV + c * 32), r);
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_free[sb]));
      const int valid = sh.seq_kv - j * BKV;
      if (valid < BKV) {
#pragma unroll
        for (int e = 0; e < BKV; ++e)
          if (e >= valid) s[e] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int e = 4; e < BKV; e += 4) {
        mx0 = fmaxf(mx0, s[e]);
        mx1 = fmaxf(mx1, s[e + 1]);
        mx2 = fmaxf(mx2, s[e + 2]);
        mx3 = fmaxf(mx3, s[e + 3]);
      }
      const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sh.scale_log2);
      const float alpha = ex2(m_run - m_new);  // 0 on the first tile (m_run = -inf)
      const float neg_m = -m_new;
      float l0 = 0.0f, l1 = 0.0f;
      uint32_t pk[BKV / 2];
#pragma unroll
      for (int e = 0; e < BKV; e += 2) {
        const float p0 = ex2(fmaf(s[e], sh.scale_log2, neg_m));
        const float p1 = ex2(fmaf(s[e + 1], sh.scale_log2, neg_m));
        l0 += p0;
        l1 += p1;
        pk[e / 2] = cvt2(p0, p1);
      }
      l_run = fmaf(l_run, alpha, l0 + l1);
      m_run = m_new;
      if (j >= 1) {
        // P_{j-1} V_{j-1} must be done: it reads the P buffer and writes O.
        if (!warp_wait(smem_u32(o_done), (uint32_t)(j - 1) & 1u, abort_flag, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            const uint32_t ta = lane_base + COL_O + (uint32_t)(c * 32);
            tmem_ld32(ta, r);
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st32(ta, r);
          }
          tmem_st_wait();
        }
      }
      // P row -> shared memory, K-major with 128-byte swizzle: key chunk c
      // (8 keys, 16 bytes) of row r sits at atom c/8, 16-byte slot (c%8) ^ (r%8).
#pragma unroll
      for (int c = 0; c < BKV / 8; ++c) {
        uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(p_row + (c >> 3) * ATOM + (((c & 7) ^ (row & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(p_full));
    }
    if (ok && warp_wait(smem_u32(o_done), (uint32_t)(tiles - 1) & 1u, abort_flag, lane)) {
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      const int qrow = q0 + row;
      __nv_bfloat16* dst = out + ((int64_t)batch * sh.seq_q + qrow) * sh.out_ts + (int64_t)head * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + COL_O + (uint32_t)(c * 32), r);
        if (qrow < sh.seq_q) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[8 * q + e]) * inv_l;
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
// 128 tokens x 64 columns, 128-byte swizzle, zero fill past the sequence.
int make_map(CUtensorMap* map, const void* base, int64_t heads, int64_t seq, int64_t batch, int64_t ts) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(LR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)(heads * D), (cuuint64_t)seq, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ts * 2), (cuuint64_t)(seq * ts * 2)};
  cuuint32_t box[3] = {64, 128, 1};
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
  int st = attn::make_map(&mq, q, heads, seq_q, batch, q_token_stride);
  if (st) return st;
  st = attn::make_map(&mk, k, heads, seq_kv, batch, k_token_stride);
  if (st) return st;
  st = attn::make_map(&mv, v, heads, seq_kv, batch, v_token_stride);
  if (st) return st;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(attn::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn::SMEM_BYTES) != cudaSuccess)
      return launch_status("attention: configuring shared memory");
    if (dev >= 0 && dev < 64) configured[dev] = true;
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
