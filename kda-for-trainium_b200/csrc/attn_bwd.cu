// Grouped-query attention backward (head_dim 128), flash-style on tcgen05:
// P and dS live only in shared memory, one 128 x 128 block at a time.
//
// One CTA per (batch b, kv head g, key block j of 128 keys).  It keeps dV_j and
// dK_j in tensor memory and walks every query block i of the group's heads
// (causal: only blocks at or after the key block):
//   S^T  = K_j Q_i^T                  (keys x queries, TMEM)
//   P^T  = 2^(S^T scale log2e - lse)  (row warps, half a key row -- 64
//                                      queries -- per thread; bf16 into
//                                      shared memory)
//   dP^T = V_j dO_i^T                 (TMEM)
//   dS'^T = P^T (dP^T - di)           (row warps; bf16 into shared memory; the
//                                      softmax scale is applied to dK and dQ at
//                                      the end instead of to every element)
//   dV_j += P^T dO_i,  dK_j += dS'^T Q_i   (TMEM accumulators)
//   dQ_i^T = K_j^T dS'^T              (TMEM, into dP^T's columns: lane = head
//                                      dimension, column = query), added into
//                                      an fp32 dQ in global memory by the dQ
//                                      warps, one 128-byte line per warp
//                                      instruction (red.global.add.f32)
// lse (each query row's log2-sum-exp of the scaled scores) comes from the
// forward, di = rowsum(dout * out) from a row kernel.  Every operand tile is
// loaded once with one 128-byte-swizzled layout (two 64-column halves of 128
// rows): read K-major where its rows index M or N, and MN-major (64-element
// atoms 16 KB apart, 8-row groups 1024 B apart) where its rows index K --
// Q_i and dO_i serve both S^T / dP^T (K-major) and dK / dV (MN-major), K_j
// both S^T (K-major A) and dQ^T (MN-major A), dS'^T both dK (K-major A) and
// dQ^T (MN-major B).
//
// Issue order per query block i (one tensor-core queue):
//   dP(i) | dV(i) | S(i+1) | dQ(i) dK(i)
// S(i+1) goes in as soon as the row warps have copied S(i) out of TMEM, so
// they start on P(i+1) right after dS(i); dQ(i) goes before dK(i) so its
// columns are read out (and dP(i+1) can reuse them) while dK(i) runs.
//
// 512 threads: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer,
// warp 2 scheduler (performs every mbarrier wait the issuer needs and releases
// it group by group at a named barrier: an mbarrier wait in the issuing thread
// would stall behind its queued MMAs), warp 3 idle, warps 4-7 / 8-11 row warps
// (key rows; queries [0, 64) / [64, 128)), warps 12-15 dQ warps
// (head-dimension rows of dQ^T).
// TMEM columns: S^T [0,128), dP^T / dQ^T [128,256), dV [256,384), dK [384,512).
// Shared memory: K_j | V_j | Q (two buffers) | dO_i | P^T | dS'^T (7 x 32 KB)
// | lse, di.
// All mbarrier waits are bounded (common.cuh); every TMA load targets one CTA.
#include <math.h>

#include "common.cuh"

KDA_DEFINE_ERROR_WORD(attn_bwd)

#define KDA_BWD_TRY(expr)                 \
  do {                                    \
    const kda_status s_ = (expr);         \
    if (s_ != KDA_OK) return s_;          \
  } while (0)

namespace kda {
namespace {

constexpr int kD = 128;
constexpr int kBlk = 128;
constexpr uint32_t kTile = kBlk * kD * 2;  // 32 KB
constexpr uint32_t kHalf = kTile / 2;
constexpr int kThreads = 512;
// Register split (setmaxnreg, per warpgroup): the control warpgroup
// (producer, issuer with its unrolled operand descriptors, scheduler) and the
// dQ warps, which hold a full 128-column row of dQ^T, take registers from the
// two row warpgroups (64 queries of a key row each).  128 x (144 + 2 x 112 +
// 144) = 65536 must not exceed the launch allocation, 512 x the compiled
// registers per thread (checked before launch: an increase beyond it would
// wait forever).
constexpr int kRegsCtl = 144;
constexpr int kRegsRow = 112;
constexpr int kRegsDq = 144;
constexpr int kRegsNeeded = (128 * (kRegsCtl + 2 * kRegsRow + kRegsDq) + kThreads - 1) / kThreads;
constexpr int kGoBarrier = 1;  // named barrier: scheduler warp + MMA warp

struct BwdParams {
  int B, S, QH, KH, rep;
  int nkb;          // key (and query) blocks per sequence
  int causal;
  float sl2;        // softmax scale * log2(e)
  float scale;      // softmax scale (applied to dK here, to dQ by the conversion)
  const float* lse;  // [B][QH][S]
  const float* di;   // [B][QH][S]
  float* dq;         // fp32 [B][QH][S][128] (the transposed dQ), zeroed before the launch, unscaled
  __nv_bfloat16* dk;  // [B][S][KH][128]
  __nv_bfloat16* dv;
};

struct Smem {
  // K_j | V_j | Q (two buffers) | dO_i | P^T | dS^T
  static constexpr uint32_t kK = 0, kV = kTile, kQ = 2 * kTile, kDO = 4 * kTile, kP = 5 * kTile, kDS = 6 * kTile;
  static constexpr uint32_t kLse = 7 * kTile;             // 128 floats
  static constexpr uint32_t kDi = kLse + 512;             // 128 floats
  static constexpr uint32_t kBars = kDi + 512;
  // kv_full q_full[2] q_free[2] do_full do_free lse_full di_full s_ready
  // dp_ready p_ready ds_ready dq_ready dq_free dkv_ready holder
  static constexpr uint32_t kNumBars = 18;
  static constexpr size_t kBytes = 1024 + kBars + kNumBars * 8 + 16;
  static_assert(kBytes > 116 * 1024 && kBytes <= 227 * 1024, "shared memory budget");
};

// Query blocks a key block visits (per head of its group): causal keeps the
// blocks at or after it (128-row blocks on both sides).
__device__ __forceinline__ void q_range(const BwdParams& p, int j, int& q0, int& nq) {
  q0 = p.causal ? j : 0;
  nq = p.nkb - q0;
}

// Query block of step `it` (head it / nq of the group): each key block starts
// its walk at a different query block, so the CTAs of one (batch, kv head)
// add into different rows of dQ at any moment instead of all into the same.
__device__ __forceinline__ int q_block(int j, int q0, int nq, int it) { return q0 + (it % nq + j) % nq; }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ float4 ld_shared_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Bits [a, b) of a 32-bit word (empty when a >= b); a, b may lie outside [0, 32].
__device__ __forceinline__ uint32_t range_mask(int a, int b) {
  a = a < 0 ? 0 : a;
  b = b > 32 ? 32 : b;
  if (a >= b) return 0u;
  const uint32_t hi = b >= 32 ? 0xffffffffu : ((1u << b) - 1u);
  return hi & ~((1u << a) - 1u);
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                    const BwdParams p, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::kBars);
  uint64_t* kv_full = bars + 0;     // K_j, V_j landed
  uint64_t* q_full = bars + 1;      // [2] Q_i landed in buffer i % 2
  uint64_t* q_free = bars + 3;      // [2] the MMAs that read buffer i % 2 (last: dK) are done
  uint64_t* do_full = bars + 5;     // dO_i landed
  uint64_t* do_free = bars + 6;     // the MMAs that read dO_i (last: dV) are done
  uint64_t* lse_full = bars + 7;    // lse_i landed (loaded once the row warps wrote P(i - 1))
  uint64_t* di_full = bars + 8;     // di_i landed (loaded once the row warps wrote dS(i - 1))
  uint64_t* s_ready = bars + 9;     // S^T(i) in TMEM (and every earlier MMA done)
  uint64_t* dp_ready = bars + 10;   // dP^T(i) in TMEM
  uint64_t* p_ready = bars + 11;    // P^T(i) in shared memory, S^T(i) read out (8 warps)
  uint64_t* ds_ready = bars + 12;   // dS^T(i) in shared memory, dP^T(i) read out (8 warps)
  uint64_t* dq_ready = bars + 13;   // dQ^T(i) in TMEM
  uint64_t* dq_free = bars + 14;    // dQ^T(i) read out of TMEM (4 warps)
  uint64_t* dkv_ready = bars + 15;  // every MMA done: dV_j, dK_j final
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // heaviest key blocks first (causal: block j visits nkb - j query blocks)
  const int bg = static_cast<int>(blockIdx.x) % (p.B * p.KH);
  const int j = static_cast<int>(blockIdx.x) / (p.B * p.KH);
  const int b = bg / p.KH, g = bg - (bg / p.KH) * p.KH;
  int q0, nq;
  q_range(p, j, q0, nq);
  const int n_iter = p.rep * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_free[t], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_free, 1);
    mbar_init(lse_full, 1);
    mbar_init(di_full, 1);
    mbar_init(s_ready, 1);
    mbar_init(dp_ready, 1);
    mbar_init(p_ready, 8);   // one arrival per row warp
    mbar_init(ds_ready, 8);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 4);   // one arrival per dQ warp
    mbar_init(dkv_ready, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // launched at 128 registers per thread: the control warpgroup grows to
  // kRegsCtl (an increase: .inc), the row warpgroups shrink (.dec), the dQ
  // warpgroup grows (.inc)
  static_assert(kRegsCtl >= 128 && kRegsRow <= 128 && kRegsDq >= 128, "setmaxnreg directions");
  if (warp < 4) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsCtl));

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(kv_full, 2 * kTile);
      for (int hh = 0; hh < 2; ++hh) {
        tma_load_4d(smem + Smem::kK + hh * kHalf, &tmK, kv_full, hh * 64, g, j * kBlk, b);
        tma_load_4d(smem + Smem::kV + hh * kHalf, &tmV, kv_full, hh * 64, g, j * kBlk, b);
      }
      uint32_t q_issued = 0;  // Q buffers with a load in flight at the end
      for (int it = 0; it < n_iter && ok; ++it) {
        const uint32_t pprev = static_cast<uint32_t>(it - 1) & 1u;
        const int h = g * p.rep + it / nq;
        const int s0 = q_block(j, q0, nq, it) * kBlk;
        const int qb = it & 1;
        const int64_t drow = (static_cast<int64_t>(b) * p.QH + h) * p.S + s0;  // dout / lse / di row
        const int valid = p.S - s0 < kBlk ? p.S - s0 : kBlk;  // query rows of the block inside S
        const uint32_t vbytes = static_cast<uint32_t>(valid) * 4u;
        // Q_i into buffer i % 2 once dK of block i - 2 is done
        if (it >= 2) ok = mbar_wait(&q_free[qb], static_cast<uint32_t>((it >> 1) - 1) & 1u, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(&q_full[qb], kTile);
        for (int hh = 0; hh < 2; ++hh)
          tma_load_4d(smem + Smem::kQ + qb * kTile + hh * kHalf, &tmQ, &q_full[qb], hh * 64, h, s0, b);
        q_issued |= 1u << qb;
        // lse_i once the row warps are done with P(i - 1)
        if (it >= 1) ok = mbar_wait(p_ready, pprev, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(lse_full, vbytes);
        bulk_load_1d(smem + Smem::kLse, p.lse + drow, vbytes, lse_full);
        // dO_i once dV of block i - 1 is done
        if (it >= 1) ok = mbar_wait(do_free, pprev, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(do_full, kTile);
        for (int hh = 0; hh < 2; ++hh)
          tma_load_2d(smem + Smem::kDO + hh * kHalf, &tmDO, do_full, hh * 64, static_cast<int>(drow));
        // di_i once the row warps are done with dS(i - 1)
        if (it >= 1) ok = mbar_wait(ds_ready, pprev, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(di_full, vbytes);
        bulk_load_1d(smem + Smem::kDi, p.di + drow, vbytes, di_full);
      }
      // no copy may still be writing shared memory when the CTA exits
      if (ok) ok = mbar_wait(kv_full, 0u, err, kErrWaitDrain);
      if (ok && n_iter > 0) {
        const uint32_t last = static_cast<uint32_t>(n_iter - 1);
        mbar_wait(lse_full, last & 1u, err, kErrWaitDrain);
        mbar_wait(do_full, last & 1u, err, kErrWaitDrain);
        mbar_wait(di_full, last & 1u, err, kErrWaitDrain);
        for (int t = 0; t < 2; ++t)
          if (q_issued & (1u << t)) {
            const uint32_t lt = (last & 1u) == static_cast<uint32_t>(t) ? last : last - 1u;  // last use of buffer t
            mbar_wait(&q_full[t], (lt >> 1) & 1u, err, kErrWaitDrain);
          }
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------ MMA issuer / scheduler
    // Both warps walk the same schedule of MMA groups and meet at the go
    // barrier before each one; the scheduler's lane 0 has waited for the
    // group's inputs.
    const bool sched = warp == 2;
    constexpr uint32_t kIdKK = idesc_bf16_f32(kBlk, kBlk, 0, 0);  // K-major A, K-major B
    constexpr uint32_t kIdKM = idesc_bf16_f32(kBlk, kBlk, 0, 1);  // K-major A, MN-major B
    constexpr uint32_t kIdMM = idesc_bf16_f32(kBlk, kBlk, 1, 1);  // MN-major A, MN-major B
    // Descriptors built once per tile and view; a K step adds a constant to
    // the start-address field (16-byte units, no carry below 256 KB).
    // K-major view (rows = M or N, 64-element halves along K): K step kk at
    // (kk / 4) halves + (kk % 4) x 32 bytes.  MN-major view (rows = K): K
    // step kk at kk x 16 rows x 128 bytes, the two 64-element MN atoms 16 KB
    // apart.
    const uint64_t kK = smem_desc_sw128(smem_u32(smem + Smem::kK), 16, 1024);
    const uint64_t kV = smem_desc_sw128(smem_u32(smem + Smem::kV), 16, 1024);
    const uint64_t kQ = smem_desc_sw128(smem_u32(smem + Smem::kQ), 16, 1024);
    const uint64_t kDO = smem_desc_sw128(smem_u32(smem + Smem::kDO), 16, 1024);
    const uint64_t kP = smem_desc_sw128(smem_u32(smem + Smem::kP), 16, 1024);
    const uint64_t kDS = smem_desc_sw128(smem_u32(smem + Smem::kDS), 16, 1024);
    const uint64_t mK = smem_desc_sw128(smem_u32(smem + Smem::kK), kHalf, 1024);
    const uint64_t mQ = smem_desc_sw128(smem_u32(smem + Smem::kQ), kHalf, 1024);
    const uint64_t mDO = smem_desc_sw128(smem_u32(smem + Smem::kDO), kHalf, 1024);
    const uint64_t mDS = smem_desc_sw128(smem_u32(smem + Smem::kDS), kHalf, 1024);
    auto ko = [](int kk) { return static_cast<uint64_t>(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4); };
    auto mo = [](int kk) { return static_cast<uint64_t>(kk * 128); };
    auto qoff = [](int it) { return static_cast<uint64_t>((it & 1) * (kTile >> 4)); };
    // scheduler: wait (lane 0) for up to two barriers, then meet the MMA warp
    auto sched_wait = [&](uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2) -> bool {
      bool good = true;
      if (lane == 0) {
        if (b1) good = mbar_wait(b1, p1, err, kErrWaitFull);
        if (good && b2) good = mbar_wait(b2, p2, err, kErrWaitAccumFree);
      }
      return go_barrier64<kGoBarrier>(__shfl_sync(0xffffffffu, good, 0));
    };
    // S^T(i) = K_j Q_i^T
    auto s_group = [&](int it) {
      if (lane == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_bf16(tmem + 0, kK + ko(kk), kQ + qoff(it) + ko(kk), kIdKK, kk != 0 ? 1u : 0u);
        umma_commit(s_ready);
      }
      __syncwarp();
    };
    bool ok = true;
    bool any = false;
    if (n_iter > 0) {
      ok = sched ? sched_wait(kv_full, 0u, &q_full[0], 0u) : go_barrier64<kGoBarrier>(true);
      if (ok && !sched) {
        s_group(0);
        any = true;
      }
    }
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t par = static_cast<uint32_t>(it) & 1u;
      // dP^T(i) = V_j dO_i^T into the columns of dQ^T(i - 1) once it is read
      if (sched) {
        ok = sched_wait(do_full, par, it > 0 ? dq_free : nullptr, par ^ 1u);
      } else {
        ok = go_barrier64<kGoBarrier>(true);
        if (ok && lane == 0) {
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) umma_bf16(tmem + 128, kV + ko(kk), kDO + ko(kk), kIdKK, kk != 0);
          umma_commit(dp_ready);
        }
        __syncwarp();
      }
      if (!ok) break;
      // dV_j += P^T(i) dO_i
      if (sched) {
        ok = sched_wait(p_ready, par, nullptr, 0u);
      } else {
        ok = go_barrier64<kGoBarrier>(true);
        if (ok && lane == 0) {
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk)
            umma_bf16(tmem + 256, kP + ko(kk), mDO + mo(kk), kIdKM, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(do_free);
        }
        __syncwarp();
      }
      if (!ok) break;
      // S^T(i + 1): its columns were read out before p_ready(i)
      if (it + 1 < n_iter) {
        if (sched) {
          ok = sched_wait(&q_full[(it + 1) & 1], static_cast<uint32_t>((it + 1) >> 1) & 1u, nullptr, 0u);
        } else {
          ok = go_barrier64<kGoBarrier>(true);
          if (ok) s_group(it + 1);
        }
        if (!ok) break;
      }
      // dQ^T(i) = K_j^T dS'^T(i) into dP^T(i)'s columns, then dK_j += dS'^T(i) Q_i
      if (sched) {
        ok = sched_wait(ds_ready, par, nullptr, 0u);
      } else {
        ok = go_barrier64<kGoBarrier>(true);
        if (ok && lane == 0) {
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk) umma_bf16(tmem + 128, mK + mo(kk), mDS + mo(kk), kIdMM, kk != 0);
          umma_commit(dq_ready);
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk)
            umma_bf16(tmem + 384, kDS + ko(kk), mQ + qoff(it) + mo(kk), kIdKM, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&q_free[it & 1]);
        }
        __syncwarp();
      }
    }
    if (!sched && lane == 0 && any) {
      umma_commit(dkv_ready);
      // every issued MMA must finish before TMEM is released
      mbar_wait(dkv_ready, 0u, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------- row warps
    // two warpgroups: grp 0 takes queries [0, 64) of every key row, grp 1
    // queries [64, 128) -- each writes one 64-query half of the P^T and dS^T
    // tiles -- so every SM partition runs two row warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsRow));
    const int grp = (warp - 4) >> 2;
    const int kr = (warp & 3) * 32 + lane;  // key row of this thread (TMEM lane)
    const int kpos = j * kBlk + kr;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float* lse_s = reinterpret_cast<const float*>(smem + Smem::kLse);
    const float* di_s = reinterpret_cast<const float*>(smem + Smem::kDi);
    const uint32_t prow = smem_u32(smem + Smem::kP) + static_cast<uint32_t>(kr * 128);
    const uint32_t dsrow = smem_u32(smem + Smem::kDS) + static_cast<uint32_t>(kr * 128);
    const uint32_t rsw = static_cast<uint32_t>(kr & 7);
    // live queries of this key row: [qlo, S) -- from the key itself when causal,
    // none when the key is past S
    const int qlo = kpos >= p.S ? p.S : (p.causal ? kpos : 0);
    bool ok = true;
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t par = static_cast<uint32_t>(it) & 1u;
      const int s0 = q_block(j, q0, nq, it) * kBlk;
      ok = mbar_wait(s_ready, par, err, kErrWaitAccum) && mbar_wait(lse_full, par, err, kErrWaitFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // P^T row (this group's 64 queries): 2^(s * scale log2e - lse[q]); zero
      // for keys / queries past S and (causal) keys after the query (bit mask
      // per 32 queries: one code path for every block, the select only where
      // a bit is clear).  32 queries at a time: 16 packed words, stored as four
      // 16-byte units of the K-major, 128-byte-swizzled P^T tile (queries
      // [8u, 8u + 8) of a 64-query half = unit u).
      auto p_chunk = [&](const int k, const int odd, const uint32_t (&sv)[32]) {
        const int c = 2 * k + odd;
        const uint32_t live = range_mask(qlo - s0 - c * 32, p.S - s0 - c * 32);
        float e[32];
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          const float4 l4 = ld_shared_f4(lse_s + c * 32 + 4 * i4);
          e[4 * i4 + 0] = exp2_approx(fmaf(__uint_as_float(sv[4 * i4 + 0]), p.sl2, -l4.x));
          e[4 * i4 + 1] = exp2_approx(fmaf(__uint_as_float(sv[4 * i4 + 1]), p.sl2, -l4.y));
          e[4 * i4 + 2] = exp2_approx(fmaf(__uint_as_float(sv[4 * i4 + 2]), p.sl2, -l4.z));
          e[4 * i4 + 3] = exp2_approx(fmaf(__uint_as_float(sv[4 * i4 + 3]), p.sl2, -l4.w));
        }
        if (live != 0xffffffffu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) e[i] = (live >> i) & 1u ? e[i] : 0.f;
        }
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = odd * 4 + u4;  // unit within the half
          st_shared_v4(prow + k * kHalf + ((static_cast<uint32_t>(u) ^ rsw) << 4),
                       pack_bf16x2(e[8 * u4], e[8 * u4 + 1]), pack_bf16x2(e[8 * u4 + 2], e[8 * u4 + 3]),
                       pack_bf16x2(e[8 * u4 + 4], e[8 * u4 + 5]), pack_bf16x2(e[8 * u4 + 6], e[8 * u4 + 7]));
        }
      };
      {
        uint32_t sa[32], sb[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 64 * grp, sa);
        tmem_ld_32x32b_x32(tmem + lane_base + 64 * grp + 32, sb);
        tmem_ld_wait();
        p_chunk(grp, 0, sa);
        p_chunk(grp, 1, sb);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive_warp(p_ready);
      // dS'^T row: P^T (dP^T - di[q])
      ok = mbar_wait(dp_ready, par, err, kErrWaitAccum) && mbar_wait(di_full, par, err, kErrWaitFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // the row's P values back from shared memory (this thread's own row of
      // the P^T tile: no other thread writes it before the next block); a
      // masked entry (P = 0) stays 0 whatever di holds past S
      auto ds_chunk = [&](const int k, const int odd, const uint32_t (&dv)[32]) {
        const int c = 2 * k + odd;
        const uint32_t live = range_mask(qlo - s0 - c * 32, p.S - s0 - c * 32);
        float w[32];
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = odd * 4 + u4;
          const uint4 pv = ld_shared_v4(prow + k * kHalf + ((static_cast<uint32_t>(u) ^ rsw) << 4));
          const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int q4 = 8 * u4 + 4 * h2;  // first of four queries
            const float4 d4 = ld_shared_f4(di_s + c * 32 + q4);
            const float2 pa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pw[2 * h2]));
            const float2 pb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pw[2 * h2 + 1]));
            // dP - di as one packed FMA: di x (-1) + dP
            const float2 m1 = make_float2(-1.f, -1.f);
            const float2 ta = __ffma2_rn(make_float2(d4.x, d4.y), m1,
                                         make_float2(__uint_as_float(dv[q4]), __uint_as_float(dv[q4 + 1])));
            const float2 tb = __ffma2_rn(make_float2(d4.z, d4.w), m1,
                                         make_float2(__uint_as_float(dv[q4 + 2]), __uint_as_float(dv[q4 + 3])));
            const float2 ra = __fmul2_rn(pa, ta), rb = __fmul2_rn(pb, tb);
            w[q4] = ra.x;
            w[q4 + 1] = ra.y;
            w[q4 + 2] = rb.x;
            w[q4 + 3] = rb.y;
          }
        }
        if (live != 0xffffffffu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = (live >> i) & 1u ? w[i] : 0.f;
        }
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = odd * 4 + u4;
          st_shared_v4(dsrow + k * kHalf + ((static_cast<uint32_t>(u) ^ rsw) << 4),
                       pack_bf16x2(w[8 * u4], w[8 * u4 + 1]), pack_bf16x2(w[8 * u4 + 2], w[8 * u4 + 3]),
                       pack_bf16x2(w[8 * u4 + 4], w[8 * u4 + 5]), pack_bf16x2(w[8 * u4 + 6], w[8 * u4 + 7]));
        }
      };
      {
        uint32_t da[32], db[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 128 + 64 * grp, da);
        tmem_ld_32x32b_x32(tmem + lane_base + 128 + 64 * grp + 32, db);
        tmem_ld_wait();
        ds_chunk(grp, 0, da);
        ds_chunk(grp, 1, db);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive_warp(ds_ready);
    }
    // dV_j (group 0), dK_j (group 1; bf16, dK times the softmax scale) once
    // every MMA is done (every key block visits at least one query block)
    if (ok) ok = mbar_wait(dkv_ready, 0u, err, kErrWaitAccum);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      {
        const int which = grp;
        __nv_bfloat16* dst = (which == 0 ? p.dv : p.dk) +
                             ((static_cast<int64_t>(b) * p.S + kpos) * p.KH + g) * kD;
        const float f = which == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256 + which * 128 + c * 32, r);
          tmem_ld_wait();
          if (kpos < p.S) {
            uint4* o = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              o[q] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * q]) * f, __uint_as_float(r[8 * q + 1]) * f),
                                pack_bf16x2(__uint_as_float(r[8 * q + 2]) * f, __uint_as_float(r[8 * q + 3]) * f),
                                pack_bf16x2(__uint_as_float(r[8 * q + 4]) * f, __uint_as_float(r[8 * q + 5]) * f),
                                pack_bf16x2(__uint_as_float(r[8 * q + 6]) * f, __uint_as_float(r[8 * q + 7]) * f));
          }
        }
      }
    }
  } else if (warp >= 12) {
    // ----------------------------------------------------------- dQ warps
    // Thread = head-dimension index d of dQ^T (TMEM lane), 128 query columns:
    // read the whole row, free the columns, then add each query's value into
    // the fp32 scratch at [b][h][s0 + q][d] -- the warp's 32 lanes cover one
    // 128-byte line, consecutive queries 512 bytes apart (immediate offsets).
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsDq));
    const int d = (warp & 3) * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t par = static_cast<uint32_t>(it) & 1u;
      const int h = g * p.rep + it / nq;
      const int s0 = q_block(j, q0, nq, it) * kBlk;
      ok = mbar_wait(dq_ready, par, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t r[128];
      tmem_ld_32x32b_x32(tmem + lane_base + 128, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(tmem + lane_base + 160, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_32x32b_x32(tmem + lane_base + 192, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
      tmem_ld_32x32b_x32(tmem + lane_base + 224, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive_warp(dq_free);
      float* dst = p.dq + ((static_cast<int64_t>(b) * p.QH + h) * p.S + s0) * kD + d;
      const int nvalid = p.S - s0 < kBlk ? p.S - s0 : kBlk;
      if (nvalid == kBlk) {
#pragma unroll
        for (int q = 0; q < kBlk; ++q)
          asm volatile("red.global.add.f32 [%0], %1;" ::"l"(dst + q * kD), "f"(__uint_as_float(r[q])) : "memory");
      } else {
#pragma unroll
        for (int q = 0; q < kBlk; ++q)
          if (q < nvalid)
            asm volatile("red.global.add.f32 [%0], %1;" ::"l"(dst + q * kD), "f"(__uint_as_float(r[q])) : "memory");
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// fp32 [B][QH][S][128] times f -> bf16 [B][S][QH][128], 8 values per thread
// (16 threads per 128-value row; i enumerates the output in order)
__global__ void __launch_bounds__(256) dq_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                         int64_t n8, int S, int QH, float f) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  const int64_t row = i >> 4;  // (b, s, h) of the output
  const int h = static_cast<int>(row % QH);
  const int64_t bs = row / QH;
  const int64_t b = bs / S, s = bs - (bs / S) * S;
  const float4* src = reinterpret_cast<const float4*>(x + ((b * QH + h) * S + s) * kD) + 2 * (i & 15);
  const float4 a = src[0], c = src[1];
  reinterpret_cast<uint4*>(y)[i] = make_uint4(pack_bf16x2(a.x * f, a.y * f), pack_bf16x2(a.z * f, a.w * f),
                                              pack_bf16x2(c.x * f, c.y * f), pack_bf16x2(c.z * f, c.w * f));
}

// [B][S][H][128] as a 4-D map {128, H, S, B}; box {64, 1, 128, 1}
kda_status tmap_bshd(CUtensorMap* m, const void* base, int64_t B, int64_t S, int64_t H) {
  const uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(H), static_cast<uint64_t>(S),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(kD) * 2, static_cast<uint64_t>(H) * kD * 2,
                               static_cast<uint64_t>(S) * H * kD * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kBlk), 1};
  return make_tmap_bf16(m, base, 4, dims, strides, box);
}

}  // namespace

size_t attn_backward_scratch_bytes(int64_t B, int64_t S, int64_t QH) {
  return static_cast<size_t>(B) * S * QH * kD * 4;  // fp32 dQ
}

// dq, dk, dv (bf16, [B,S,H,128]) of the attention whose inputs are q, k
// ([B,S,H,128], already rotated when RoPE is on), dout (B, QH, S, 128), the
// forward's per-row log2-sum-exp `lse` and di = rowsum(dout * out) (both
// [B][QH][S]); `dq32` is fp32 scratch of attn_backward_scratch_bytes().
kda_status attn_backward_flash(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                               const __nv_bfloat16* dout, const float* lse, const float* di, __nv_bfloat16* dq,
                               __nv_bfloat16* dk, __nv_bfloat16* dv, float* dq32, int64_t B, int64_t S, int64_t QH,
                               int64_t KH, bool causal, cudaStream_t st) {
  CUtensorMap tk, tv, tq, tdo;
  KDA_BWD_TRY(tmap_bshd(&tk, k, B, S, KH));
  KDA_BWD_TRY(tmap_bshd(&tv, v, B, S, KH));
  KDA_BWD_TRY(tmap_bshd(&tq, q, B, S, QH));
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(B * QH * S)};
    const uint64_t strides[1] = {static_cast<uint64_t>(kD) * 2};
    const uint32_t box[2] = {64, static_cast<uint32_t>(kBlk)};
    KDA_BWD_TRY(make_tmap_bf16(&tdo, dout, 2, dims, strides, box));
  }
  if (cudaMemsetAsync(dq32, 0, attn_backward_scratch_bytes(B, S, QH), st) != cudaSuccess)
    return launch_status("attn_backward: memset");
  BwdParams p{};
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.QH = static_cast<int>(QH);
  p.KH = static_cast<int>(KH);
  p.rep = static_cast<int>(QH / KH);
  p.nkb = static_cast<int>((S + kBlk - 1) / kBlk);
  p.causal = causal ? 1 : 0;
  p.scale = 1.0f / sqrtf(static_cast<float>(kD));
  p.sl2 = p.scale * 1.4426950408889634f;
  p.lse = lse;
  p.di = di;
  p.dq = dq32;
  p.dk = dk;
  p.dv = dv;
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, attn_bwd_kernel) != cudaSuccess) return launch_status("attn_backward: attributes");
    if (fa.numRegs < kRegsNeeded) {
      set_error("attn_backward: kernel compiled to %d registers/thread, its register split needs %d", fa.numRegs,
                kRegsNeeded);
      return KDA_UNSUPPORTED;
    }
    if (cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Smem::kBytes)) != cudaSuccess)
      return launch_status("attn_backward: cudaFuncSetAttribute");
    attr_set[dev].store(true, std::memory_order_release);
  }
  const unsigned grid = static_cast<unsigned>(B * KH * p.nkb);
  attn_bwd_kernel<<<grid, kThreads, Smem::kBytes, st>>>(tk, tv, tq, tdo, p, kda_err_ptr_attn_bwd());
  KDA_BWD_TRY(launch_status("attn_bwd_kernel"));
  const int64_t n8 = B * S * QH * kD / 8;
  dq_to_bf16_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, st>>>(dq32, dq, n8, p.S, p.QH, p.scale);
  return launch_status("attn_backward: dq to bf16");
}

}  // namespace kda
