// Grouped-query attention backward (head_dim 128), flash-style on tcgen05:
// P and dS live only in shared memory, one 128 x 128 block at a time.
//
// One CTA per (batch b, kv head g, key block j of 128 keys).  It keeps dV_j and
// dK_j in tensor memory and walks every query block i of the group's heads
// (causal: only blocks at or after the key block):
//   S^T  = K_j Q_i^T                 (keys x queries, TMEM)
//   P^T  = 2^(S^T scale log2e - lse)  (row warps, one key row per thread;
//                                      bf16 into shared memory)
//   dP^T = V_j dO_i^T                (TMEM)
//   dS^T = P^T (dP^T - di) scale     (row warps; bf16 into shared memory)
//   dV_j += P^T dO_i,  dK_j += dS^T Q_i    (TMEM accumulators)
//   dQ_i  = dS K_j                   (TMEM, into dP^T's columns), added into an
//                                      fp32 dQ in global memory by the dQ
//                                      warps (red.global.add.v4.f32)
// lse (each query row's log2-sum-exp of the scaled scores) comes from the
// forward, di = rowsum(dout * out) from a row kernel.  Every operand tile is
// loaded once per use site with one 128-byte-swizzled layout (two 64-column
// halves of 128 rows): read K-major where its rows index M or N, and MN-major
// (64-element atoms 16 KB apart, 8-row groups 1024 B apart) where its rows
// index K -- Q_i and dO_i serve both S^T / dP^T (K-major) and dK / dV
// (MN-major), K_j both S^T and dQ, dS^T both dK (K-major A) and dQ (MN-major A).
//
// 384 threads: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer (its
// lane 0 also performs the mbarrier waits its MMAs need), warps 4-7 row warps
// (key rows), warps 8-11 dQ warps (query rows); warps 2-3 idle.
// TMEM columns: S^T [0,128), dP^T / dQ [128,256), dV [256,384), dK [384,512).
// Shared memory: K_j | V_j | Q (two buffers, the next block's lands during
// this one) | dO_i | P^T | dS^T (7 x 32 KB) | lse, di.
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
constexpr int kThreads = 384;
// Register split (setmaxnreg, per warpgroup): the dQ warpgroup gives
// registers to the row warpgroup, which holds a key row's 64 packed P values
// beside 32 scores; the MMA issuer keeps its operand descriptors live.
// 128 x (152 + 200 + 104) = 58368 must not exceed the launch allocation, 384 x
// the compiled registers per thread (checked before launch: an increase
// beyond it would wait forever).
constexpr int kRegsCtl = 152;
constexpr int kRegsRow = 200;
constexpr int kRegsDq = 104;
constexpr int kRegsNeeded = (128 * (kRegsCtl + kRegsRow + kRegsDq) + kThreads - 1) / kThreads;

struct BwdParams {
  int B, S, QH, KH, rep;
  int nkb;          // key (and query) blocks per sequence
  int causal;
  float sl2;        // softmax scale * log2(e)
  float scale;      // softmax scale
  const float* lse;  // [B][QH][S]
  const float* di;   // [B][QH][S]
  float* dq;         // fp32 [B][S][QH][128], zeroed before the launch
  __nv_bfloat16* dk;  // [B][S][KH][128]
  __nv_bfloat16* dv;
};

struct Smem {
  // K_j | V_j | Q (two buffers) | dO_i | P^T | dS^T
  static constexpr uint32_t kK = 0, kV = kTile, kQ = 2 * kTile, kDO = 4 * kTile, kP = 5 * kTile, kDS = 6 * kTile;
  static constexpr uint32_t kLse = 7 * kTile;             // 128 floats
  static constexpr uint32_t kDi = kLse + 512;             // 128 floats
  static constexpr uint32_t kBars = kDi + 512;
  // kv_full q_full[2] q_free[2] do_full do_free ld_full s_ready dp_ready
  // p_ready ds_ready dq_ready dq_free dkv_ready holder
  static constexpr uint32_t kNumBars = 16;
  static constexpr size_t kBytes = 1024 + kBars + kNumBars * 8 + 16;
  static_assert(kBytes > 116 * 1024 && kBytes <= 227 * 1024, "shared memory budget");
};

// Query blocks a key block visits (per head of its group): causal keeps the
// blocks at or after it (128-row blocks on both sides).
__device__ __forceinline__ void q_range(const BwdParams& p, int j, int& q0, int& nq) {
  q0 = p.causal ? j : 0;
  nq = p.nkb - q0;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
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
  uint64_t* ld_full = bars + 7;     // lse_i, di_i landed (loaded once the row warps finished i - 1)
  uint64_t* s_ready = bars + 8;     // S^T in TMEM (and every earlier MMA done)
  uint64_t* dp_ready = bars + 9;    // dP^T in TMEM
  uint64_t* p_ready = bars + 10;    // P^T in shared memory (128 arrivals)
  uint64_t* ds_ready = bars + 11;   // dS^T in shared memory (128 arrivals)
  uint64_t* dq_ready = bars + 12;   // dQ_i in TMEM
  uint64_t* dq_free = bars + 13;    // dQ_i read out of TMEM (128 arrivals)
  uint64_t* dkv_ready = bars + 14;  // every MMA done: dV_j, dK_j final
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 15);

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
    mbar_init(ld_full, 1);
    mbar_init(s_ready, 1);
    mbar_init(dp_ready, 1);
    mbar_init(p_ready, 128);
    mbar_init(ds_ready, 128);
    mbar_init(dq_ready, 1);
    mbar_init(dq_free, 128);
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
  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));

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
        const int h = g * p.rep + it / nq;
        const int s0 = (q0 + it % nq) * kBlk;
        const int qb = it & 1;
        const int64_t drow = (static_cast<int64_t>(b) * p.QH + h) * p.S + s0;  // dout / lse / di row
        // Q_i into buffer i % 2 once dK of block i - 2 is done
        if (it >= 2) ok = mbar_wait(&q_free[qb], static_cast<uint32_t>((it >> 1) - 1) & 1u, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(&q_full[qb], kTile);
        for (int hh = 0; hh < 2; ++hh)
          tma_load_4d(smem + Smem::kQ + qb * kTile + hh * kHalf, &tmQ, &q_full[qb], hh * 64, h, s0, b);
        q_issued |= 1u << qb;
        // dO_i once dV of block i - 1 is done
        if (it >= 1) ok = mbar_wait(do_free, static_cast<uint32_t>(it - 1) & 1u, err, kErrWaitEmpty);
        if (!ok) break;
        mbar_arrive_expect_tx(do_full, kTile);
        for (int hh = 0; hh < 2; ++hh)
          tma_load_2d(smem + Smem::kDO + hh * kHalf, &tmDO, do_full, hh * 64, static_cast<int>(drow));
        // lse_i, di_i once the row warps are done with block i - 1
        if (it >= 1) ok = mbar_wait(ds_ready, static_cast<uint32_t>(it - 1) & 1u, err, kErrWaitEmpty);
        if (!ok) break;
        const int valid = p.S - s0 < kBlk ? p.S - s0 : kBlk;  // query rows of the block inside S
        const uint32_t vbytes = static_cast<uint32_t>(valid) * 4u;
        mbar_arrive_expect_tx(ld_full, 2 * vbytes);
        bulk_load_1d(smem + Smem::kLse, p.lse + drow, vbytes, ld_full);
        bulk_load_1d(smem + Smem::kDi, p.di + drow, vbytes, ld_full);
      }
      // no copy may still be writing shared memory when the CTA exits
      if (ok) ok = mbar_wait(kv_full, 0u, err, kErrWaitDrain);
      if (ok && n_iter > 0) {
        const uint32_t last = static_cast<uint32_t>(n_iter - 1);
        mbar_wait(do_full, last & 1u, err, kErrWaitDrain);
        mbar_wait(ld_full, last & 1u, err, kErrWaitDrain);
        for (int t = 0; t < 2; ++t)
          if (q_issued & (1u << t)) {
            const uint32_t lt = (last & 1u) == static_cast<uint32_t>(t) ? last : last - 1u;  // last use of buffer t
            mbar_wait(&q_full[t], (lt >> 1) & 1u, err, kErrWaitDrain);
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
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
      bool ok = mbar_wait(kv_full, 0u, err, kErrWaitFull);
      bool any = false;
      for (int it = 0; it < n_iter && ok; ++it) {
        const uint32_t par = static_cast<uint32_t>(it) & 1u;
        const int qb = it & 1;
        const uint64_t kQb = kQ + static_cast<uint64_t>(qb * (kTile >> 4)), mQb = mQ + static_cast<uint64_t>(qb * (kTile >> 4));
        // S^T = K_j Q_i^T (its columns were last read by the row warps for
        // block i - 1, before the dV of that block was issued)
        ok = mbar_wait(&q_full[qb], static_cast<uint32_t>(it >> 1) & 1u, err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) umma_bf16(tmem + 0, kK + ko(kk), kQb + ko(kk), kIdKK, kk != 0);
        umma_commit(s_ready);
        any = true;
        // dP^T = V_j dO_i^T, into the columns of block i - 1's dQ once it is read
        ok = mbar_wait(do_full, par, err, kErrWaitFull);
        if (ok && it > 0) ok = mbar_wait(dq_free, par ^ 1u, err, kErrWaitAccumFree);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) umma_bf16(tmem + 128, kV + ko(kk), kDO + ko(kk), kIdKK, kk != 0);
        umma_commit(dp_ready);
        // dV_j += P^T dO_i
        ok = mbar_wait(p_ready, par, err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          umma_bf16(tmem + 256, kP + ko(kk), mDO + mo(kk), kIdKM, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(do_free);
        // dK_j += dS^T Q_i, then dQ_i = dS K_j into dP^T's columns
        ok = mbar_wait(ds_ready, par, err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk)
          umma_bf16(tmem + 384, kDS + ko(kk), mQb + mo(kk), kIdKM, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&q_free[qb]);
#pragma unroll
        for (int kk = 0; kk < kBlk / 16; ++kk) umma_bf16(tmem + 128, mDS + mo(kk), mK + mo(kk), kIdMM, kk != 0);
        umma_commit(dq_ready);
      }
      if (any) {
        umma_commit(dkv_ready);
        // every issued MMA must finish before TMEM is released
        mbar_wait(dkv_ready, 0u, err, kErrWaitDrain);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------- row warps
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsRow));
    const int kr = (warp & 3) * 32 + lane;  // key row of this thread (TMEM lane)
    const int kpos = j * kBlk + kr;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float* lse_s = reinterpret_cast<const float*>(smem + Smem::kLse);
    const float* di_s = reinterpret_cast<const float*>(smem + Smem::kDi);
    const uint32_t prow = smem_u32(smem + Smem::kP) + static_cast<uint32_t>(kr * 128);
    const uint32_t dsrow = smem_u32(smem + Smem::kDS) + static_cast<uint32_t>(kr * 128);
    const uint32_t rsw = static_cast<uint32_t>(kr & 7);
    bool ok = true;
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t par = static_cast<uint32_t>(it) & 1u;
      const int s0 = (q0 + it % nq) * kBlk;
      ok = mbar_wait(s_ready, par, err, kErrWaitAccum) && mbar_wait(ld_full, par, err, kErrWaitFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // P^T row: 2^(s * scale log2e - lse[q]); zero for keys / queries past S
      // and (causal) keys after the query.  32 queries at a time: 16 packed
      // words, stored as four 16-byte units of the K-major, 128-byte-swizzled
      // P^T tile (queries [8u, 8u + 8) of a 64-query half = unit u)
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32];
        tmem_ld_32x32b_x32(tmem + lane_base + c * 32, sv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float e[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int qc = c * 32 + 2 * i + u;
            const int qpos = s0 + qc;
            const bool live = kpos < p.S && qpos < p.S && (!p.causal || kpos <= qpos);
            e[u] = live ? exp2_approx(fmaf(__uint_as_float(sv[2 * i + u]), p.sl2, -lse_s[qc])) : 0.f;
          }
          pk[c * 16 + i] = pack_bf16x2(e[0], e[1]);
        }
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = (c & 1) * 4 + u4;  // unit within the half
          const int i = c * 16 + u4 * 4;
          st_shared_v4(prow + (c >> 1) * kHalf + ((static_cast<uint32_t>(u) ^ rsw) << 4), pk[i], pk[i + 1],
                       pk[i + 2], pk[i + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
      // dS^T row: P^T (dP^T - di[q]) scale
      ok = mbar_wait(dp_ready, par, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t dv[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 128 + c * 32, dv);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const __nv_bfloat162 pp = *reinterpret_cast<const __nv_bfloat162*>(&pk[c * 16 + i]);
          const float2 pf = __bfloat1622float2(pp);
          const int qc = c * 32 + 2 * i;
          // a masked entry (P = 0) stays 0 whatever di holds past S
          w[i] = pack_bf16x2(pf.x != 0.f ? pf.x * (__uint_as_float(dv[2 * i]) - di_s[qc]) * p.scale : 0.f,
                             pf.y != 0.f ? pf.y * (__uint_as_float(dv[2 * i + 1]) - di_s[qc + 1]) * p.scale : 0.f);
        }
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = (c & 1) * 4 + u4;
          st_shared_v4(dsrow + (c >> 1) * kHalf + ((static_cast<uint32_t>(u) ^ rsw) << 4), w[4 * u4], w[4 * u4 + 1],
                       w[4 * u4 + 2], w[4 * u4 + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    // dV_j, dK_j (bf16) once every MMA is done (every key block visits at
    // least one query block)
    if (ok) ok = mbar_wait(dkv_ready, 0u, err, kErrWaitAccum);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        __nv_bfloat16* dst = (which == 0 ? p.dv : p.dk) +
                             ((static_cast<int64_t>(b) * p.S + kpos) * p.KH + g) * kD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256 + which * 128 + c * 32, r);
          tmem_ld_wait();
          if (kpos < p.S) {
            uint4* o = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              o[q] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1])),
                                pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                                pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                                pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
          }
        }
      }
    }
  } else if (warp >= 8) {
    // ----------------------------------------------------------- dQ warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsDq));
    const int qr = (warp & 3) * 32 + lane;  // query row of this thread (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_iter && ok; ++it) {
      const uint32_t par = static_cast<uint32_t>(it) & 1u;
      const int h = g * p.rep + it / nq;
      const int qpos = (q0 + it % nq) * kBlk + qr;
      ok = mbar_wait(dq_ready, par, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float* dst = p.dq + ((static_cast<int64_t>(b) * p.S + qpos) * p.QH + h) * kD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 128 + c * 32, r);
        tmem_ld_wait();
        if (qpos < p.S) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + c * 32 + 4 * q),
                         "f"(__uint_as_float(r[4 * q])), "f"(__uint_as_float(r[4 * q + 1])),
                         "f"(__uint_as_float(r[4 * q + 2])), "f"(__uint_as_float(r[4 * q + 3]))
                         : "memory");
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// fp32 [rows][128] -> bf16, 8 values per thread
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                                          int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  const float4 a = reinterpret_cast<const float4*>(x)[2 * i], c = reinterpret_cast<const float4*>(x)[2 * i + 1];
  reinterpret_cast<uint4*>(y)[i] =
      make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(c.x, c.y), pack_bf16x2(c.z, c.w));
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
  f32_to_bf16_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, st>>>(dq32, dq, n8);
  return launch_status("attn_backward: dq to bf16");
}

}  // namespace kda
