// Grouped-query attention forward (head_dim 128) on tcgen05 tensor cores.
//
// Work unit = (batch b, query head h, 256 query rows as two 128-row tiles).
// One CTA per SM, persistent over units ordered heaviest-first (causal),
// 384 threads:
//   warp 0       TMA producer: the two Q tiles once per unit, then the K/V
//                tiles through a 3-slot ring in the order they are used:
//                K_0, then K_{j+1}, V_j for j = 0, 1, ...  V is read from a
//                transposed copy V^T [B][KH][128][S] made by a pre-pass, so
//                every MMA reads a K-major B operand (alternating K-major and
//                MN-major B operands costs the tensor core about a quarter of
//                its throughput).
//   warp 1       TMEM allocator + MMA issuer: S_t = Q_t K_0^T for both tiles,
//                then per block j  S_t = Q_t K_{j+1}^T (t = 0, 1) and
//                O_t (+)= P_t V_j (t = 0, 1), all SS form (operands in shared
//                memory).  Each group of 16 MMAs ends with one commit that
//                releases its K or V ring slot; that release is also the
//                signal "S(j+1) ready" / "O += P V_j done" for the softmax.
//                The issuing thread touches no shared memory: a shared-memory
//                access (an mbarrier wait included) from the thread that
//                issues tcgen05.mma stalls behind the queued MMAs and idles
//                the tensor core for a few hundred cycles.
//   warp 2       scheduler: performs every mbarrier wait the MMA issuer needs
//                (Q and ring slots loaded, S copied out by both softmax
//                warpgroups, P written) and releases the MMA warp group by
//                group through a named barrier (bar.red, which also carries an
//                ok flag so an expired wait stops both warps together).
//   warp 3       idle (completes warpgroup 0, which hands its registers to the
//                softmax warpgroups through setmaxnreg)
//   warps 4-7    softmax warpgroup for Q tile 0, warps 8-11 for Q tile 1; the
//                two run concurrently.  One query row per thread: the whole
//                128-key S row is loaded from TMEM into registers (its TMEM
//                columns are then released to the next QK) -> causal / length
//                mask -> row max -> online max with lazy rescale (O only
//                corrected when the running max grows by more than 2^8) ->
//                P = 2^(s - m) as bf16 in registers (2 of every 16 pairs of
//                exponentials by a polynomial on the FMA pipe, the rest by ex2
//                on the MUFU pipe) -> (once PV(j-1) is done)
//                into shared memory in the 128-byte swizzled K-major layout
//                the MMA reads; after the last block O / l -> bf16 -> global.
// TMEM columns: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512).
// Shared memory: Q0 | Q1 | P0 | P1 | ring (3 x 32 KB) = 224 KB.
// K/V tiles of query head h come from kv head h / (QH/KH) (GQA sharing
// through L2).  RoPE (optional) is applied by a pre-pass that rotates q and k
// once into the caller's workspace using a cos/sin table built in double
// precision.  All mbarrier waits are bounded (common.cuh); every TMA load
// targets one CTA.
#include <math.h>

#include "common.cuh"

KDA_DEFINE_ERROR_WORD(attn)

namespace kda {
namespace {

constexpr int kD = 128;           // head dim
constexpr int kBlk = 128;         // rows per Q tile and keys per K/V block
constexpr int kSlots = 3;         // K/V ring depth
constexpr uint32_t kTile = kBlk * kD * 2;  // 32 KB: one Q, P, K or V^T tile
constexpr uint32_t kHalf = kTile / 2;      // one 64-column half of a tile
constexpr int kThreads = 384;  // 3 warpgroups
// Register split (setmaxnreg): warpgroup 0 (TMA, MMA, scheduler and an idle
// warp) gives registers to the two softmax warpgroups.  The shares add up to
// the launch allocation exactly: 384 x 168 = 128 x 104 + 256 x 200 = 64512,
// so the kernel must be compiled to 168 registers per thread (checked before
// launch; an increase beyond the launch allocation would wait forever).
constexpr int kRegsLaunch = 168;
constexpr int kRegsLow = 104;
constexpr int kRegsHigh = 200;
static_assert(kThreads * kRegsLaunch >= 128 * kRegsLow + 256 * kRegsHigh, "register split must fit the launch");
__host__ __device__ constexpr uint32_t col_s(int t) { return t ? 128u : 0u; }
__host__ __device__ constexpr uint32_t col_o(int t) { return t ? 384u : 256u; }
constexpr uint32_t kTmemCols = 512;
constexpr int kGoBarrier = 1;  // named barrier: scheduler warp + MMA warp
// Pairs of keys (bit i of 16) whose exponentials are computed by a polynomial
// on the FMA pipe instead of ex2 on the MUFU pipe: both softmax warpgroups
// share one MUFU pipe per SM partition, which otherwise bounds the softmax.
constexpr uint32_t kPolyPairs = 0x0101u;  // pairs 0 and 8

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

struct AttnParams {
  int B, S, QH, KH, n_rep;
  int npairs;       // 256-row query units per head
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  int64_t out_row_stride;   // elements between consecutive query rows
  int64_t out_head_stride;  // elements between heads (same position)
  int64_t out_batch_stride;
  float* lse;  // optional [B][QH][S]: each row's log2-sum-exp of the scaled scores (for the backward)
};

// smem: Q0 | Q1 | P0 | P1 | ring (kSlots x 32 KB) | barriers.  Every tile is
// two 16 KB halves of 64 columns, 128-byte rows, 128-byte swizzle.
struct Smem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kP = 2 * kTile;
  static constexpr uint32_t kRing = 4 * kTile;
  static constexpr uint32_t kBars = kRing + kSlots * kTile;
  // slot_full[kSlots] slot_free[kSlots] q_full s_free p_full drain holder
  static constexpr uint32_t kNumBars = 2 * kSlots + 5;
  static constexpr size_t kBytes = 1024 + kBars + kNumBars * 8 + 16;
  static_assert(kBytes > 116 * 1024 && kBytes <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void unit_coords(int u, const AttnParams& p, int& b, int& h, int& qp) {
  const int heads = p.B * p.QH;
  const int level = u / heads;  // heaviest (last) query units first
  const int bh = u - level * heads;
  qp = p.causal ? (p.npairs - 1 - level) : level;
  b = bh / p.QH;
  h = bh - b * p.QH;
}

// K/V blocks a unit visits: both tiles share the count; tile 0 sees its last
// block fully masked when causal.
__device__ __forceinline__ int num_kv_blocks(const AttnParams& p, int qp) {
  const int all = (p.S + kBlk - 1) / kBlk;
  const int need = 2 * qp + 2;
  return p.causal ? (need < all ? need : all) : all;
}

// Ring items of a unit with nb blocks, in load order K_0, K_1, V_0, K_2, V_1,
// ..., K_{nb-1}, V_{nb-2}, V_{nb-1}; `base` counts the items of earlier units.
// Item x lives in slot x % kSlots; its slot's barriers complete once per item,
// so the phase of item x is (x / kSlots) & 1.
__device__ __forceinline__ uint32_t item_k(uint32_t base, int j) {
  return base + (j == 0 ? 0u : 2u * static_cast<uint32_t>(j) - 1u);
}
__device__ __forceinline__ uint32_t item_v(uint32_t base, int j, int nb) {
  return base + (j == nb - 1 ? 2u * static_cast<uint32_t>(nb) - 1u : 2u * static_cast<uint32_t>(j) + 2u);
}
__device__ __forceinline__ uint32_t item_slot(uint32_t x) { return x % kSlots; }
__device__ __forceinline__ uint32_t item_par(uint32_t x) { return (x / kSlots) & 1u; }

__global__ void __launch_bounds__(kThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnParams p, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::kBars);
  uint64_t* slot_full = bars;            // [kSlots] TMA bytes landed
  uint64_t* slot_free = bars + kSlots;   // [kSlots] MMA group that read the slot is done
  uint64_t* q_full = bars + 2 * kSlots;  // both Q tiles landed
  uint64_t* s_free = q_full + 1;         // both softmax warpgroups copied S out of TMEM (8 warps)
  uint64_t* p_full = q_full + 2;         // both softmax warpgroups wrote P (8 warps)
  uint64_t* drain = q_full + 3;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(q_full + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_free[s], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(s_free, 8);  // one arrival per softmax warp
    mbar_init(p_full, 8);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int units = p.B * p.QH * p.npairs;
  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    uint32_t base = 0, prev_qk_last = 0;
    uint32_t issued = 0, last_par = 0;
    bool ok = true;
    bool first = true;
    // Load ring item x: a K tile (keys [j*128, +128) x d) or a V^T tile (d x
    // the same keys), as two 64-column halves.
    auto load_item = [&](uint32_t x, bool is_v, int kvh, int j, int b) -> bool {
      const uint32_t s = item_slot(x);
      bool good = true;
      if (lane == 0) good = mbar_wait(&slot_free[s], item_par(x) ^ 1u, err, kErrWaitEmpty);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) return false;
      if (lane == 0) {
        uint8_t* dst = smem + Smem::kRing + s * kTile;
        mbar_arrive_expect_tx(&slot_full[s], kTile);
        if (is_v) {
          tma_load_4d(dst, &tmV, &slot_full[s], j * kBlk, 0, kvh, b);
          tma_load_4d(dst + kHalf, &tmV, &slot_full[s], j * kBlk + 64, 0, kvh, b);
        } else {
          tma_load_4d(dst, &tmK, &slot_full[s], 0, kvh, j * kBlk, b);
          tma_load_4d(dst + kHalf, &tmK, &slot_full[s], 64, kvh, j * kBlk, b);
        }
        issued |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (item_par(x) << s);
      }
      return true;
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, h, qp;
      unit_coords(u, p, b, h, qp);
      const int kvh = h / p.n_rep;
      const int nb = num_kv_blocks(p, qp);
      // Q is free once the previous unit's last QK group (which read its
      // last K item) is done
      if (!first && lane == 0) ok = mbar_wait(&slot_free[item_slot(prev_qk_last)], item_par(prev_qk_last), err,
                                              kErrWaitEmpty);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      first = false;
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, 2 * kTile);
        for (int t = 0; t < 2; ++t) {
          const int row = qp * 2 * kBlk + t * kBlk;
          tma_load_4d(smem + Smem::kQ + t * kTile, &tmQ, q_full, 0, h, row, b);
          tma_load_4d(smem + Smem::kQ + t * kTile + kHalf, &tmQ, q_full, 64, h, row, b);
        }
      }
      ok = load_item(item_k(base, 0), false, kvh, 0, b);
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb) ok = load_item(item_k(base, j + 1), false, kvh, j + 1, b);
        if (ok) ok = load_item(item_v(base, j, nb), true, kvh, j, b);
      }
      prev_qk_last = item_k(base, nb - 1);
      base += 2u * static_cast<uint32_t>(nb);
    }
    if (lane == 0) {
      for (int s = 0; s < kSlots; ++s)
        if (issued & (1u << s)) mbar_wait(&slot_full[s], (last_par >> s) & 1u, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ---------------------------------------------- MMA issuer / scheduler
    // Both warps walk the same schedule of 16-MMA groups and meet at the go
    // barrier before each one.
    const bool sched = warp == 2;
    constexpr uint32_t kIdQK = idesc_bf16_f32(kBlk, kBlk, 0, 0);
    constexpr uint32_t kIdPV = idesc_bf16_f32(kBlk, kD, 0, 0);
    uint32_t base = 0, gb = 0;  // ring items and blocks of earlier units
    int uc = 0;
    bool ok = true;
    bool any = false;
    // scheduler: wait for the inputs of one group (lane 0), then meet the MMA warp
    auto sched_wait = [&](uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2, uint64_t* b3, uint32_t p3) -> bool {
      bool good = true;
      if (lane == 0) {
        if (b1) good = mbar_wait(b1, p1, err, kErrWaitFull);
        if (good && b2) good = mbar_wait(b2, p2, err, kErrWaitFull);
        if (good && b3) good = mbar_wait(b3, p3, err, kErrWaitAccum);
      }
      return go_barrier64<kGoBarrier>(__shfl_sync(0xffffffffu, good, 0));
    };
    // S_t = Q_t K^T for both tiles from ring item x, then release the item
    auto qk_group = [&](uint32_t x) {
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(smem + Smem::kRing + item_slot(x) * kTile);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t q_addr = smem_u32(smem + Smem::kQ + t * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_bf16(tmem + col_s(t), smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), kIdQK, kk != 0 ? 1u : 0u);
          }
        }
        umma_commit(&slot_free[item_slot(x)]);
      }
      __syncwarp();
    };
    // O_t (+)= P_t V^T-tile for both tiles from ring item x, then release it
    auto pv_group = [&](uint32_t x, bool first) {
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(smem + Smem::kRing + item_slot(x) * kTile);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint32_t p_addr = smem_u32(smem + Smem::kP + t * kTile);
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_bf16(tmem + col_o(t), smem_desc_sw128(p_addr + off, 16, 1024),
                      smem_desc_sw128(v_addr + off, 16, 1024), kIdPV, (!first || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&slot_free[item_slot(x)]);
      }
      __syncwarp();
    };
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
      int b, h, qp;
      unit_coords(u, p, b, h, qp);
      const int nb = num_kv_blocks(p, qp);
      // group: S = Q K_0^T (needs Q, K_0, and S released by the softmax of
      // the previous block, if any)
      {
        const uint32_t x = item_k(base, 0);
        if (sched) {
          ok = sched_wait(q_full, static_cast<uint32_t>(uc) & 1u, &slot_full[item_slot(x)], item_par(x),
                          gb > 0 ? s_free : nullptr, (gb - 1u) & 1u);
        } else {
          ok = go_barrier64<kGoBarrier>(true);
          if (ok) {
            tc_fence_after();
            qk_group(x);
            any = true;
          }
        }
        if (!ok) break;
      }
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb) {
          // S = Q K_{j+1}^T once both softmax warpgroups copied S(j) out
          const uint32_t x = item_k(base, j + 1);
          if (sched) {
            ok = sched_wait(&slot_full[item_slot(x)], item_par(x), s_free, (gb + j) & 1u, nullptr, 0u);
          } else {
            ok = go_barrier64<kGoBarrier>(true);
            if (ok) {
              tc_fence_after();
              qk_group(x);
            }
          }
          if (!ok) break;
        }
        // O += P(j) V_j once both softmax warpgroups wrote P(j)
        const uint32_t x = item_v(base, j, nb);
        if (sched) {
          ok = sched_wait(&slot_full[item_slot(x)], item_par(x), p_full, (gb + j) & 1u, nullptr, 0u);
        } else {
          ok = go_barrier64<kGoBarrier>(true);
          if (ok) {
            tc_fence_after();
            pv_group(x, j == 0);
          }
        }
      }
      base += 2u * static_cast<uint32_t>(nb);
      gb += static_cast<uint32_t>(nb);
    }
    // every issued MMA must finish before TMEM is released
    if (!sched && lane == 0 && any) {
      umma_commit(drain);
      mbar_wait(drain, 0, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // --------------------------------------------------- softmax / epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    const int t = (warp - 4) >> 2;  // Q tile of this warpgroup
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t scol = tmem + lane_base + col_s(t);
    const uint32_t ocol = tmem + lane_base + col_o(t);
    // this thread's 128-byte row in each 16 KB half of P_t; 16-byte unit u of
    // the row sits at ((u ^ (r & 7)) * 16) (128-byte swizzle)
    const uint32_t prow = smem_u32(smem + Smem::kP + t * kTile) + r * 128;
    const uint32_t rsw = r & 7;
    uint32_t base = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, h, qp;
      unit_coords(u, p, b, h, qp);
      const int nb = num_kv_blocks(p, qp);
      const int q0 = qp * 2 * kBlk + t * kBlk;  // first query row of this tile
      const int qpos = q0 + r;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nb; ++j) {
        // S(j) is ready once the QK group that read K_j released its slot
        const uint32_t xk = item_k(base, j);
        ok = mbar_wait(&slot_free[item_slot(xk)], item_par(xk), err, kErrWaitAccum);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // the whole 128-key row of S_t in registers, then hand the columns
        // back for S(j+1)
        uint32_t sv[kBlk];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tmem_ld_32x32b_x32(scol + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[c * 32]));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive_warp(s_free);
        const int k0 = j * kBlk;
        // masks only touch the diagonal / ragged blocks (block-uniform branch)
        const bool masked_blk = (p.causal && k0 + kBlk - 1 > q0) || (k0 + kBlk > p.S);
        if (masked_blk) {
          const int lim_c = p.causal ? qpos - k0 + 1 : kBlk;
          const int lim_s = p.S - k0;
          const int lim = lim_c < lim_s ? lim_c : lim_s;  // keys [k0, k0 + lim) are visible
#pragma unroll
          for (int i = 0; i < kBlk; ++i)
            if (i >= lim) sv[i] = 0xff800000u;  // -inf
        }
        // raw row max (the scale is positive): 3-input max, eight chains
        float mxa[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mxa[k] = fmaxf(__uint_as_float(sv[k]), __uint_as_float(sv[k + 8]));
#pragma unroll
        for (int i = 16; i < kBlk; i += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) mxa[k] = fmax3(mxa[k], __uint_as_float(sv[i + k]), __uint_as_float(sv[i + 8 + k]));
        const float mx = fmax3(fmax3(mxa[0], mxa[1], mxa[2]), fmax3(mxa[3], mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])) *
                         p.scale_log2;
        const float m_new = fmaxf(m_run, mx);
        bool rescale = false;
        float factor = 1.f;
        if (j == 0) {
          m_run = m_new;
        } else if (m_new > m_run + 8.0f) {
          factor = exp2_approx(m_run - m_new);
          m_run = m_new;
          rescale = true;
        }
        const float mb = (m_run == -INFINITY) ? 0.f : m_run;
        // P = 2^(s * scale - m) as bf16, all 128 keys in registers
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nm2 = make_float2(-mb, -mb);
        float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};  // independent chains
        uint32_t pk[kBlk / 2];
#pragma unroll
        for (int i = 0; i < kBlk / 2; ++i) {
          const float2 v = make_float2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
          const float2 a = __ffma2_rn(v, sc2, nm2);
          const float2 e = ((kPolyPairs >> (i & 15)) & 1u) ? exp2_poly2_lp(a)
                                                            : make_float2(exp2_approx(a.x), exp2_approx(a.y));
          sum2[i & 3] = __fadd2_rn(sum2[i & 3], e);
          pk[i] = pack_bf16x2(e.x, e.y);
        }
        const float sum = ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y)) +
                          ((sum2[2].x + sum2[2].y) + (sum2[3].x + sum2[3].y));
        l_run = l_run * factor + sum;
        // O += P(j-1) V_{j-1} must be done before P is overwritten or O
        // rescaled (for j == 0 the previous unit's epilogue already waited)
        if (j > 0) {
          const uint32_t xv = item_v(base, j - 1, nb);
          ok = mbar_wait(&slot_free[item_slot(xv)], item_par(xv), err, kErrWaitAccum);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
        }
        const bool any_rescale = __any_sync(0xffffffffu, rescale);
        if (any_rescale) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t rr[32];
            tmem_ld_32x32b_x32(ocol + c * 32, rr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * factor);
            tmem_st_32x32b_x32(ocol + c * 32, rr);
          }
        }
        // keys [8u, 8u + 8) of half h: 16-byte unit u of this row, swizzled
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int uu = 0; uu < 8; ++uu) {
            const int i = hh * 32 + uu * 4;
            st_shared_v4(prow + hh * kHalf + ((static_cast<uint32_t>(uu) ^ rsw) << 4), pk[i], pk[i + 1], pk[i + 2],
                         pk[i + 3]);
          }
        fence_proxy_async_smem();
        if (any_rescale) tmem_st_wait();
        tc_fence_before();
        mbar_arrive_warp(p_full);
      }
      if (!ok) break;
      // epilogue: O_t / l -> bf16 -> global, once the last PV group is done
      const uint32_t xv = item_v(base, nb - 1, nb);
      ok = mbar_wait(&slot_free[item_slot(xv)], item_par(xv), err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      if (p.lse && qpos < p.S)
        p.lse[(static_cast<int64_t>(b) * p.QH + h) * p.S + qpos] = (m_run == -INFINITY ? 0.f : m_run) + __log2f(l_run);
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(b) * p.out_batch_stride +
                            static_cast<int64_t>(h) * p.out_head_stride + static_cast<int64_t>(qpos) * p.out_row_stride;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rr[32];
        tmem_ld_32x32b_x32(ocol + c * 32, rr);
        tmem_ld_wait();
        if (qpos < p.S) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(rr[8 * q + 0]) * inv_l, __uint_as_float(rr[8 * q + 1]) * inv_l);
            v.y = pack_bf16x2(__uint_as_float(rr[8 * q + 2]) * inv_l, __uint_as_float(rr[8 * q + 3]) * inv_l);
            v.z = pack_bf16x2(__uint_as_float(rr[8 * q + 4]) * inv_l, __uint_as_float(rr[8 * q + 5]) * inv_l);
            v.w = pack_bf16x2(__uint_as_float(rr[8 * q + 6]) * inv_l, __uint_as_float(rr[8 * q + 7]) * inv_l);
            dst[q] = v;
          }
        }
      }
      base += 2u * static_cast<uint32_t>(nb);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ RoPE
// cos/sin table [S][64] (double-precision angles, rounded to fp32).
__global__ void rope_table_kernel(float2* __restrict__ tab, int S, double log2_theta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S * (kD / 2)) return;
  const int pos = i / (kD / 2), f = i % (kD / 2);
  const double inv_freq = exp2(-(2.0 * f / kD) * log2_theta);
  double sn, cs;
  sincos(static_cast<double>(pos) * inv_freq, &sn, &cs);
  tab[i] = make_float2(static_cast<float>(cs), static_cast<float>(sn));
}

// x [B,S,H,128] bf16 -> out (same layout), half-split rotation (INV: by the
// negated angle, the transpose of the rotation); one thread per (row, 8
// consecutive frequencies).
template <bool INV>
__global__ void rope_rotate_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out,
                                   const float2* __restrict__ tab, int64_t rows, int S, int H) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * 8) return;
  const int64_t row = t / 8;
  const int f0 = static_cast<int>(t % 8) * 8;
  const int pos = static_cast<int>((row / H) % S);
  const __nv_bfloat16* xr = x + row * kD;
  const uint4 a = *reinterpret_cast<const uint4*>(xr + f0);
  const uint4 c = *reinterpret_cast<const uint4*>(xr + 64 + f0);
  const __nv_bfloat16* a16 = reinterpret_cast<const __nv_bfloat16*>(&a);
  const __nv_bfloat16* c16 = reinterpret_cast<const __nv_bfloat16*>(&c);
  float o0[8], o1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 cs = tab[pos * (kD / 2) + f0 + i];
    const float sn = INV ? -cs.y : cs.y;
    const float x0 = __bfloat162float(a16[i]), x1 = __bfloat162float(c16[i]);
    o0[i] = x0 * cs.x - x1 * sn;
    o1[i] = x0 * sn + x1 * cs.x;
  }
  uint4 r0, r1;
  r0.x = pack_bf16x2(o0[0], o0[1]); r0.y = pack_bf16x2(o0[2], o0[3]);
  r0.z = pack_bf16x2(o0[4], o0[5]); r0.w = pack_bf16x2(o0[6], o0[7]);
  r1.x = pack_bf16x2(o1[0], o1[1]); r1.y = pack_bf16x2(o1[2], o1[3]);
  r1.z = pack_bf16x2(o1[4], o1[5]); r1.w = pack_bf16x2(o1[6], o1[7]);
  __nv_bfloat16* orow = out + row * kD;
  *reinterpret_cast<uint4*>(orow + f0) = r0;
  *reinterpret_cast<uint4*>(orow + 64 + f0) = r1;
}

// ------------------------------------------------------------- V^T copy
// v [B][S][KH][128] -> vt [B][KH][128][S8] (S8 = S rounded up to 8 so rows
// are 16-byte aligned for TMA; keys [S, S8) are written as zeros).  One CTA
// per (64 keys, kv head, batch): the tile goes through padded shared memory
// so both the reads and the writes are 16-byte coalesced.
constexpr int kTrKeys = 64;
__global__ void __launch_bounds__(256) v_transpose_kernel(const __nv_bfloat16* __restrict__ v,
                                                          __nv_bfloat16* __restrict__ vt, int S, int S8, int KH) {
  __shared__ __align__(16) __nv_bfloat16 tile[kTrKeys][kD + 8];
  const int s0 = blockIdx.x * kTrKeys;
  const int kvh = blockIdx.y, b = blockIdx.z;
  // read 64 rows of 256 bytes (16 units of 8 values per row)
  for (int i = threadIdx.x; i < kTrKeys * 16; i += 256) {
    const int row = i >> 4, unit = i & 15;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (s0 + row < S)
      val = *reinterpret_cast<const uint4*>(v + ((static_cast<int64_t>(b) * S + s0 + row) * KH + kvh) * kD + unit * 8);
    *reinterpret_cast<uint4*>(&tile[row][unit * 8]) = val;
  }
  __syncthreads();
  // write 128 rows (d) of 64 keys: 8 units of 8 keys per row
  __nv_bfloat16* dst = vt + (static_cast<int64_t>(b) * KH + kvh) * kD * S8;
  for (int i = threadIdx.x; i < kD * (kTrKeys / 8); i += 256) {
    const int d = i >> 3, unit = i & 7;
    const int k = s0 + unit * 8;
    if (k >= S8) continue;
    __align__(16) __nv_bfloat16 w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = tile[unit * 8 + e][d];
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(d) * S8 + k) = *reinterpret_cast<const uint4*>(w);
  }
}

inline size_t al256(size_t n) { return (n + 255) & ~size_t(255); }
inline int64_t keys8(int64_t S) { return (S + 7) & ~int64_t(7); }

// [B][S][H][128] as a 4-D map {128, H, S, B} (rows past S read as zeros);
// box {64, 1, 128, 1}.
kda_status tmap_heads(CUtensorMap* m, const void* base, int64_t B, int64_t S, int64_t H) {
  const uint64_t dims[4] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(H), static_cast<uint64_t>(S),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(kD) * 2, static_cast<uint64_t>(H) * kD * 2,
                               static_cast<uint64_t>(S) * H * kD * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(kBlk), 1};
  return make_tmap_bf16(m, base, 4, dims, strides, box);
}

// V^T [B][KH][128][S8] as a 4-D map {S8, 128, KH, B}; box {64, 128, 1, 1}
// (keys past S8 read as zeros).
kda_status tmap_vt(CUtensorMap* m, const void* base, int64_t B, int64_t S8, int64_t KH) {
  const uint64_t dims[4] = {static_cast<uint64_t>(S8), static_cast<uint64_t>(kD), static_cast<uint64_t>(KH),
                            static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(S8) * 2, static_cast<uint64_t>(kD) * S8 * 2,
                               static_cast<uint64_t>(KH) * kD * S8 * 2};
  const uint32_t box[4] = {64, static_cast<uint32_t>(kD), 1, 1};
  return make_tmap_bf16(m, base, 4, dims, strides, box);
}

}  // namespace

// RoPE for the attention backward in another translation unit: the table of
// S positions x 64 frequencies (cos, sin) and the rotation of [rows][128]
// bf16 rows whose position is (row / H) % S, forward or inverse.
kda_status rope_table(float2* tab, int64_t S, float theta, cudaStream_t st) {
  const int64_t nt = S * (kD / 2);
  rope_table_kernel<<<static_cast<unsigned>((nt + 255) / 256), 256, 0, st>>>(tab, static_cast<int>(S),
                                                                             log2(static_cast<double>(theta)));
  return launch_status("rope_table_kernel");
}
kda_status rope_rotate_rows(const __nv_bfloat16* x, __nv_bfloat16* out, const float2* tab, int64_t rows, int64_t S,
                            int64_t H, bool inverse, cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((rows * 8 + 255) / 256);
  if (inverse)
    rope_rotate_kernel<true><<<grid, 256, 0, st>>>(x, out, tab, rows, static_cast<int>(S), static_cast<int>(H));
  else
    rope_rotate_kernel<false><<<grid, 256, 0, st>>>(x, out, tab, rows, static_cast<int>(S), static_cast<int>(H));
  return launch_status("rope_rotate_kernel");
}
}  // namespace kda

using namespace kda;

extern "C" size_t kda_gqa_full_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                              float rope_theta) {
  if (B <= 0 || S <= 0 || QH <= 0 || KH <= 0 || D != kD) return 0;
  // V^T, then (with RoPE) the rotated q and k and the cos/sin table
  size_t n = al256(static_cast<size_t>(B) * KH * kD * keys8(S) * 2);
  if (rope_theta > 0.f)
    n += al256(static_cast<size_t>(B) * S * QH * kD * 2) + al256(static_cast<size_t>(B) * S * KH * kD * 2) +
         al256(static_cast<size_t>(S) * (kD / 2) * 8);
  return n;
}

extern "C" kda_status kda_gqa_full_bf16(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S,
                                        int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  return kda::gqa_forward(q, k, v, out, B, S, QH, KH, D, causal, rope_theta, out_bshd, workspace, workspace_bytes,
                          nullptr, static_cast<cudaStream_t>(stream));
}

// The forward plus every query row's log2-sum-exp of the scaled scores,
// lse [B][QH][S] fp32 -- what kda_gqa_full_backward_saved_bf16 needs instead
// of recomputing the forward.
extern "C" kda_status kda_gqa_full_lse_bf16(const void* q, const void* k, const void* v, void* out, float* lse,
                                            int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D, int causal,
                                            float rope_theta, int out_bshd, void* workspace, size_t workspace_bytes,
                                            void* stream) {
  KDA_CHECK_ARG(lse, "gqa_full_lse: null lse pointer");
  KDA_CHECK_SUPPORTED((reinterpret_cast<uintptr_t>(lse) & 15u) == 0, "gqa_full_lse: lse must be 16-byte aligned");
  return kda::gqa_forward(q, k, v, out, B, S, QH, KH, D, causal, rope_theta, out_bshd, workspace, workspace_bytes,
                          lse, static_cast<cudaStream_t>(stream));
}

kda_status kda::gqa_forward(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S, int64_t QH,
                            int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd, void* workspace,
                            size_t workspace_bytes, float* lse, cudaStream_t stream) {
  KDA_CHECK_ARG(q && k && v && out, "gqa_full: null pointer");
  KDA_CHECK_ARG(B > 0 && S > 0 && QH > 0 && KH > 0 && QH % KH == 0 && B * S < (1ll << 31) / QH,
                "gqa_full: bad sizes B=%lld S=%lld QH=%lld KH=%lld", (long long)B, (long long)S, (long long)QH,
                (long long)KH);
  KDA_CHECK_SUPPORTED(D == kD, "gqa_full: head_dim must be 128, got %lld", (long long)D);
  KDA_CHECK_SUPPORTED(QH <= 65535 && KH <= 65535 && B <= 65535, "gqa_full: too many heads or batches");
  const bool al = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                    reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  KDA_CHECK_SUPPORTED(al, "gqa_full: pointers must be 16-byte aligned");
  const size_t need = kda_gqa_full_workspace_size(B, S, QH, KH, D, rope_theta);
  KDA_CHECK_ARG(workspace && workspace_bytes >= need, "gqa_full: workspace of %zu bytes required, got %zu", need,
                workspace_bytes);
  cudaStream_t st = stream;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  KDA_CHECK_SUPPORTED((reinterpret_cast<uintptr_t>(w) & 15u) == 0, "gqa_full: workspace must be 16-byte aligned");
  const int64_t S8 = keys8(S);
  auto* vt = reinterpret_cast<__nv_bfloat16*>(w);
  w += al256(static_cast<size_t>(B) * KH * kD * S8 * 2);
  v_transpose_kernel<<<dim3(static_cast<unsigned>((S + kTrKeys - 1) / kTrKeys), static_cast<unsigned>(KH),
                           static_cast<unsigned>(B)),
                       256, 0, st>>>(static_cast<const __nv_bfloat16*>(v), vt, static_cast<int>(S),
                                     static_cast<int>(S8), static_cast<int>(KH));
  if (launch_status("gqa_full v transpose") != KDA_OK) return KDA_CUDA_ERROR;
  const void* qs = q;
  const void* ks = k;
  if (rope_theta > 0.f) {
    auto* qr = reinterpret_cast<__nv_bfloat16*>(w);
    auto* kr = reinterpret_cast<__nv_bfloat16*>(w + al256(static_cast<size_t>(B) * S * QH * kD * 2));
    auto* tab = reinterpret_cast<float2*>(w + al256(static_cast<size_t>(B) * S * QH * kD * 2) +
                                          al256(static_cast<size_t>(B) * S * KH * kD * 2));
    const int nt = static_cast<int>(S * (kD / 2));
    rope_table_kernel<<<(nt + 255) / 256, 256, 0, st>>>(tab, static_cast<int>(S), log2(static_cast<double>(rope_theta)));
    const int64_t qrows = B * S * QH, krows = B * S * KH;
    rope_rotate_kernel<false><<<static_cast<unsigned>((qrows * 8 + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(q), qr, tab, qrows, static_cast<int>(S), static_cast<int>(QH));
    rope_rotate_kernel<false><<<static_cast<unsigned>((krows * 8 + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(k), kr, tab, krows, static_cast<int>(S), static_cast<int>(KH));
    if (launch_status("gqa_full rope") != KDA_OK) return KDA_CUDA_ERROR;
    qs = qr;
    ks = kr;
  }
  CUtensorMap tq, tk, tv;
  kda_status s;
  if ((s = tmap_heads(&tq, qs, B, S, QH)) != KDA_OK) return s;
  if ((s = tmap_heads(&tk, ks, B, S, KH)) != KDA_OK) return s;
  if ((s = tmap_vt(&tv, vt, B, S8, KH)) != KDA_OK) return s;
  AttnParams p{};
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.QH = static_cast<int>(QH);
  p.KH = static_cast<int>(KH);
  p.n_rep = static_cast<int>(QH / KH);
  p.npairs = static_cast<int>((S + 2 * kBlk - 1) / (2 * kBlk));
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(kD)));
  p.out = out;
  p.lse = lse;
  if (out_bshd) {
    p.out_row_stride = QH * kD;
    p.out_head_stride = kD;
    p.out_batch_stride = S * QH * kD;
  } else {
    p.out_row_stride = kD;
    p.out_head_stride = S * kD;
    p.out_batch_stride = QH * S * kD;
  }
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    // the setmaxnreg split only balances when the kernel launches with
    // exactly kRegsLaunch registers per thread
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, attn_kernel) != cudaSuccess) return launch_status("gqa_full: attributes");
    KDA_CHECK_SUPPORTED(fa.numRegs == kRegsLaunch,
                        "gqa_full: attention kernel compiled to %d registers/thread, its register split needs %d",
                        fa.numRegs, kRegsLaunch);
    if (cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Smem::kBytes)) != cudaSuccess)
      return launch_status("gqa_full: cudaFuncSetAttribute");
    attr_set[dev].store(true, std::memory_order_release);
  }
  const long long units = static_cast<long long>(B) * QH * p.npairs;
  const int grid = static_cast<int>(units < num_sms() ? units : num_sms());
  attn_kernel<<<grid, kThreads, Smem::kBytes, st>>>(tq, tk, tv, p, kda_err_ptr_attn());
  return launch_status("attn_kernel");
}
