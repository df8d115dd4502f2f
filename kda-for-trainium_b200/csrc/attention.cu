// Grouped-query attention forward (head_dim 128) on tcgen05 tensor cores.
//
// Work unit = (batch b, query head h, 128-query block).  One CTA per SM,
// persistent over units ordered heaviest-first (causal), 192 threads:
//   warp 0     TMA producer: Q tile once per unit, then K/V tiles through a
//              5-slot ring in the exact order the MMA consumes them
//              (K0, K1, V0, K2, V1, ..., V_last).
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S[j%2] = Q K_j^T           (SS form, 128x128x128)
//                O     += P_j V_j           (TS form: P_j read from TMEM)
//              issued as QK(0), {QK(j+1), PV(j)}...; S is double buffered so
//              QK(j+1) overlaps the softmax of block j.
//   warps 2-5  softmax / correction / epilogue, one query row per thread:
//              S row from TMEM -> scale, causal / length mask -> online max
//              with lazy rescale (O is only rescaled when the running max
//              grows by more than 2^8) -> P = 2^(s - m) as bf16 written back
//              over S in TMEM -> after the last block O / l -> bf16 -> global.
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384); P_j aliases S[j%2].
// K/V tiles for head h are read from kv head h / (QH/KH) (GQA sharing via L2).
// RoPE (optional) is applied by a pre-pass that rotates q and k once into the
// caller's workspace using a cos/sin table built in double precision.
// All waits are bounded (common.cuh); every TMA load targets one CTA.
#include <math.h>

#include "common.cuh"

KDA_DEFINE_ERROR_WORD(attn)

namespace kda {
namespace {

constexpr int kD = 128;           // head dim
constexpr int kBlk = 128;         // query rows per unit and keys per block
constexpr int kSlots = 5;         // K/V ring depth
constexpr uint32_t kTile = kBlk * kD * 2;  // 32 KB: one Q, K or V tile
constexpr int kThreads = 192;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256, kTmemCols = 512;

struct AttnParams {
  int B, S, QH, KH, n_rep;
  int nqb;          // query blocks per head
  int causal;
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  int64_t out_row_stride;   // elements between consecutive query rows
  int64_t out_head_stride;  // elements between heads (same position)
  int64_t out_batch_stride;
};

// smem: Q (32 KB) | ring (kSlots x 32 KB) | barriers
struct Smem {
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kRing = kTile;
  static constexpr uint32_t kBars = kRing + kSlots * kTile;
  // slot_full[5] slot_empty[5] q_full q_empty s_full[2] p_full pv o_free drain tmem_holder
  static constexpr uint32_t kNumBars = 2 * kSlots + 9;
  static constexpr size_t kBytes = 1024 + kBars + kNumBars * 8 + 16;
};

__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void unit_coords(int u, const AttnParams& p, int& b, int& h, int& qb) {
  const int heads = p.B * p.QH;
  const int level = u / heads;  // heaviest (last) query blocks first
  const int bh = u - level * heads;
  qb = p.causal ? (p.nqb - 1 - level) : level;
  b = bh / p.QH;
  h = bh - b * p.QH;
}

__device__ __forceinline__ int num_kv_blocks(const AttnParams& p, int qb) {
  const int all = (p.S + kBlk - 1) / kBlk;
  return p.causal ? (qb + 1 < all ? qb + 1 : all) : all;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnParams p, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::kBars);
  uint64_t* slot_full = bars;
  uint64_t* slot_empty = bars + kSlots;
  uint64_t* q_full = bars + 2 * kSlots;
  uint64_t* q_empty = q_full + 1;
  uint64_t* s_full = q_full + 2;  // [2]
  uint64_t* p_full = q_full + 4;
  uint64_t* pv_bar = q_full + 5;
  uint64_t* o_free = q_full + 6;
  uint64_t* drain = q_full + 7;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(q_full + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(pv_bar, 1);
    mbar_init(o_free, 128);
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
  const int units = p.B * p.QH * p.nqb;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int slot = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, last_par = 0;
    bool ok = true;
    int uc = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
      int b, h, qb;
      unit_coords(u, p, b, h, qb);
      const int kvh = h / p.n_rep;
      const int nb = num_kv_blocks(p, qb);
      const int row_q = qb * kBlk;
      if (lane == 0) ok = mbar_wait(q_empty, (uc & 1) ^ 1, err, kErrWaitEmpty);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, kTile);
        tma_load_4d(smem + Smem::kQ, &tmQ, q_full, 0, h, row_q, b);
        tma_load_4d(smem + Smem::kQ + kTile / 2, &tmQ, q_full, 64, h, row_q, b);
      }
      // K0, then {K(j+1), V(j)} -- the order the MMA issuer consumes them
      auto load = [&](bool isK, int j) -> bool {
        bool good = true;
        if (lane == 0) good = mbar_wait(&slot_empty[slot], phase ^ 1u, err, kErrWaitEmpty);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
        if (lane == 0) {
          uint8_t* dst = smem + Smem::kRing + slot * kTile;
          const CUtensorMap* m = isK ? &tmK : &tmV;
          mbar_arrive_expect_tx(&slot_full[slot], kTile);
          tma_load_4d(dst, m, &slot_full[slot], 0, kvh, j * kBlk, b);
          tma_load_4d(dst + kTile / 2, m, &slot_full[slot], 64, kvh, j * kBlk, b);
          issued |= 1u << slot;
          last_par = (last_par & ~(1u << slot)) | (phase << slot);
        }
        if (++slot == kSlots) {
          slot = 0;
          phase ^= 1u;
        }
        return true;
      };
      ok = load(true, 0);
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb) ok = load(true, j + 1);
        if (ok) ok = load(false, j);
      }
    }
    if (lane == 0) {
      for (int s = 0; s < kSlots; ++s)
        if (issued & (1u << s)) mbar_wait(&slot_full[s], (last_par >> s) & 1u, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t kIdQK = idesc_bf16_f32(kBlk, kBlk, 0, 0);
    constexpr uint32_t kIdPV = idesc_bf16_f32(kBlk, kD, 0, 1);
    int slot = 0;
    uint32_t phase = 0;
    uint32_t pcount = 0;  // blocks whose P was consumed (global)
    bool ok = true;
    bool any = false;
    int uc = 0;
    uint32_t sbuf = 0;  // S buffer of the next QK
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++uc) {
      int b, h, qb;
      unit_coords(u, p, b, h, qb);
      const int nb = num_kv_blocks(p, qb);
      if (lane == 0) ok = mbar_wait(q_full, uc & 1, err, kErrWaitFull);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t q_addr = smem_u32(smem + Smem::kQ);
      auto issue_qk = [&](int jj) -> bool {
        bool good = true;
        if (lane == 0) good = mbar_wait(&slot_full[slot], phase, err, kErrWaitFull);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t k_addr = smem_u32(smem + Smem::kRing + slot * kTile);
          const uint32_t d = tmem + (sbuf ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kTile / 2) + (kk & 3) * 32;
            umma_bf16(d, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024), kIdQK,
                      kk != 0 ? 1u : 0u);
          }
          umma_commit(&slot_empty[slot]);
          umma_commit(&s_full[sbuf]);
          if (jj == nb - 1) umma_commit(q_empty);
          any = true;
        }
        __syncwarp();
        sbuf ^= 1u;
        if (++slot == kSlots) {
          slot = 0;
          phase ^= 1u;
        }
        return true;
      };
      if (!issue_qk(0)) break;
      for (int j = 0; j < nb && ok; ++j) {
        if (j + 1 < nb && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        // PV(j): P_j in S[(j's buffer)], V_j in the next slot
        if (lane == 0) {
          ok = mbar_wait(p_full, pcount & 1u, err, kErrWaitAccum);
          if (ok && j == 0) ok = mbar_wait(o_free, (uc & 1) ^ 1, err, kErrWaitAccumFree);
          if (ok) ok = mbar_wait(&slot_full[slot], phase, err, kErrWaitFull);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          // block j used S buffer: the buffer toggled once per QK; QK(j) was
          // issued (j+1 < nb ? 2 : 1) QKs ago in this loop position.
          const uint32_t pbuf = (j + 1 < nb) ? (sbuf ^ 0u) : (sbuf ^ 1u);
          const uint32_t a_t = tmem + (pbuf ? kColS1 : kColS0);
          const uint32_t v_addr = smem_u32(smem + Smem::kRing + slot * kTile);
#pragma unroll
          for (int kk = 0; kk < kBlk / 16; ++kk) {
            umma_bf16_ts(tmem + kColO, a_t + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kTile / 2, 1024), kIdPV,
                         (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&slot_empty[slot]);
          umma_commit(pv_bar);
        }
        __syncwarp();
        ++pcount;
        if (++slot == kSlots) {
          slot = 0;
          phase ^= 1u;
        }
      }
    }
    // every issued MMA must finish before TMEM is released
    if (lane == 0 && any) {
      umma_commit(drain);
      mbar_wait(drain, 0, err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------- softmax / epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t sph[2] = {0u, 0u};
    uint32_t pvcount = 0;
    uint32_t sbuf = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int b, h, qb;
      unit_coords(u, p, b, h, qb);
      const int nb = num_kv_blocks(p, qb);
      const int qpos = qb * kBlk + r;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nb; ++j) {
        ok = mbar_wait(&s_full[sbuf], sph[sbuf], err, kErrWaitAccum);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        sph[sbuf] ^= 1u;
        tc_fence_after();
        const uint32_t scol = tmem + lane_base + (sbuf ? kColS1 : kColS0);
        float s[kBlk];
        {
          uint32_t rr[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tmem_ld_32x32b_x32(scol + c * 32, rr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(rr[i]) * p.scale_log2;
          }
        }
        const int k0 = j * kBlk;
        const bool diag = p.causal && (j == qb);
        const bool tail = (k0 + kBlk > p.S);
        if (diag || tail) {
#pragma unroll
          for (int i = 0; i < kBlk; ++i) {
            const bool masked = (diag && i > r) || (k0 + i >= p.S);
            if (masked) s[i] = -INFINITY;
          }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < kBlk; ++i) mx = fmaxf(mx, s[i]);
        float m_new = fmaxf(m_run, mx);
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
        float sum = 0.f;
        uint32_t pk[kBlk / 2];
#pragma unroll
        for (int i = 0; i < kBlk / 2; ++i) {
          const float e0 = exp2_approx(s[2 * i] - mb);
          const float e1 = exp2_approx(s[2 * i + 1] - mb);
          sum += e0 + e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        l_run = l_run * factor + sum;
        // O must hold PV(j-1) before it is rescaled and before P_j replaces S
        if (j > 0) {
          ok = mbar_wait(pv_bar, pvcount & 1u, err, kErrWaitAccum);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          ++pvcount;
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
            const uint32_t ocol = tmem + lane_base + kColO;
            uint32_t rr[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              tmem_ld_32x32b_x32(ocol + c * 32, rr);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * factor);
              tmem_st_32x32b_x32(ocol + c * 32, rr);
            }
          }
        }
        {
          uint32_t lo[32], hi[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            lo[i] = pk[i];
            hi[i] = pk[32 + i];
          }
          tmem_st_32x32b_x32(scol, lo);
          tmem_st_32x32b_x32(scol + 32, hi);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(p_full);
        sbuf ^= 1u;
      }
      if (!ok) break;
      // epilogue: wait for PV(nb-1), O / l -> bf16 -> global
      ok = mbar_wait(pv_bar, pvcount & 1u, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      ++pvcount;
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(b) * p.out_batch_stride +
                            static_cast<int64_t>(h) * p.out_head_stride + static_cast<int64_t>(qpos) * p.out_row_stride;
      const uint32_t ocol = tmem + lane_base + kColO;
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
      tc_fence_before();
      mbar_arrive(o_free);
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

// x [B,S,H,128] bf16 -> out (same layout), half-split rotation; one thread
// per (row, 8 consecutive frequencies).
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
    const float x0 = __bfloat162float(a16[i]), x1 = __bfloat162float(c16[i]);
    o0[i] = x0 * cs.x - x1 * cs.y;
    o1[i] = x0 * cs.y + x1 * cs.x;
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

inline size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

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

}  // namespace
}  // namespace kda

using namespace kda;

extern "C" size_t kda_gqa_full_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                              float rope_theta) {
  if (B <= 0 || S <= 0 || QH <= 0 || KH <= 0 || D != kD || !(rope_theta > 0.f)) return 0;
  return al256(static_cast<size_t>(B) * S * QH * kD * 2) + al256(static_cast<size_t>(B) * S * KH * kD * 2) +
         al256(static_cast<size_t>(S) * (kD / 2) * 8);
}

extern "C" kda_status kda_gqa_full_bf16(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S,
                                        int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  KDA_CHECK_ARG(q && k && v && out, "gqa_full: null pointer");
  KDA_CHECK_ARG(B > 0 && S > 0 && QH > 0 && KH > 0 && QH % KH == 0 && B * S < (1ll << 31) / QH,
                "gqa_full: bad sizes B=%lld S=%lld QH=%lld KH=%lld", (long long)B, (long long)S, (long long)QH,
                (long long)KH);
  KDA_CHECK_SUPPORTED(D == kD, "gqa_full: head_dim must be 128, got %lld", (long long)D);
  KDA_CHECK_SUPPORTED(QH <= 65535 && KH <= 65535, "gqa_full: too many heads");
  const bool al = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                    reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  KDA_CHECK_SUPPORTED(al, "gqa_full: pointers must be 16-byte aligned");
  const size_t need = kda_gqa_full_workspace_size(B, S, QH, KH, D, rope_theta);
  KDA_CHECK_ARG(need == 0 || (workspace && workspace_bytes >= need),
                "gqa_full: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const void* qs = q;
  const void* ks = k;
  if (need) {
    uint8_t* w = static_cast<uint8_t*>(workspace);
    KDA_CHECK_SUPPORTED((reinterpret_cast<uintptr_t>(w) & 15u) == 0, "gqa_full: workspace must be 16-byte aligned");
    auto* qr = reinterpret_cast<__nv_bfloat16*>(w);
    auto* kr = reinterpret_cast<__nv_bfloat16*>(w + al256(static_cast<size_t>(B) * S * QH * kD * 2));
    auto* tab = reinterpret_cast<float2*>(w + al256(static_cast<size_t>(B) * S * QH * kD * 2) +
                                          al256(static_cast<size_t>(B) * S * KH * kD * 2));
    const int nt = static_cast<int>(S * (kD / 2));
    rope_table_kernel<<<(nt + 255) / 256, 256, 0, st>>>(tab, static_cast<int>(S), log2(static_cast<double>(rope_theta)));
    const int64_t qrows = B * S * QH, krows = B * S * KH;
    rope_rotate_kernel<<<static_cast<unsigned>((qrows * 8 + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(q), qr, tab, qrows, static_cast<int>(S), static_cast<int>(QH));
    rope_rotate_kernel<<<static_cast<unsigned>((krows * 8 + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(k), kr, tab, krows, static_cast<int>(S), static_cast<int>(KH));
    if (launch_status("gqa_full rope") != KDA_OK) return KDA_CUDA_ERROR;
    qs = qr;
    ks = kr;
  }
  CUtensorMap tq, tk, tv;
  kda_status s;
  if ((s = tmap_heads(&tq, qs, B, S, QH)) != KDA_OK) return s;
  if ((s = tmap_heads(&tk, ks, B, S, KH)) != KDA_OK) return s;
  if ((s = tmap_heads(&tv, v, B, S, KH)) != KDA_OK) return s;
  AttnParams p{};
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.QH = static_cast<int>(QH);
  p.KH = static_cast<int>(KH);
  p.n_rep = static_cast<int>(QH / KH);
  p.nqb = static_cast<int>((S + kBlk - 1) / kBlk);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(kD)));
  p.out = out;
  if (out_bshd) {
    p.out_row_stride = QH * kD;
    p.out_head_stride = kD;
    p.out_batch_stride = S * QH * kD;
  } else {
    p.out_row_stride = kD;
    p.out_head_stride = S * kD;
    p.out_batch_stride = QH * S * kD;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Smem::kBytes)) != cudaSuccess)
      return launch_status("gqa_full: cudaFuncSetAttribute");
    attr_set[dev] = true;
  }
  const long long units = static_cast<long long>(B) * QH * p.nqb;
  const int grid = static_cast<int>(units < num_sms() ? units : num_sms());
  attn_kernel<<<grid, kThreads, Smem::kBytes, st>>>(tq, tk, tv, p, kda_err_ptr_attn());
  return launch_status("attn_kernel");
}
