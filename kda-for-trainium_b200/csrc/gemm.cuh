// The tcgen05 GEMM engine shared by every contraction in the library.
//
//   TMA (128-byte swizzle) -> STAGES-deep shared-memory ring -> tcgen05.mma
//   (M=128, N=BN, K=16, bf16 x bf16 -> fp32) issued by one thread ->
//   double-buffered TMEM accumulator (2 x BN columns) -> epilogue warps
//   (tcgen05.ld -> registers -> fused epilogue -> global).
//
// One CTA per SM, persistent over output tiles (grouped raster for L2 reuse).
// Warp roles: warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31, i.e. tile
// rows).  All waits are bounded (common.cuh).  No TMA multicast anywhere.
//
// Operand layouts (per k-block of 64):
//   A K-major  : one box {64 k, 128 m}        -> rows of 128 B, SBO 1024
//   A MN-major : two boxes {64 m, 64 k}       -> MN atoms at LBO 8192, SBO 1024
//   B K-major  : one box {64 k, BN n}         -> rows of 128 B, SBO 1024
//   B MN-major : BN/64 boxes {64 n, 64 k}     -> MN atoms at LBO 8192, SBO 1024
// B modes: single B; DUAL (B columns [0,BN/2) from map B, [BN/2,BN) from
// map B2 at the same output columns -- SwiGLU's gate|up pair); KEXT (k-blocks
// past p.k_blocks read A2/B2 -- LoRA's K-extension into one accumulator).
#pragma once

#include "common.cuh"

namespace kda {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr uint32_t kABytes = BM * BK * 2;

enum BMode { B_SINGLE = 0, B_DUAL = 1, B_KEXT = 2 };
enum Epi { EPI_BF16 = 0, EPI_SWIGLU = 1, EPI_RESID_F32 = 2, EPI_SOFTMAX = 3 };

struct Params {
  int M, N, K;        // output rows / output columns of one tile grid / contraction
  int k_blocks;       // ceil(K / BK) for maps A/B
  int k_blocks2;      // KEXT: extra k-blocks read from maps A2/B2
  int batch;          // BATCHED: number of independent problems (3-D maps)
  int m_tiles, n_tiles;
  int group_m;        // raster group height (in m-tiles)
  void* out;          // bf16 or fp32 output
  int64_t ldo;        // output row stride (elements)
  int64_t out_bstride;  // BATCHED output batch stride (elements)
  const __nv_bfloat16* z;  // EPI_RESID_F32: residual (bf16), row stride ldz
  int64_t ldz;
  float* rowsq;       // EPI_RESID_F32: per-row sum of squares (atomic)
};

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t kBBytes = BN * BK * 2;
  static constexpr uint32_t kStage = kABytes + kBBytes;
  static constexpr uint32_t kBarOff = STAGES * kStage;
  static constexpr uint32_t kNumBars = 2 * STAGES + 5;
  static constexpr size_t kBytes = 1024 /*align slack*/ + kBarOff + kNumBars * 8 + 16;
};

template <int BN>
struct TmemCols {
  static constexpr uint32_t kCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                    : (2 * BN <= 256) ? 256 : 512;
};

// Work is enumerated as (unit, sub): a CTA owns whole units (persistent
// stride over units) and walks their subs in order.  Plain GEMMs: one tile
// per unit.  Row softmax: a unit is one 128-row block of one batch entry and
// its subs sweep the n-tiles twice (statistics pass, then output pass).
template <int EPI>
__device__ __forceinline__ void work_coords(int unit, int sub, const Params& p, int& b, int& m_tile, int& n_tile);

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& b, int& m_tile, int& n_tile) {
  const int per_batch = p.m_tiles * p.n_tiles;
  b = tile / per_batch;
  const int t = tile - b * per_batch;
  const int group = p.group_m * p.n_tiles;
  const int gidx = t / group;
  const int first_m = gidx * p.group_m;
  const int rem = p.m_tiles - first_m;
  const int gm = rem < p.group_m ? rem : p.group_m;
  const int in = t - gidx * group;
  m_tile = first_m + in % gm;
  n_tile = in / gm;
}

template <int EPI>
__device__ __forceinline__ void work_coords(int unit, int sub, const Params& p, int& b, int& m_tile, int& n_tile) {
  if (EPI == EPI_SOFTMAX) {
    b = unit / p.m_tiles;
    m_tile = unit - b * p.m_tiles;
    n_tile = sub < p.n_tiles ? sub : sub - p.n_tiles;
  } else {
    tile_coords(unit, p, b, m_tile, n_tile);
  }
}

template <int EPI>
__host__ __device__ __forceinline__ int num_units(const Params& p) {
  return EPI == EPI_SOFTMAX ? p.batch * p.m_tiles : p.batch * p.m_tiles * p.n_tiles;
}
template <int EPI>
__host__ __device__ __forceinline__ int subs_per_unit(const Params& p) {
  return EPI == EPI_SOFTMAX ? 2 * p.n_tiles : 1;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool BATCHED, int BMODE, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                const Params p, unsigned* err) {
  using S = Smem<BN, STAGES>;
  constexpr uint32_t kCols = TmemCols<BN>::kCols;
  constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be a multiple of 64, at most 256");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiThreads);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (BMODE != B_SINGLE) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int units = num_units<EPI>(p);
  const int subs = subs_per_unit<EPI>(p);
  const int k_total = p.k_blocks + (BMODE == B_KEXT ? p.k_blocks2 : 0);

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, last_par = 0;  // per-stage bit masks for the drain
    bool ok = true;
    for (int w = 0, unit = blockIdx.x, sub = 0; unit < units && ok; ++w) {
      int b, mt, nt;
      work_coords<EPI>(unit, sub, p, b, mt, nt);
      if (++sub == subs) {
        sub = 0;
        unit += gridDim.x;
      }
      const int m0 = mt * BM;
      const int n0 = nt * (BMODE == B_DUAL ? BN / 2 : BN);
      for (int kb = 0; kb < k_total; ++kb) {
        if (lane == 0) ok = mbar_wait(&empty[stage], phase ^ 1u, err, kErrWaitEmpty);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) {
          uint8_t* sa = smem + stage * S::kStage;
          uint8_t* sb = sa + kABytes;
          uint64_t* bar = &full[stage];
          mbar_arrive_expect_tx(bar, S::kStage);
          const bool ext = (BMODE == B_KEXT) && kb >= p.k_blocks;
          const CUtensorMap* ma = ext ? &tmA2 : &tmA;
          const CUtensorMap* mb = ext ? &tmB2 : &tmB;
          const int k0 = (ext ? kb - p.k_blocks : kb) * BK;
          // A tile
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) {
              if (BATCHED)
                tma_load_3d(sa + j * 8192, ma, bar, m0 + j * 64, k0, b);
              else
                tma_load_2d(sa + j * 8192, ma, bar, m0 + j * 64, k0);
            }
          } else {
            if (BATCHED)
              tma_load_3d(sa, ma, bar, k0, m0, b);
            else
              tma_load_2d(sa, ma, bar, k0, m0);
          }
          // B tile
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              const CUtensorMap* mj = mb;
              int nj = n0 + j * 64;
              if (BMODE == B_DUAL && j >= BN / 128) {
                mj = &tmB2;
                nj = n0 + (j - BN / 128) * 64;
              }
              if (BATCHED)
                tma_load_3d(sb + j * 8192, mj, bar, nj, k0, b);
              else
                tma_load_2d(sb + j * 8192, mj, bar, nj, k0);
            }
          } else {
            if (BMODE == B_DUAL) {
              tma_load_2d(sb, mb, bar, k0, n0);
              tma_load_2d(sb + (BN / 2) * 128, &tmB2, bar, k0, n0);
            } else if (BATCHED) {
              tma_load_3d(sb, mb, bar, k0, n0, b);
            } else {
              tma_load_2d(sb, mb, bar, k0, n0);
            }
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Every issued copy must land before the CTA may exit.
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s)
        if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    bool any = false;
    const long long my_work = units > static_cast<int>(blockIdx.x)
                                  ? static_cast<long long>((units - 1 - blockIdx.x) / gridDim.x + 1) * subs
                                  : 0;
    for (long long w = 0; w < my_work && ok; ++w) {
      if (lane == 0) ok = mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kErrWaitAccumFree);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int kb = 0; kb < k_total; ++kb) {
        if (lane == 0) ok = mbar_wait(&full[stage], phase, err, kErrWaitFull);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * S::kStage);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            umma_bf16(d, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          any = true;
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // All issued MMAs must finish before TMEM is released.
    if (lane == 0 && any) {
      umma_commit(drain);
      mbar_wait(drain, 0, err, kErrWaitDrain);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    float row_max = -INFINITY, row_sum = 0.f;  // EPI_SOFTMAX running statistics
    for (int unit = blockIdx.x, sub = 0; unit < units;) {
      int b, mt, nt;
      work_coords<EPI>(unit, sub, p, b, mt, nt);
      const int cur_sub = sub;
      if (++sub == subs) {
        sub = 0;
        unit += gridDim.x;
      }
      ok = mbar_wait(&tfull[acc], acc_phase, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int gm = mt * BM + row;
      const bool row_ok = gm < p.M;
      if (EPI == EPI_BF16) {
        const int n0 = nt * BN;
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) +
                              (BATCHED ? static_cast<int64_t>(b) * p.out_bstride : 0) +
                              static_cast<int64_t>(gm) * p.ldo;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (row_ok && gn < p.N) {
            if (gn + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(orow + gn);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 v;
                v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
                v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
                v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
                v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
                dst[q] = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (gn + j < p.N) orow[gn + j] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          }
        }
      } else if (EPI == EPI_SWIGLU) {
        // gate in accumulator columns [0, BN/2), up in [BN/2, BN)
        const int n0 = nt * (BN / 2);
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(gm) * p.ldo;
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tb + c * 32, rg);
          tmem_ld_32x32b_x32(tb + BN / 2 + c * 32, ru);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (row_ok && gn < p.N) {
            float h[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) h[j] = silu_f32(__uint_as_float(rg[j])) * __uint_as_float(ru[j]);
            if (gn + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(orow + gn);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 v;
                v.x = pack_bf16x2(h[8 * q + 0], h[8 * q + 1]);
                v.y = pack_bf16x2(h[8 * q + 2], h[8 * q + 3]);
                v.z = pack_bf16x2(h[8 * q + 4], h[8 * q + 5]);
                v.w = pack_bf16x2(h[8 * q + 6], h[8 * q + 7]);
                dst[q] = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (gn + j < p.N) orow[gn + j] = __float2bfloat16_rn(h[j]);
            }
          }
        }
      } else if (EPI == EPI_SOFTMAX) {
        // pass 0 (cur_sub < n_tiles): online max / sum of exp over the row;
        // pass 1: out = exp(x - max) / sum, bf16.
        constexpr float kL2e = 1.4426950408889634f;
        const int n0 = nt * BN;
        if (cur_sub == 0) {
          row_max = -INFINITY;
          row_sum = 0.f;
        }
        const bool stats = cur_sub < p.n_tiles;
        const float inv_sum = stats ? 0.f : 1.0f / row_sum;
        const float mb = row_max * kL2e;
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(b) * p.out_bstride +
                              static_cast<int64_t>(gm) * p.ldo;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (gn >= p.N) continue;
          if (stats) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (gn + j < p.N) mx = fmaxf(mx, __uint_as_float(r[j]));
            const float m_new = fmaxf(row_max, mx);
            const float mnb = m_new * kL2e;
            float s = row_sum * exp2_approx(fmaf(row_max, kL2e, -mnb));
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (gn + j < p.N) s += exp2_approx(fmaf(__uint_as_float(r[j]), kL2e, -mnb));
            row_sum = s;
            row_max = m_new;
          } else if (row_ok) {
            float e[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) e[j] = exp2_approx(fmaf(__uint_as_float(r[j]), kL2e, -mb)) * inv_sum;
            if (gn + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(orow + gn);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 v;
                v.x = pack_bf16x2(e[8 * q + 0], e[8 * q + 1]);
                v.y = pack_bf16x2(e[8 * q + 2], e[8 * q + 3]);
                v.z = pack_bf16x2(e[8 * q + 4], e[8 * q + 5]);
                v.w = pack_bf16x2(e[8 * q + 6], e[8 * q + 7]);
                dst[q] = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (gn + j < p.N) orow[gn + j] = __float2bfloat16_rn(e[j]);
            }
          }
        }
      } else {  // EPI_RESID_F32: y = acc + z (fp32 out), row sum of squares
        const int n0 = nt * BN;
        float* orow = reinterpret_cast<float*>(p.out) + static_cast<int64_t>(gm) * p.ldo;
        const __nv_bfloat16* zrow = p.z + static_cast<int64_t>(gm) * p.ldz;
        float ss = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (row_ok && gn < p.N) {
            if (gn + 32 <= p.N) {
              const uint4* zs = reinterpret_cast<const uint4*>(zrow + gn);
              float4* dst = reinterpret_cast<float4*>(orow + gn);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 zv = zs[q];
                const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
                float y[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(&zw[e]);
                  y[2 * e] = __uint_as_float(r[8 * q + 2 * e]) + __bfloat162float(z2.x);
                  y[2 * e + 1] = __uint_as_float(r[8 * q + 2 * e + 1]) + __bfloat162float(z2.y);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = fmaf(y[e], y[e], ss);
                dst[2 * q] = make_float4(y[0], y[1], y[2], y[3]);
                dst[2 * q + 1] = make_float4(y[4], y[5], y[6], y[7]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (gn + j < p.N) {
                  const float y = __uint_as_float(r[j]) + __bfloat162float(zrow[gn + j]);
                  ss = fmaf(y, y, ss);
                  orow[gn + j] = y;
                }
              }
            }
          }
        }
        if (row_ok) atomicAdd(&p.rowsq[gm], ss);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kCols);
}

// Host-side launch of one instantiation.
template <int BN, bool A_MN, bool B_MN, int EPI, bool BATCHED, int BMODE, int STAGES>
kda_status launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2, const CUtensorMap& b2,
                  const Params& p, unsigned* err, cudaStream_t st) {
  auto kern = gemm_kernel<BN, A_MN, B_MN, EPI, BATCHED, BMODE, STAGES>;
  constexpr size_t smem = Smem<BN, STAGES>::kBytes;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      set_error("gemm: cudaFuncSetAttribute(%zu B smem): %s", smem, cudaGetErrorString(e));
      return KDA_CUDA_ERROR;
    }
    attr_set[dev] = true;
  }
  const long long tiles = num_units<EPI>(p);
  if (tiles <= 0) return KDA_OK;
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  kern<<<grid, kThreads, smem, st>>>(a, b, a2, b2, p, err);
  return launch_status("gemm_kernel");
}

}  // namespace gemm
}  // namespace kda
