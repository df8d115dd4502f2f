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
// rows; 2..9 for the softmax epilogue), last warp = scheduler: it performs
// the mbarrier waits of the MMA issuer (stage loaded, accumulator free) and
// releases it k-block by k-block through a named barrier, so the issuing
// thread never touches shared memory between MMAs (such an access stalls
// behind the queued MMAs).  All mbarrier waits are bounded (common.cuh).
// Every TMA load targets one CTA.
//
// Operand layouts (per k-block of 64):
//   A K-major  : one box {64 k, 128 m}        -> rows of 128 B, SBO 1024
//   A MN-major : two boxes {64 m, 64 k}       -> MN atoms at LBO 8192, SBO 1024
//   B K-major  : one box {64 k, BN n}         -> rows of 128 B, SBO 1024
//   B MN-major : BN/64 boxes {64 n, 64 k}     -> MN atoms at LBO 8192, SBO 1024
// B modes: single B; DUAL (B columns [0,BN/2) from map B, [BN/2,BN) from
// map B2 at the same output columns -- SwiGLU's gate|up pair); KEXT (k-blocks
// past p.k_blocks read A2/B2 -- LoRA's K-extension into one accumulator);
// SPLIT3 (three passes over K into one accumulator: A.B2, A2.B, then A.B --
// the bf16x3 product of fp32 operands split as hi = A/B, lo = A2/B2; the two
// small correction passes first, so they are not added to an accumulator that
// already holds the full-size hi.hi sum).
#pragma once

#include "common.cuh"

namespace kda {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;     // TMA warp + MMA warp + 4 epilogue warps
constexpr int kEpiThreads = 128;
// The row-softmax epilogue runs 16 warps: four per TMEM lane quadrant, each
// taking a quarter of a tile's columns (four warps per SM partition keep the
// MUFU pipe busy through each other's TMEM loads and stores).
__host__ __device__ constexpr int epi_warps(int epi, bool batched = false);
__host__ __device__ constexpr int sched_warp(int epi, bool batched = false) { return 2 + epi_warps(epi, batched); }
__host__ __device__ constexpr int threads_for(int epi, bool batched = false) {
  return 32 * (sched_warp(epi, batched) + 1);
}
constexpr int kGoBarrier = 2;  // named barrier: scheduler warp + MMA warp (1 is the softmax epilogue's)
constexpr uint32_t kABytes = BM * BK * 2;

// B_SPLIT3F (CTA pairs): the bf16x3 product with all four split operands of a
// k-block in one stage (A hi, A lo, B hi, B lo: each tile read once) and two
// TMEM accumulators -- hi.lo + lo.hi in columns [0, BN), hi.hi in [BN, 2 BN),
// added in the epilogue -- so the corrections never meet the full-size sum
// inside the tensor core; the accumulator pair fills TMEM, so it is single
// buffered.
enum BMode { B_SINGLE = 0, B_DUAL = 1, B_KEXT = 2, B_SPLIT3 = 3, B_SPLIT3F = 4 };
// EPI_F32: split-K partial sums, fp32, to out[k part][M][ldo] (plain stores)
// EPI_F32OUT: fp32 output through TMA stores of 32-row x 16-column boxes
enum Epi : int { EPI_BF16 = 0, EPI_SWIGLU = 1, EPI_SOFTMAX = 3, EPI_RESID_BF16 = 4, EPI_F32 = 5, EPI_F32OUT = 6 };
// Batched bf16 GEMMs (bmm: one k-block per tile, so the epilogue is the
// whole cost of a tile) run 8 epilogue warps, two per lane quadrant, each
// storing half of the tile's columns.  The row softmax (exponential-bound)
// runs 16.
__host__ __device__ constexpr int epi_warps(int epi, bool batched) {
  return epi == EPI_SOFTMAX ? 16 : ((batched && epi == EPI_BF16) ? 8 : 4);
}

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
  const __nv_bfloat16* z;  // EPI_RESID_BF16: residual (bf16), row stride ldz
  int64_t ldz;
  float* rowsq;       // EPI_RESID_BF16: per-row sum of squares of y (atomic)
  int k_split;        // EPI_F32: K parts of k_blocks k-blocks each (units = tiles x parts)
  // TAIL (bf16 pair GEMM, plain or residual): tiles [tail_first, tiles) -- the last,
  // partial wave -- are cut into tail_parts K ranges of tail_kb k-blocks, one
  // unit each; every part writes its fp32 partial tile to tail_part and counts
  // itself in tail_cnt (zeroed before the launch), and the part that arrives
  // last sums all parts in part order and stores the tile.
  int tail_first, tail_parts, tail_kb;
  float* tail_part;    // [tail tile][part][CTA of the pair][BN columns][128 rows]
  unsigned* tail_cnt;  // [tail tile][CTA of the pair]
};

enum Epi : int;
template <int BN, int STAGES, bool PAIR = false, int NEPI = 4, int NSTAT = 0, int OPX = 1>
struct Smem {
  // a CTA of a pair holds its 128 rows of A and half of the BN columns of B
  // (OPX = 2: hi and lo halves of both, B_SPLIT3F)
  static constexpr uint32_t kBBytes = (PAIR ? BN / 2 : BN) * BK * 2;
  static constexpr uint32_t kStage = OPX * (kABytes + kBBytes);
  static constexpr uint32_t kBarOff = STAGES * kStage;
  static constexpr uint32_t kNumBars = 2 * STAGES + 6;
  // epilogue staging: NEPI warps x 2 buffers x (32 rows x 64 B), 1024-aligned,
  // then the row-statistics exchange area (NSTAT parts x 128 rows x {max, sum})
  static constexpr uint32_t kStageOff = (kBarOff + kNumBars * 8 + 16 + 1023) & ~1023u;
  static constexpr uint32_t kStageBytes = NEPI * 2 * 2048;
  static constexpr uint32_t kStatOff = kStageOff + kStageBytes;
  static constexpr size_t kBytes = 1024 /*align slack*/ + kStatOff + NSTAT * 128 * 8;
  static_assert(kBytes > 116 * 1024, "one TMEM-allocating CTA per SM requires > 116 KB of shared memory");
  static_assert(kBytes <= 227 * 1024, "shared memory budget");
};

// Write one warp's 32 x 32 bf16 chunk (16 packed words per lane = one row)
// into a 64B-swizzled staging buffer and hand it to a TMA bulk store.  Two
// buffers per warp alternate; a buffer is rewritten only after the store that
// read it two chunks ago has finished reading.
template <bool BATCHED>
__device__ __forceinline__ void stage_store(const uint32_t (&w)[16], uint8_t* warp_stage, int& sbuf,
                                            const CUtensorMap* tm, int x, int y, int z, int lane) {
  uint8_t* buf = warp_stage + sbuf * 2048;
  if (lane == 0) bulk_wait_read_le1();
  __syncwarp();
  const int sw = (lane >> 1) & 3;  // SWIZZLE_64B: 16-byte chunk ^= (row / 2) % 4
  uint4* row = reinterpret_cast<uint4*>(buf + lane * 64);
  row[0 ^ sw] = make_uint4(w[0], w[1], w[2], w[3]);
  row[1 ^ sw] = make_uint4(w[4], w[5], w[6], w[7]);
  row[2 ^ sw] = make_uint4(w[8], w[9], w[10], w[11]);
  row[3 ^ sw] = make_uint4(w[12], w[13], w[14], w[15]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (BATCHED)
      tma_store_3d(tm, buf, x, y, z);
    else
      tma_store_2d(tm, buf, x, y);
    bulk_commit();
  }
  sbuf ^= 1;
}

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
__device__ __forceinline__ void work_coords(int unit, int sub, const Params& p, int& b, int& m_tile, int& n_tile,
                                            int n_base, int n_count);

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

// Row softmax: this CTA sweeps n-tiles [n_base, n_base + n_count) (all of
// them, or its half of a row block split over a CTA pair).
template <int EPI>
__device__ __forceinline__ void work_coords(int unit, int sub, const Params& p, int& b, int& m_tile, int& n_tile,
                                            int n_base, int n_count) {
  if (EPI == EPI_SOFTMAX) {
    b = unit / p.m_tiles;
    m_tile = unit - b * p.m_tiles;
    n_tile = n_base + (sub < n_count ? sub : sub - n_count);
  } else if (EPI == EPI_F32) {
    tile_coords(unit / p.k_split, p, b, m_tile, n_tile);  // the k parts of a tile are adjacent units
  } else if (p.tail_parts > 1 && unit >= p.tail_first) {
    tile_coords(p.tail_first + (unit - p.tail_first) / p.tail_parts, p, b, m_tile, n_tile);
  } else {
    tile_coords(unit, p, b, m_tile, n_tile);
  }
}

template <int EPI>
__host__ __device__ __forceinline__ int num_units(const Params& p) {
  if (EPI == EPI_SOFTMAX) return p.batch * p.m_tiles;
  const int tiles = p.batch * p.m_tiles * p.n_tiles;
  if (EPI == EPI_F32) return tiles * p.k_split;
  return p.tail_parts > 1 ? p.tail_first + (tiles - p.tail_first) * p.tail_parts : tiles;
}

// The k-blocks [kb0, kb0 + nkb) of a unit: all k_total of them, or one K part
// of a tail tile.
__host__ __device__ __forceinline__ void unit_kblocks(int unit, const Params& p, int k_total, int& kb0, int& nkb) {
  kb0 = 0;
  nkb = k_total;
  if (p.tail_parts > 1 && unit >= p.tail_first) {
    const int part = (unit - p.tail_first) % p.tail_parts;
    kb0 = part * p.tail_kb;
    const int end = kb0 + p.tail_kb < p.k_blocks ? kb0 + p.tail_kb : p.k_blocks;
    nkb = end - kb0;
  }
}
template <int EPI>
__host__ __device__ __forceinline__ int subs_per_unit(const Params& p) {
  return EPI == EPI_SOFTMAX ? 2 * p.n_tiles : 1;
}

// PAIR: two CTAs of a cluster share one 256 x BN tile.  Each loads its own
// 128 rows of A and half of B's columns; the leader (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256 whose results land in each CTA's own
// TMEM (its 128 rows); MMA completion is signalled to both CTAs' barriers.
// CSPLIT (row softmax only): the two CTAs of a cluster split each row block's
// n-tiles in half and exchange their row statistics through distributed
// shared memory after the statistics pass (twice as many, half as long units
// per CTA pair: the grid tail shrinks).
template <int BN, bool A_MN, bool B_MN, int EPI, bool BATCHED, int BMODE, int STAGES, bool PAIR = false,
          bool CSPLIT = false, bool TAIL = false>
__global__ void __launch_bounds__(threads_for(EPI, BATCHED), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                const __grid_constant__ CUtensorMap tmOut, const Params p, unsigned* err) {
  // row-softmax statistics area: one 128-row block per column part, plus (CSPLIT)
  // two exchange buffers and one block holding their two mbarriers
  using S = Smem<BN, STAGES, PAIR, epi_warps(EPI, BATCHED),
                 EPI == EPI_SOFTMAX ? epi_warps(EPI) / 4 + (CSPLIT ? 3 : 0) : 0, BMODE == B_SPLIT3F ? 2 : 1>;
  constexpr bool kOneAcc = BMODE == B_SPLIT3F;  // one accumulator pair, single buffered
  static_assert(BMODE != B_SPLIT3F || (PAIR && !BATCHED && EPI == EPI_F32OUT && BN == 256),
                "the fused split product is for fp32-output pair GEMMs");
  constexpr bool kCluster = PAIR || CSPLIT;
  static_assert(!CSPLIT || (EPI == EPI_SOFTMAX && !PAIR), "column split is for the single-CTA row softmax");
  constexpr int kEpi = 32 * epi_warps(EPI, BATCHED);  // epilogue threads
  constexpr uint32_t kCols = TmemCols<BN>::kCols;
  constexpr uint32_t kIdesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
  constexpr int kBHalf = PAIR ? BN / 2 : BN;  // B columns held by this CTA
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be a multiple of 64, at most 256");
  static_assert(!PAIR || B_MN || BMODE == B_SINGLE || BMODE == B_KEXT,
                "CTA-pair mode loads B K-major only for single and K-extended B");
  static_assert(!PAIR || EPI != EPI_SOFTMAX, "row softmax runs on single CTAs");
  static_assert(EPI != EPI_F32 || (!PAIR && !BATCHED && BMODE == B_SINGLE),
                "split-K partials come from the single-CTA plain GEMM");
  static_assert(EPI != EPI_F32OUT || !BATCHED, "fp32 output: 2-D GEMMs");
  static_assert(!TAIL || ((EPI == EPI_BF16 || EPI == EPI_RESID_BF16) && PAIR && !BATCHED && BMODE == B_SINGLE),
                "the tail split is for the plain bf16 pair GEMM");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tail_bar = drain + 1;  // TAIL: the other parts' partials arriving in the idle operand ring
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 2 * kEpi : kEpi);
    }
    if (CSPLIT) {
      // exchange barriers: 128 remote arrivals (the peer's part-0 threads)
      uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + S::kStatOff + (epi_warps(EPI) / 4 + 2) * 128 * 8);
      mbar_init(&xbar[0], 128);
      mbar_init(&xbar[1], 128);
    }
    mbar_init(drain, 1);
    mbar_init(tail_bar, 1);
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
    if (PAIR) {
      tmem_alloc_pair(tmem_holder, kCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, kCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (kCluster)
    cluster_sync_all();  // peer barriers are initialised before any remote arrival
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int units = num_units<EPI>(p);
  const uint32_t rank = kCluster ? cluster_ctarank() : 0u;
  const int first_unit = kCluster ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int unit_stride = kCluster ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int tile_rows = PAIR ? 2 * BM : BM;
  const uint32_t row_rank = PAIR ? rank : 0u;  // CTA pairs split rows, CSPLIT pairs split columns
  const int n_count = CSPLIT ? (p.n_tiles + 1) / 2 : p.n_tiles;
  const int n_base = CSPLIT ? static_cast<int>(rank) * n_count : 0;
  const int subs = EPI == EPI_SOFTMAX ? 2 * n_count : subs_per_unit<EPI>(p);
  const int k_total = p.k_blocks + (BMODE == B_KEXT ? p.k_blocks2 : 0) + (BMODE == B_SPLIT3 ? 2 * p.k_blocks : 0);

  pdl_trigger();  // a kernel queued behind this one may start its prologue
  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    // The producer is the only reader of the inputs (everything else is fed
    // through its barriers), so it alone waits for a preceding kernel that
    // was allowed to overlap this one (programmatic dependent launch).
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0, last_par = 0;  // per-stage bit masks for the drain
    bool ok = true;
    pdl_wait();
    for (int unit = first_unit, sub = 0; unit < units && ok;) {
      int b, mt, nt;
      work_coords<EPI>(unit, sub, p, b, mt, nt, n_base, n_count);
      // EPI_F32: this unit's k part starts k_blocks k-blocks per part in
      const int kpart0 = EPI == EPI_F32 ? (unit % p.k_split) * p.k_blocks : 0;
      int ukb0 = 0, unkb = k_total;
      if (TAIL) unit_kblocks(unit, p, k_total, ukb0, unkb);
      if (++sub == subs) {
        sub = 0;
        unit += unit_stride;
      }
      const int m0 = mt * tile_rows + static_cast<int>(row_rank) * BM;
      // B columns this CTA loads: DUAL pairs split gate (rank 0) / up (rank 1)
      const int n0 = nt * (BMODE == B_DUAL ? BN / 2 : BN) + ((PAIR && BMODE != B_DUAL) ? static_cast<int>(rank) * kBHalf : 0);
      for (int kb = 0; kb < unkb; ++kb) {
        // paired release (even STAGES): the even stage waits for its pair
        if (lane == 0 && (STAGES % 2 != 0 || (stage & 1) == 0))
          ok = mbar_wait(&empty[STAGES % 2 != 0 ? stage : (stage | 1)], phase ^ 1u, err, kErrWaitEmpty);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) {
          uint8_t* sa = smem + stage * S::kStage;
          uint8_t* sb = sa + kABytes;
          uint64_t* bar = &full[stage];
          if (PAIR && BMODE == B_SPLIT3F) {
            // A hi | A lo | B hi | B lo of one k-block, all four into this stage
            if (rank == 0) mbar_arrive_expect_tx(bar, 2 * S::kStage);
            const uint32_t lbar = mapa_shared(smem_u32(bar), 0);
            const int k0 = (ukb0 + kb) * BK;
#pragma unroll
            for (int hl = 0; hl < 2; ++hl) {
              uint8_t* a_dst = sa + hl * kABytes;
              const CUtensorMap* ma = hl ? &tmA2 : &tmA;
              if (A_MN) {
#pragma unroll
                for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * 8192, ma, lbar, m0 + j * 64, k0);
              } else {
                tma_load_2d_pair(a_dst, ma, lbar, k0, m0);
              }
              uint8_t* b_dst = sa + 2 * kABytes + hl * S::kBBytes;
              const CUtensorMap* mb = hl ? &tmB2 : &tmB;
#pragma unroll
              for (int j = 0; j < kBHalf / 64; ++j) tma_load_2d_pair(b_dst + j * 8192, mb, lbar, n0 + j * 64, k0);
            }
            issued |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
          } else if (PAIR) {
            // both CTAs' copies complete on the leader's barrier
            if (rank == 0) mbar_arrive_expect_tx(bar, 2 * S::kStage);
            const uint32_t lbar = mapa_shared(smem_u32(bar), 0);
            const bool ext = (BMODE == B_KEXT) && kb >= p.k_blocks;
            const int seg = BMODE == B_SPLIT3 ? kb / p.k_blocks : 0;  // SPLIT3: hi.lo, lo.hi, hi.hi
            const CUtensorMap* ma = (ext || (BMODE == B_SPLIT3 && seg == 1)) ? &tmA2 : &tmA;
            const CUtensorMap* mb = (ext || (BMODE == B_SPLIT3 && seg == 0)) ? &tmB2
                                    : ((BMODE == B_DUAL && rank == 1) ? &tmB2 : &tmB);
            const int k0 = (ext ? kb - p.k_blocks : ukb0 + kb - seg * p.k_blocks) * BK;
            if (A_MN) {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) {
                if (BATCHED)
                  tma_load_3d_pair(sa + j * 8192, ma, lbar, m0 + j * 64, k0, b);
                else
                  tma_load_2d_pair(sa + j * 8192, ma, lbar, m0 + j * 64, k0);
              }
            } else {
              if (BATCHED)
                tma_load_3d_pair(sa, ma, lbar, k0, m0, b);
              else
                tma_load_2d_pair(sa, ma, lbar, k0, m0);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < kBHalf / 64; ++j) {
                if (BATCHED)
                  tma_load_3d_pair(sb + j * 8192, mb, lbar, n0 + j * 64, k0, b);
                else
                  tma_load_2d_pair(sb + j * 8192, mb, lbar, n0 + j * 64, k0);
              }
            } else {
              // K-major B (rows = this CTA's kBHalf output columns, 64 k per
              // row): one box, the layout of a K-major A tile
              if (BATCHED)
                tma_load_3d_pair(sb, mb, lbar, k0, n0, b);
              else
                tma_load_2d_pair(sb, mb, lbar, k0, n0);
            }
            issued |= 1u << stage;
            last_par = (last_par & ~(1u << stage)) | (phase << stage);
          }
        }
        if (!PAIR && lane == 0) {
          uint8_t* sa = smem + stage * S::kStage;
          uint8_t* sb = sa + kABytes;
          uint64_t* bar = &full[stage];
          mbar_arrive_expect_tx(bar, S::kStage);
          const bool ext = (BMODE == B_KEXT) && kb >= p.k_blocks;
          const int seg = BMODE == B_SPLIT3 ? kb / p.k_blocks : 0;  // SPLIT3: hi.lo, lo.hi, hi.hi
          const CUtensorMap* ma = (ext || (BMODE == B_SPLIT3 && seg == 1)) ? &tmA2 : &tmA;
          const CUtensorMap* mb = (ext || (BMODE == B_SPLIT3 && seg == 0)) ? &tmB2 : &tmB;
          const int k0 = (ext ? kb - p.k_blocks : kpart0 + kb - seg * p.k_blocks) * BK;
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
    // Every issued copy must land before the CTA may exit (in pair mode the
    // copies complete on the leader's barriers; the final cluster barrier
    // keeps the peer alive until the leader has drained).
    if (lane == 0 && (!PAIR || rank == 0)) {
      for (int s = 0; s < STAGES; ++s)
        if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp == 1 && PAIR && rank != 0) {
    // the peer CTA of a pair issues no MMAs (its warp 1 only owns TMEM)
  } else if (warp == 1) {
    // -------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    bool any = false;
    const long long my_work =
        units > first_unit ? static_cast<long long>((units - 1 - first_unit) / unit_stride + 1) * subs : 0;
    for (long long w = 0; w < my_work && ok; ++w) {
      const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
      int ukb0 = 0, unkb = k_total;
      if (TAIL) unit_kblocks(first_unit + static_cast<int>(w / subs) * unit_stride, p, k_total, ukb0, unkb);
      for (int kb = 0; kb < unkb; ++kb) {
        // the scheduler warp has seen this stage loaded (and, for kb == 0,
        // the accumulator free)
        ok = go_barrier64<kGoBarrier>(true);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0 && BMODE == B_SPLIT3F) {
          // corrections (hi.lo, lo.hi) into columns [0, BN), hi.hi into [BN, 2 BN)
          const uint32_t ah_addr = smem_u32(smem + stage * S::kStage);
          const uint32_t al_addr = ah_addr + kABytes;
          const uint32_t bh_addr = ah_addr + 2 * kABytes;
          const uint32_t bl_addr = bh_addr + S::kBBytes;
          const uint32_t d_corr = tmem_base;
          const uint32_t d_main = tmem_base + static_cast<uint32_t>(BN);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            auto adesc = [&](uint32_t base) {
              return A_MN ? smem_desc_sw128(base + kk * 2048, 8192, 1024) : smem_desc_sw128(base + kk * 32, 16, 1024);
            };
            auto bdesc = [&](uint32_t base) {
              return B_MN ? smem_desc_sw128(base + kk * 2048, 8192, 1024) : smem_desc_sw128(base + kk * 32, 16, 1024);
            };
            const uint32_t first = (kb | kk) != 0 ? 1u : 0u;
            umma_bf16_pair(d_corr, adesc(ah_addr), bdesc(bl_addr), kIdesc, first);
            umma_bf16_pair(d_corr, adesc(al_addr), bdesc(bh_addr), kIdesc, 1u);
            umma_bf16_pair(d_main, adesc(ah_addr), bdesc(bh_addr), kIdesc, first);
          }
          if (STAGES % 2 != 0 || (stage & 1)) umma_commit_pair(&empty[stage], 0x3);
          any = true;
        } else if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * S::kStage);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            if (PAIR)
              umma_bf16_pair(d, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
            else
              umma_bf16(d, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          // With an even number of stages, stages are released in pairs: one
          // commit after the odd stage also covers the even one before it (a
          // commit costs the issuing thread ~one MMA; halving them measured
          // 1.9-2.3 % faster on the large pair GEMMs)
          if (STAGES % 2 != 0 || (stage & 1)) {
            if (PAIR)
              umma_commit_pair(&empty[stage], 0x3);
            else
              umma_commit(&empty[stage]);
          }
          any = true;
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) {
        if (PAIR)
          umma_commit_pair(&tfull[acc], 0x3);
        else
          umma_commit(&tfull[acc]);
      }
      __syncwarp();
      if (kOneAcc) {
        acc_phase ^= 1u;
      } else {
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
    // All issued MMAs must finish before TMEM is released.
    if (lane == 0 && any) {
      if (PAIR)
        umma_commit_pair(drain, 0x1);
      else
        umma_commit(drain);
      mbar_wait(drain, 0, err, kErrWaitDrain);
    }
    __syncwarp();
  } else if (warp == sched_warp(EPI, BATCHED)) {
    // --------------------------------------------------------- scheduler
    // Same walk over work units and k-blocks as the MMA issuer, one go
    // barrier per k-block.  In a pair only the leader CTA issues MMAs.
    if (!(PAIR && rank != 0)) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const long long my_work =
          units > first_unit ? static_cast<long long>((units - 1 - first_unit) / unit_stride + 1) * subs : 0;
      for (long long w = 0; w < my_work && ok; ++w) {
        int ukb0 = 0, unkb = k_total;
        if (TAIL) unit_kblocks(first_unit + static_cast<int>(w / subs) * unit_stride, p, k_total, ukb0, unkb);
        for (int kb = 0; kb < unkb; ++kb) {
          bool good = true;
          if (lane == 0) {
            if (kb == 0) good = mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kErrWaitAccumFree);
            if (good) good = mbar_wait(&full[stage], phase, err, kErrWaitFull);
          }
          ok = go_barrier64<kGoBarrier>(__shfl_sync(0xffffffffu, good, 0));
          if (!ok) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (kOneAcc) {
          acc_phase ^= 1u;
        } else {
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
        }
      }
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int part = (warp - 2) >> 2;  // which group of the tile's columns (more than 4 epilogue warps)
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    float row_max = -INFINITY, row_sum = 0.f;  // EPI_SOFTMAX running statistics
    uint32_t xunit = 0;                          // CSPLIT: statistics exchanges done
    uint8_t* warp_stage = smem + S::kStageOff + (warp - 2) * 4096;
    int sbuf = 0;
    // the tail counters are zeroed by the kernel this one may overlap
    if (TAIL) pdl_wait();
    for (int unit = first_unit, sub = 0; unit < units;) {
      int b, mt, nt;
      work_coords<EPI>(unit, sub, p, b, mt, nt, n_base, n_count);
      const int cur_sub = sub;
      const int cur_unit = unit;
      if (++sub == subs) {
        sub = 0;
        unit += unit_stride;
      }
      const int row0 = mt * tile_rows + static_cast<int>(row_rank) * BM;  // this CTA's first output row
      ok = mbar_wait(&tfull[acc], acc_phase, err, kErrWaitAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int gm = row0 + row;
      const bool row_ok = gm < p.M;
      if (TAIL && cur_unit >= p.tail_first) {
        // One K part of a tail tile: this CTA's 128 x BN fp32 partial goes to
        // global memory column-major (a warp stores 128 contiguous bytes per
        // column).  The part that arrives last sums all parts in part order --
        // its own from TMEM, the others brought into the operand ring by bulk
        // copies: a tail unit is its CTA's last, so the ring is idle.
        const int t = cur_unit - p.tail_first;
        const int tt = t / p.tail_parts;
        const int kpart = t - tt * p.tail_parts;
        constexpr int kSlab = BN * BM;  // floats per (tile, part, CTA of the pair)
        auto slab = [&](int q) {
          return p.tail_part + (static_cast<size_t>(tt * p.tail_parts + q) * 2 + row_rank) * kSlab;
        };
        float* mine = slab(kpart);
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          uint32_t r[2][32];
          tmem_ld_32x32b_x32(tb + c * 32, r[0]);
          tmem_ld_32x32b_x32(tb + c * 32 + 32, r[1]);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < 32; ++j) mine[((c + h) * 32 + j) * BM + row] = __uint_as_float(r[h][j]);
        }
        __threadfence();
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("bar.sync 3, %0;" ::"n"(kEpi) : "memory");
        if (threadIdx.x == 64) tmem_holder[1] = atomicAdd(&p.tail_cnt[tt * 2 + row_rank], 1u);
        asm volatile("bar.sync 3, %0;" ::"n"(kEpi) : "memory");
        if (tmem_holder[1] == static_cast<uint32_t>(p.tail_parts - 1)) {
          // columns per round: the other parts' slices of a round fill at most the ring
          constexpr int kRingFloats = STAGES * static_cast<int>(S::kStage) / 4;
          int cr = BN;
          while (cr > 32 && (p.tail_parts - 1) * cr * BM > kRingFloats) cr >>= 1;
          float* ring = reinterpret_cast<float*>(smem);
          const int n0 = nt * BN;
          uint32_t tphase = 0;
          float tss = 0.f;  // EPI_RESID_BF16: this row's sum of squares of y over the tile
#pragma unroll 1
          // every epilogue thread runs every round (the named barrier below
          // counts them), whatever happened to its waits
          for (int c0 = 0; c0 < BN; c0 += cr) {
            if (threadIdx.x == 64 && ok) {
              __threadfence();
              asm volatile("fence.proxy.async.global;" ::: "memory");
              fence_proxy_async_smem();  // the previous round's reads of the ring come first
              mbar_arrive_expect_tx(tail_bar, static_cast<uint32_t>((p.tail_parts - 1) * cr * BM * 4));
              int slot = 0;
              for (int q = 0; q < p.tail_parts; ++q) {
                if (q == kpart) continue;
                bulk_load_1d(ring + slot * cr * BM, slab(q) + c0 * BM, static_cast<uint32_t>(cr * BM * 4), tail_bar);
                ++slot;
              }
            }
            if (ok) ok = mbar_wait(tail_bar, tphase, err, kErrWaitFull);
            ok = __all_sync(0xffffffffu, ok);
            tphase ^= 1u;
            if (ok) {
#pragma unroll 1
              for (int c = c0 / 32; c < (c0 + cr) / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tb + c * 32, r);
                tmem_ld_wait();
                if (n0 + c * 32 >= p.N) continue;
                float sum[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[j] = 0.f;
                int slot = 0;
                for (int q = 0; q < p.tail_parts; ++q) {
                  if (q == kpart) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] += __uint_as_float(r[j]);
                  } else {
                    const float* src = ring + slot * cr * BM + (c * 32 - c0) * BM + row;
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[j] += src[j * BM];
                    ++slot;
                  }
                }
                if (EPI == EPI_RESID_BF16) {
                  // y = acc + z, as the residual epilogue forms it
                  const int gn = n0 + c * 32;
                  const __nv_bfloat16* zrow = p.z + static_cast<int64_t>(gm) * p.ldz;
                  if (row_ok && gn + 32 <= p.N) {
                    const uint4* zs = reinterpret_cast<const uint4*>(zrow + gn);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      float zf[8];
                      unpack_bf16x8(zs[q], zf);
#pragma unroll
                      for (int e = 0; e < 8; ++e) sum[8 * q + e] += zf[e];
                    }
                  } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                      sum[j] = (row_ok && gn + j < p.N) ? sum[j] + __bfloat162float(zrow[gn + j]) : 0.f;
                  }
#pragma unroll
                  for (int j = 0; j < 32; ++j) tss = fmaf(sum[j], sum[j], tss);
                }
                uint32_t w[16];
#pragma unroll
                for (int q = 0; q < 16; ++q) w[q] = pack_bf16x2(sum[2 * q], sum[2 * q + 1]);
                stage_store<false>(w, warp_stage, sbuf, &tmOut, n0 + c * 32, row0 + quad * 32, 0, lane);
              }
            }
            asm volatile("bar.sync 3, %0;" ::"n"(kEpi) : "memory");  // the ring is read before it is refilled
          }
          if (EPI == EPI_RESID_BF16 && row_ok && ok) atomicAdd(&p.rowsq[gm], tss);
          if (threadIdx.x == 64) p.tail_cnt[tt * 2 + row_rank] = 0u;
        }
        if (!ok) break;
      } else if (EPI == EPI_BF16) {
        const int n0 = nt * BN;
        constexpr int kChunks = BN / 32 / (epi_warps(EPI, BATCHED) / 4);  // 32-column chunks per warp
        // two 32-column chunks per TMEM wait
#pragma unroll 1
        for (int c = part * kChunks; c < (part + 1) * kChunks; c += 2) {
          uint32_t r[2][32];
          tmem_ld_32x32b_x32(tb + c * 32, r[0]);
          tmem_ld_32x32b_x32(tb + c * 32 + 32, r[1]);
          tmem_ld_wait();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (n0 + (c + h) * 32 < p.N) {
              uint32_t w[16];
#pragma unroll
              for (int q = 0; q < 16; ++q)
                w[q] = pack_bf16x2(__uint_as_float(r[h][2 * q]), __uint_as_float(r[h][2 * q + 1]));
              stage_store<BATCHED>(w, warp_stage, sbuf, &tmOut, n0 + (c + h) * 32, row0 + quad * 32, b, lane);
            }
          }
        }
      } else if (EPI == EPI_SWIGLU) {
        // gate in accumulator columns [0, BN/2), up in [BN/2, BN)
        const int n0 = nt * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tb + c * 32, rg);
          tmem_ld_32x32b_x32(tb + BN / 2 + c * 32, ru);
          tmem_ld_wait();
          if (n0 + c * 32 < p.N) {
            uint32_t w[16];
#pragma unroll
            for (int q = 0; q < 16; ++q)
              w[q] = pack_bf16x2(silu_f32(__uint_as_float(rg[2 * q])) * __uint_as_float(ru[2 * q]),
                                 silu_f32(__uint_as_float(rg[2 * q + 1])) * __uint_as_float(ru[2 * q + 1]));
            stage_store<false>(w, warp_stage, sbuf, &tmOut, n0 + c * 32, row0 + quad * 32, 0, lane);
          }
        }
      } else if (EPI == EPI_SOFTMAX) {
        // pass 0 (cur_sub < n_tiles): online max / sum of exp over this
        // thread's quarter of each tile row; after the last tile the four
        // parts of every row are merged through shared memory.  pass 1: out =
        // exp(x - max) / sum, bf16.  The thread's 64 columns come out of TMEM
        // in one batch (one wait), then one max, at most one rescale of the
        // running sum, and 32 independent pairs of exponentials (a few of every
        // 16 pairs by the FMA-pipe polynomial, the rest on MUFU).
        constexpr float kL2e = 1.4426950408889634f;
        // exponential pairs taken by the FMA-pipe polynomial (bit i of 16):
        // 4 of 16 in the statistics pass, 2 of 16 in the output pass (swept:
        // all on MUFU or more on the FMA pipe in either pass is slower)
        constexpr uint32_t kPolyStats = 0x1111u;
        constexpr uint32_t kPolyOut = 0x0101u;
        constexpr int kParts = epi_warps(EPI_SOFTMAX) / 4;
        constexpr int kHalfCols = BN / kParts;  // columns per thread
        const int c0 = nt * BN + part * kHalfCols;  // first column of this part of the tile
        const int lim = p.N - c0;                   // valid columns of this part
        if (cur_sub == 0) {
          row_max = -INFINITY;
          row_sum = 0.f;
        }
        const float2 sc2 = make_float2(kL2e, kL2e);
        uint32_t r[kHalfCols];
#pragma unroll
        for (int c = 0; c < kHalfCols / 32; ++c)
          tmem_ld_32x32b_x32(tb + part * kHalfCols + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
        tmem_ld_wait();
        if (cur_sub < n_count) {
          if (lim > 0) {
            if (lim < kHalfCols) {
#pragma unroll
              for (int j = 0; j < kHalfCols; ++j)
                if (j >= lim) r[j] = 0xff800000u;  // -inf: no weight
            }
            float m8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) m8[k] = fmaxf(__uint_as_float(r[k]), __uint_as_float(r[k + 8]));
#pragma unroll
            for (int j = 16; j < kHalfCols; j += 16)
#pragma unroll
              for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], __uint_as_float(r[j + k]), __uint_as_float(r[j + 8 + k]));
            const float cm = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), m8[6]), m8[7]);
            if (cm > row_max) {  // rescale the running sum to the new max
              row_sum *= exp2_approx((row_max - cm) * kL2e);
              row_max = cm;
            }
            const float mb = row_max * kL2e;
            const float2 nm2 = make_float2(-mb, -mb);
            float2 s2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                            make_float2(0.f, 0.f)};
#pragma unroll
            for (int j = 0; j < kHalfCols / 2; ++j) {
              const float2 a =
                  __ffma2_rn(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), sc2, nm2);
              const float2 e = ((kPolyStats >> (j & 15)) & 1u) ? exp2_poly2_lp(a)
                                                              : make_float2(exp2_approx(a.x), exp2_approx(a.y));
              s2[j & 3] = __fadd2_rn(s2[j & 3], e);
            }
            row_sum += ((s2[0].x + s2[0].y) + (s2[1].x + s2[1].y)) + ((s2[2].x + s2[2].y) + (s2[3].x + s2[3].y));
          }
          if (cur_sub == n_count - 1) {
            // merge the column parts of each row
            float2* stat = reinterpret_cast<float2*>(smem + S::kStatOff);
            stat[part * 128 + row] = make_float2(row_max, row_sum);
            asm volatile("bar.sync 1, %0;" ::"n"(kEpi) : "memory");
            float2 ps[kParts];
            float m = -INFINITY;
#pragma unroll
            for (int q = 0; q < kParts; ++q) {
              ps[q] = stat[q * 128 + row];
              m = fmaxf(m, ps[q].x);
            }
            float sum = 0.f;
#pragma unroll
            for (int q = 0; q < kParts; ++q) sum += ps[q].y * exp2_approx((ps[q].x - m) * kL2e);
            row_sum = sum;
            row_max = m;
            asm volatile("bar.sync 1, %0;" ::"n"(kEpi) : "memory");
            if (CSPLIT) {
              // swap the row statistics with the peer CTA (the other half of
              // the row block's columns): part-0 threads write this CTA's
              // statistics into the peer's exchange buffer and release-arrive
              // on its barrier; everyone waits for the peer's statistics
              float2* xch = stat + kParts * 128;                            // [2][128]
              uint64_t* xbar = reinterpret_cast<uint64_t*>(xch + 2 * 128);  // [2]
              const int buf = static_cast<int>(xunit & 1u);
              if (part == 0) {
                st_cluster_f32x2(mapa_shared(smem_u32(&xch[buf * 128 + row]), rank ^ 1u), row_max, row_sum);
                mbar_arrive_remote(mapa_shared(smem_u32(&xbar[buf]), rank ^ 1u));
              }
              ok = mbar_wait_cluster(&xbar[buf], (xunit >> 1) & 1u, err, kErrWaitPeer);
              ok = __all_sync(0xffffffffu, ok);
              if (!ok) break;
              const float2 o = xch[buf * 128 + row];
              const float m2 = fmaxf(row_max, o.x);
              row_sum = row_sum * exp2_approx((row_max - m2) * kL2e) + o.y * exp2_approx((o.x - m2) * kL2e);
              row_max = m2;
              ++xunit;
            }
          }
        } else {
          // exp(x - max) / sum = 2^(x * log2 e - (max * log2 e + log2 sum))
          const float mb = fmaf(row_max, kL2e, __log2f(row_sum));
          const float2 nm2 = make_float2(-mb, -mb);
#pragma unroll
          for (int c = 0; c < kHalfCols / 32; ++c) {
            const int gn = c0 + c * 32;
            if (gn >= p.N) continue;
            uint32_t w[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const float2 a = __ffma2_rn(
                  make_float2(__uint_as_float(r[c * 32 + 2 * q]), __uint_as_float(r[c * 32 + 2 * q + 1])), sc2, nm2);
              const float2 e = ((kPolyOut >> q) & 1u) ? exp2_poly2_lp(a)
                                                        : make_float2(exp2_approx(a.x), exp2_approx(a.y));
              w[q] = pack_bf16x2(e.x, e.y);
            }
            stage_store<true>(w, warp_stage, sbuf, &tmOut, gn, row0 + quad * 32, b, lane);
          }
        }
      } else if (EPI == EPI_F32OUT) {
        // fp32 output: each 32-column TMEM chunk leaves as two 32-row x
        // 16-column boxes (64-byte rows: the bf16 staging geometry)
        const int n0 = nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          if (BMODE == B_SPLIT3F) {
            // hi.hi + (hi.lo + lo.hi)
            uint32_t rm[32];
            tmem_ld_32x32b_x32(tb + BN + c * 32, rm);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; ++q) r[q] = __float_as_uint(__uint_as_float(rm[q]) + __uint_as_float(r[q]));
          }
          tmem_ld_wait();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int gn = n0 + c * 32 + hh * 16;
            if (gn >= p.N) continue;
            uint32_t w[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) w[q] = r[hh * 16 + q];
            stage_store<false>(w, warp_stage, sbuf, &tmOut, gn, row0 + quad * 32, 0, lane);
          }
        }
      } else if (EPI == EPI_F32) {
        // this k part's fp32 partial tile, row by row (each thread one row,
        // 128 contiguous bytes per 32-column chunk)
        float* orow = static_cast<float*>(p.out) +
                      (static_cast<int64_t>(cur_unit % p.k_split) * p.M + gm) * p.ldo;
        const int n0 = nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (!row_ok || gn >= p.N) continue;
          if (gn + 32 <= p.N) {
            float4* dst = reinterpret_cast<float4*>(orow + gn);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                   __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q)
              if (gn + q < p.N) orow[gn + q] = __uint_as_float(r[q]);
          }
        }
      } else if (EPI == EPI_RESID_BF16) {
        // y = acc + z -> bf16 out (TMA store), fp32 row sum of squares of y
        const int n0 = nt * BN;
        const __nv_bfloat16* zrow = p.z + static_cast<int64_t>(gm) * p.ldz;
        float ss0 = 0.f, ss1 = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + c * 32, r);
          tmem_ld_wait();
          const int gn = n0 + c * 32;
          if (gn >= p.N) continue;
          float y[32];
          if (row_ok && gn + 32 <= p.N) {
            const uint4* zs = reinterpret_cast<const uint4*>(zrow + gn);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float zf[8];
              unpack_bf16x8(zs[q], zf);
#pragma unroll
              for (int e = 0; e < 8; ++e) y[8 * q + e] = __uint_as_float(r[8 * q + e]) + zf[e];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              y[j] = (row_ok && gn + j < p.N) ? __uint_as_float(r[j]) + __bfloat162float(zrow[gn + j]) : 0.f;
          }
          uint32_t w[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            ss0 = fmaf(y[2 * q], y[2 * q], ss0);
            ss1 = fmaf(y[2 * q + 1], y[2 * q + 1], ss1);
            w[q] = pack_bf16x2(y[2 * q], y[2 * q + 1]);
          }
          stage_store<false>(w, warp_stage, sbuf, &tmOut, gn, row0 + quad * 32, 0, lane);
        }
        if (row_ok) atomicAdd(&p.rowsq[gm], ss0 + ss1);
      }
      tc_fence_before();
      if (PAIR && rank != 0)
        mbar_arrive_remote(mapa_shared(smem_u32(&tempty[acc]), 0));
      else
        mbar_arrive(&tempty[acc]);
      if (kOneAcc) {
        acc_phase ^= 1u;
      } else {
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();  // every TMA store issued by this warp has completed
    __syncwarp();
  }

  tc_fence_before();
  if (kCluster)
    cluster_sync_all();  // neither CTA leaves while its peer may still touch it
  else
    __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    if (PAIR)
      tmem_dealloc_pair(tmem_base, kCols);
    else
      tmem_dealloc(tmem_base, kCols);
  }
}

// Host-side launch of one instantiation.
// pdl: launch with programmatic stream serialization, so the kernel's
// prologue (barrier init, TMEM allocation) overlaps the tail of the previous
// kernel in the stream, which must call pdl_trigger(); the producer's
// pdl_wait() orders every input read after that kernel's completion.
template <int BN, bool A_MN, bool B_MN, int EPI, bool BATCHED, int BMODE, int STAGES, bool PAIR = false,
          bool CSPLIT = false, bool TAIL = false>
kda_status launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2, const CUtensorMap& b2,
                  const CUtensorMap& out, const Params& p, unsigned* err, cudaStream_t st, bool pdl = false) {
  auto kern = gemm_kernel<BN, A_MN, B_MN, EPI, BATCHED, BMODE, STAGES, PAIR, CSPLIT, TAIL>;
  constexpr size_t smem = Smem<BN, STAGES, PAIR, epi_warps(EPI, BATCHED),
                               EPI == EPI_SOFTMAX ? epi_warps(EPI) / 4 + (CSPLIT ? 3 : 0) : 0,
                               BMODE == B_SPLIT3F ? 2 : 1>::kBytes;
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      set_error("gemm: cudaFuncSetAttribute(%zu B smem): %s", smem, cudaGetErrorString(e));
      return KDA_CUDA_ERROR;
    }
    attr_set[dev].store(true, std::memory_order_release);
  }
  const long long tiles = num_units<EPI>(p);
  if (tiles <= 0) return KDA_OK;
  int grid;
  if (PAIR || CSPLIT) {
    const int pairs = num_sms() / 2;
    grid = 2 * static_cast<int>(tiles < pairs ? tiles : pairs);
  } else {
    grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads_for(EPI, BATCHED));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (PAIR || CSPLIT) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 2;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, b, a2, b2, out, p, err);
  if (e != cudaSuccess) {
    set_error("gemm_kernel%s: %s", PAIR ? " (CTA pairs)" : "", cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  return launch_status("gemm_kernel");
}

}  // namespace gemm
}  // namespace kda
