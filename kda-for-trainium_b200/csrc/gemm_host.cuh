// Host-side plumbing shared by the contraction translation units (gemm.cu,
// gemm_f32.cu, backward.cu): tensor-map encoders, tile-schedule parameters,
// the plain GEMM launcher, the RMS row pre-pass kernels, a workspace carver.
// Everything lives in an anonymous namespace, so each including unit gets its
// own copies; it launches the engine with the unit's device error word, which
// the unit provides as gemm_err_word() before including this header.
#pragma once

#include "gemm.cuh"

namespace kda {
namespace {

using gemm::Params;

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int cdiv(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }
inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// 2-D bf16 operand stored row-major [outer][inner] (inner contiguous, row
// stride ld elements); box {64 inner, box_outer}.
kda_status tmap2(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t ld, uint32_t box_outer) {
  const uint64_t dims[2] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(outer)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {64, box_outer};
  return make_tmap_bf16(m, base, 2, dims, strides, box);
}
// 3-D: [batch][outer][inner].
kda_status tmap3(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
                 int64_t bstride, uint32_t box_outer) {
  const uint64_t dims[3] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(outer),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(bstride) * 2};
  const uint32_t box[3] = {64, box_outer, 1};
  return make_tmap_bf16(m, base, 3, dims, strides, box);
}

// bf16 output [outer rows][ld] with `inner` valid columns, written by TMA
// stores of 32 x 32 boxes staged with the 64-byte swizzle.
kda_status tmap_out2(CUtensorMap* m, void* base, int64_t inner, int64_t outer, int64_t ld) {
  const uint64_t dims[2] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(outer)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {32, 32};
  return make_tmap_bf16_sw(m, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}
// fp32 output [outer rows][ld] with `inner` valid columns, TMA stores of 32-row
// x 16-column boxes (64-byte rows) staged with the 64-byte swizzle.
kda_status tmap_out2_f32(CUtensorMap* m, void* base, int64_t inner, int64_t outer, int64_t ld) {
  const uint64_t dims[2] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(outer)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 4};
  const uint32_t box[2] = {16, 32};
  return make_tmap_f32_sw(m, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}
kda_status tmap_out3(CUtensorMap* m, void* base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
                     int64_t bstride) {
  const uint64_t dims[3] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(outer),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(bstride) * 2};
  const uint32_t box[3] = {32, 32, 1};
  return make_tmap_bf16_sw(m, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
}

#define KDA_TRY(expr)                     \
  do {                                    \
    kda_status _s = (expr);               \
    if (_s != KDA_OK) return _s;          \
  } while (0)

// pair = true: tiles of 256 rows shared by a CTA pair (tcgen05 cta_group::2).
Params base_params(int64_t M, int64_t N, int64_t K, int bn_out, bool pair = false) {
  Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.k_blocks = cdiv(K, gemm::BK);
  p.k_blocks2 = 0;
  p.batch = 1;
  const int tile_rows = pair ? 2 * gemm::BM : gemm::BM;
  p.m_tiles = cdiv(M, tile_rows);
  p.n_tiles = cdiv(N, bn_out);
  // Raster: CTAs walk m fastest inside a group of group_m m-tiles.  When the
  // whole A operand fits comfortably in L2 (126 MB), one group spans all of M:
  // A stays resident and B streams from DRAM exactly once.  Otherwise the
  // group holds ~48 MB of A rows so neither operand is re-read more than a
  // few times.
  const double a_bytes = static_cast<double>(M) * K * 2;
  if (a_bytes <= 64.0 * (1 << 20)) {
    p.group_m = p.m_tiles;
  } else {
    int g = static_cast<int>((48.0 * (1 << 20)) / (static_cast<double>(tile_rows) * K * 2));
    p.group_m = g < 1 ? 1 : (g > p.m_tiles ? p.m_tiles : g);
  }
  p.ldo = N;
  p.out_bstride = 0;
  p.k_split = 1;
  return p;
}

kda_status check_dims(const char* op, int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0 || M > (1ll << 31) - 256 || N > (1ll << 31) - 256 || K > (1ll << 31) - 256) {
    set_error("%s: bad dimensions M=%lld K=%lld N=%lld", op, (long long)M, (long long)K, (long long)N);
    return KDA_INVALID_ARG;
  }
  return KDA_OK;
}

// Tail split of the pair GEMM (M > 128, K >= 256, N > 128): when the pair
// tiles leave a last, partial wave of `rem` tiles on the CTA pairs, those
// tiles are cut into `parts` K ranges (parts = pairs / rem, at most
// KDA_TAIL_MAX_PARTS, at least 4 k-blocks each) so the idle pairs share them;
// every pair then holds at most one part, as its last unit.  parts = 0: no
// split.
#ifndef KDA_TAIL_MAX_PARTS
#define KDA_TAIL_MAX_PARTS 4
#endif
struct TailPlan {
  int parts = 0, first = 0, tiles = 0, kb = 0;
  size_t part_bytes = 0, cnt_bytes = 0;  // fp32 partials, counters (each 256-aligned)
};
inline TailPlan tail_plan(int64_t M, int64_t K, int64_t N) {
  TailPlan t;
  if (!(N > 128 && M > gemm::BM && K >= 256)) return t;
  const int pairs = num_sms() / 2;
  const int tiles = cdiv(M, 2 * gemm::BM) * cdiv(N, 256);
  const int kblocks = cdiv(K, gemm::BK);
  if (pairs <= 0) return t;
  const int rem = tiles % pairs;
  if (rem == 0) return t;
  int parts = pairs / rem;
  if (parts > KDA_TAIL_MAX_PARTS) parts = KDA_TAIL_MAX_PARTS;
  if (parts > kblocks / 4) parts = kblocks / 4;
  if (parts < 2) return t;
  t.parts = parts;
  t.first = tiles - rem;
  t.tiles = rem;
  t.kb = cdiv(kblocks, parts);
  t.part_bytes = align256(static_cast<size_t>(rem) * parts * 2 * 256 * gemm::BM * 4);
  t.cnt_bytes = align256(static_cast<size_t>(rem) * 2 * 4);
  return t;
}

// out (M,N) bf16 = A (M,K) K-major @ B (K,N) MN-major, in two steps so a
// caller can encode the tensor maps (host work) before it launches the kernel
// that produces A: plan_plain_gemm() encodes, launch_plain_gemm() launches.
// With `tail` (a workspace of tail.part_bytes + tail.cnt_bytes: partials,
// then counters that must be zero at launch) the pair GEMM splits its tail.
struct PlainGemm {
  CUtensorMap ta, tb, to;
  Params p;
  int variant;  // 0: 1-CTA BN=128, 1: CTA pairs BN=256, 2: 1-CTA BN=256
};

kda_status plan_plain_gemm(PlainGemm& g, const void* A, const void* B, void* out, int64_t M, int64_t K, int64_t N,
                           const TailPlan* tail = nullptr, void* tail_ws = nullptr) {
  KDA_TRY(tmap2(&g.ta, A, K, M, K, 128));
  KDA_TRY(tmap2(&g.tb, B, N, K, N, 64));
  KDA_TRY(tmap_out2(&g.to, out, N, M, N));
  if (N <= 128) {
    g.variant = 0;
    g.p = base_params(M, N, K, 128);
  } else if (M > gemm::BM && K >= 256) {
    g.variant = 1;
    g.p = base_params(M, N, K, 256, true);
    if (tail && tail->parts > 1 && tail_ws) {
      g.p.tail_parts = tail->parts;
      g.p.tail_first = tail->first;
      g.p.tail_kb = tail->kb;
      g.p.tail_part = static_cast<float*>(tail_ws);
      g.p.tail_cnt = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(tail_ws) + tail->part_bytes);
    }
  } else {
    g.variant = 2;
    g.p = base_params(M, N, K, 256);
  }
  g.p.out = out;
  return KDA_OK;
}

// pdl: the previous kernel in the stream is one of ours that calls
// pdl_trigger() (the GEMM's prologue overlaps its tail).
kda_status launch_plain_gemm(const PlainGemm& g, cudaStream_t st, bool pdl) {
  unsigned* err = gemm_err_word();
  switch (g.variant) {
    case 0:
      return gemm::launch<128, false, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 6>(g.ta, g.tb, g.ta, g.tb, g.to,
                                                                                      g.p, err, st, pdl);
    case 1:
      if (g.p.tail_parts > 1)
        return gemm::launch<256, false, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 6, true, false, true>(
            g.ta, g.tb, g.ta, g.tb, g.to, g.p, err, st, pdl);
      return gemm::launch<256, false, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 6, true>(
          g.ta, g.tb, g.ta, g.tb, g.to, g.p, err, st, pdl);
    default:
      return gemm::launch<256, false, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 4>(g.ta, g.tb, g.ta, g.tb, g.to,
                                                                                      g.p, err, st, pdl);
  }
}

kda_status plain_gemm(const void* A, const void* B, void* out, int64_t M, int64_t K, int64_t N, cudaStream_t st) {
  PlainGemm g;
  KDA_TRY(plan_plain_gemm(g, A, B, out, M, K, N));
  return launch_plain_gemm(g, st, false);
}

// ------------------------------------------------------------ row statistics

// The first CTA of a pre-pass zeroes the GEMM's tail counters (n words; the
// GEMM queued behind the pre-pass waits for its completion before using them).
__device__ __forceinline__ void zero_words(unsigned* z, int n) {
  if (z && blockIdx.x == 0)
    for (int i = threadIdx.x; i < n; i += blockDim.x) z[i] = 0u;
}


// out = bf16((x [+ z]) * inv_rms * g): one warp per row, 8 rows per CTA,
// 16-byte loads; the row is read twice (sum of squares, then scale), the
// second time from L1/L2.  K % 8 == 0.
template <bool ADD>
__global__ void __launch_bounds__(256) rms_prep_kernel(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ z,
                                                       const float* __restrict__ g, float eps,
                                                       __nv_bfloat16* __restrict__ out, int M, int K, unsigned* zc,
                                                       int nz) {
  pdl_trigger();  // the GEMM queued behind this kernel may start its prologue
  zero_words(zc, nz);
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * K;
  const __nv_bfloat16* zr = ADD ? z + row * K : nullptr;
  float ss0 = 0.f, ss1 = 0.f;
  for (int k = lane * 8; k < K; k += 32 * 8) {
    float a[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(xr + k), a);
    if (ADD) {
      float b[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(zr + k), b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] += b[i];
    }
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      ss0 = fmaf(a[i], a[i], ss0);
      ss1 = fmaf(a[i + 1], a[i + 1], ss1);
    }
  }
  float tot = ss0 + ss1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
  __nv_bfloat16* orow = out + row * K;
  for (int k = lane * 8; k < K; k += 32 * 8) {
    float a[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(xr + k), a);
    if (ADD) {
      float b[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(zr + k), b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] += b[i];
    }
    float gv[8];
    if (g) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + k);
      const float4 g1 = *reinterpret_cast<const float4*>(g + k + 4);
      gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
      gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) gv[i] = 1.f;
    }
    uint4 o;
    o.x = pack_bf16x2(a[0] * inv * gv[0], a[1] * inv * gv[1]);
    o.y = pack_bf16x2(a[2] * inv * gv[2], a[3] * inv * gv[3]);
    o.z = pack_bf16x2(a[4] * inv * gv[4], a[5] * inv * gv[5]);
    o.w = pack_bf16x2(a[6] * inv * gv[6], a[7] * inv * gv[7]);
    *reinterpret_cast<uint4*>(orow + k) = o;
  }
}

// Same result for K = 256 * NC: the row stays in registers (lane l holds
// 16-byte chunks l, l + 32, ...), every load of the row is issued before the
// first use, and the row is read once.  Each warp takes RPW consecutive rows,
// all their loads in flight together (RPW = 2 when one row per warp would
// need more than one wave of CTAs).
template <bool ADD, int NC, int RPW>
__global__ void __launch_bounds__(256, 2) rms_prep_reg_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ z,
                                                           const float* __restrict__ g, float eps,
                                                           __nv_bfloat16* __restrict__ out, int M, unsigned* zc,
                                                           int nz) {
  pdl_trigger();  // the GEMM queued behind this kernel may start its prologue
  zero_words(zc, nz);
  constexpr int K = 256 * NC;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * RPW;
  if (row0 >= M) return;
  uint4 xv[RPW][NC], zv[RPW][ADD ? NC : 1];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (row0 + r < M) {
      const uint4* xr = reinterpret_cast<const uint4*>(x + (row0 + r) * K);
#pragma unroll
      for (int i = 0; i < NC; ++i) xv[r][i] = xr[i * 32 + lane];
      if (ADD) {
        const uint4* zr = reinterpret_cast<const uint4*>(z + (row0 + r) * K);
#pragma unroll
        for (int i = 0; i < NC; ++i) zv[r][i] = zr[i * 32 + lane];
      }
    }
  }
  // x (+ z) as fp32, unpacked from the packed registers on each use
  auto row_vals = [&](int r, int i, float (&v)[8]) {
    unpack_bf16x8(xv[r][i], v);
    if (ADD) {
      float b[8];
      unpack_bf16x8(zv[r][i], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += b[e];
    }
  };
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (row0 + r >= M) break;
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      float v[8];
      row_vals(r, i, v);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        ss0 = fmaf(v[e], v[e], ss0);
        ss1 = fmaf(v[e + 1], v[e + 1], ss1);
      }
    }
    float tot = ss0 + ss1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
    uint4* orow = reinterpret_cast<uint4*>(out + (row0 + r) * K);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int k = (i * 32 + lane) * 8;
      float a[8];
      row_vals(r, i, a);
      float gv[8];
      if (g) {
        const float4 g0 = *reinterpret_cast<const float4*>(g + k);
        const float4 g1 = *reinterpret_cast<const float4*>(g + k + 4);
        gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
        gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) gv[e] = 1.f;
      }
      uint4 o;
      o.x = pack_bf16x2(a[0] * inv * gv[0], a[1] * inv * gv[1]);
      o.y = pack_bf16x2(a[2] * inv * gv[2], a[3] * inv * gv[3]);
      o.z = pack_bf16x2(a[4] * inv * gv[4], a[5] * inv * gv[5]);
      o.w = pack_bf16x2(a[6] * inv * gv[6], a[7] * inv * gv[7]);
      orow[i * 32 + lane] = o;
    }
  }
}

// Same result for K = 2048 * NCH: one 256-thread CTA per row, thread t
// holding 16-byte chunks t, t + 256, ... in registers (every load issued
// before the first use); the sum of squares is reduced through shared memory.
template <bool ADD, int NCH>
__global__ void __launch_bounds__(256) rms_prep_cta_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ z,
                                                           const float* __restrict__ g, float eps,
                                                           __nv_bfloat16* __restrict__ out, unsigned* zc,
                                                           int nz) {
  pdl_trigger();  // the GEMM queued behind this kernel may start its prologue
  zero_words(zc, nz);
  constexpr int K = 2048 * NCH;
  __shared__ float part[8];
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
  const uint4* zr = ADD ? reinterpret_cast<const uint4*>(z + row * K) : nullptr;
  uint4 xv[NCH], zv[ADD ? NCH : 1];
#pragma unroll
  for (int i = 0; i < NCH; ++i) xv[i] = xr[i * 256 + tid];
  if (ADD) {
#pragma unroll
    for (int i = 0; i < NCH; ++i) zv[i] = zr[i * 256 + tid];
  }
  auto vals = [&](int i, float (&v)[8]) {
    unpack_bf16x8(xv[i], v);
    if (ADD) {
      float b[8];
      unpack_bf16x8(zv[i], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += b[e];
    }
  };
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    float v[8];
    vals(i, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += part[w];
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + row * K);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int k = (i * 256 + tid) * 8;
    float a[8];
    vals(i, a);
    float gv[8];
    if (g) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + k);
      const float4 g1 = *reinterpret_cast<const float4*>(g + k + 4);
      gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
      gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) gv[e] = 1.f;
    }
    uint4 o;
    o.x = pack_bf16x2(a[0] * inv * gv[0], a[1] * inv * gv[1]);
    o.y = pack_bf16x2(a[2] * inv * gv[2], a[3] * inv * gv[3]);
    o.z = pack_bf16x2(a[4] * inv * gv[4], a[5] * inv * gv[5]);
    o.w = pack_bf16x2(a[6] * inv * gv[6], a[7] * inv * gv[7]);
    orow[i * 256 + tid] = o;
  }
}

// Launch the row-statistics pre-pass: one CTA per row for K = 4096 and 8192,
// one warp per register-resident row for K = 256 * {1, 2, 4, 8} (two CTAs
// per SM fit in 128 registers per thread), the general two-read kernel
// otherwise.
template <bool ADD>
void launch_rms_prep(const __nv_bfloat16* x, const __nv_bfloat16* z, const float* g, float eps, __nv_bfloat16* a,
                     int M, int K, cudaStream_t st, unsigned* zc = nullptr, int nz = 0) {
  const unsigned grid = static_cast<unsigned>((M + 7) / 8);
  switch (K % 2048 == 0 ? K / 2048 : 0) {
    case 2: rms_prep_cta_kernel<ADD, 2><<<static_cast<unsigned>(M), 256, 0, st>>>(x, z, g, eps, a, zc, nz); return;
    case 4: rms_prep_cta_kernel<ADD, 4><<<static_cast<unsigned>(M), 256, 0, st>>>(x, z, g, eps, a, zc, nz); return;
    default: break;
  }
  // two rows per warp (K <= 1024, where both rows' registers fit) when one
  // row per warp would take more than one wave at two CTAs per SM
  const bool two = grid > 2u * static_cast<unsigned>(num_sms());
  const unsigned grid2 = static_cast<unsigned>((M + 15) / 16);
  switch (K % 256 == 0 ? K / 256 : 0) {
    case 1:
      if (two) return void(rms_prep_reg_kernel<ADD, 1, 2><<<grid2, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
      return void(rms_prep_reg_kernel<ADD, 1, 1><<<grid, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
    case 2:
      if (two) return void(rms_prep_reg_kernel<ADD, 2, 2><<<grid2, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
      return void(rms_prep_reg_kernel<ADD, 2, 1><<<grid, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
    case 4:
      if (two) return void(rms_prep_reg_kernel<ADD, 4, 2><<<grid2, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
      return void(rms_prep_reg_kernel<ADD, 4, 1><<<grid, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz));
    case 8: rms_prep_reg_kernel<ADD, 8, 1><<<grid, 256, 0, st>>>(x, z, g, eps, a, M, zc, nz); return;
    default: rms_prep_kernel<ADD><<<grid, 256, 0, st>>>(x, z, g, eps, a, M, K, zc, nz); return;
  }
}

// Same for N = 2048 * C: each CTA takes two rows, and every thread issues
// all its loads of both rows (and of g) before the first use.
template <int C>
__global__ void __launch_bounds__(256) rownorm2_inplace_kernel(__nv_bfloat16* __restrict__ out,
                                                               const float* __restrict__ rowsq,
                                                               const float* __restrict__ g, float eps, int M) {
  constexpr int N = 2048 * C;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 2;
  const int nrows = row0 + 1 < M ? 2 : 1;
  uint4 v[2][C];
  float4 g0[C], g1[C];
#pragma unroll
  for (int r = 0; r < 2; ++r)
    if (r < nrows) {
#pragma unroll
      for (int c = 0; c < C; ++c)
        v[r][c] = *reinterpret_cast<const uint4*>(out + (row0 + r) * N + c * 2048 + threadIdx.x * 8);
    }
#pragma unroll
  for (int c = 0; c < C; ++c) {
    g0[c] = g ? *reinterpret_cast<const float4*>(g + c * 2048 + threadIdx.x * 8) : make_float4(1.f, 1.f, 1.f, 1.f);
    g1[c] = g ? *reinterpret_cast<const float4*>(g + c * 2048 + threadIdx.x * 8 + 4) : make_float4(1.f, 1.f, 1.f, 1.f);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (r >= nrows) break;
    const float inv = 1.0f / sqrtf(rowsq[row0 + r] / static_cast<float>(N) + eps);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      float y[8];
      unpack_bf16x8(v[r][c], y);
      uint4 o;
      o.x = pack_bf16x2(y[0] * g0[c].x * inv, y[1] * g0[c].y * inv);
      o.y = pack_bf16x2(y[2] * g0[c].z * inv, y[3] * g0[c].w * inv);
      o.z = pack_bf16x2(y[4] * g1[c].x * inv, y[5] * g1[c].y * inv);
      o.w = pack_bf16x2(y[6] * g1[c].z * inv, y[7] * g1[c].w * inv);
      *reinterpret_cast<uint4*>(out + (row0 + r) * N + c * 2048 + threadIdx.x * 8) = o;
    }
  }
}

// out = bf16(out * g / sqrt(rowsq / N + eps)) in place, one CTA per row.
__global__ void __launch_bounds__(256) rownorm_inplace_kernel(__nv_bfloat16* __restrict__ out,
                                                              const float* __restrict__ rowsq,
                                                              const float* __restrict__ g, float eps, int N) {
  const int64_t row = blockIdx.x;
  const float inv = 1.0f / sqrtf(rowsq[row] / static_cast<float>(N) + eps);
  __nv_bfloat16* orow = out + row * N;
  for (int n = threadIdx.x * 8; n < N; n += 256 * 8) {
    float y[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(orow + n), y);
    const float4 g0 = *reinterpret_cast<const float4*>(g + n);
    const float4 g1 = *reinterpret_cast<const float4*>(g + n + 4);
    uint4 o;
    o.x = pack_bf16x2(y[0] * g0.x * inv, y[1] * g0.y * inv);
    o.y = pack_bf16x2(y[2] * g0.z * inv, y[3] * g0.w * inv);
    o.z = pack_bf16x2(y[4] * g1.x * inv, y[5] * g1.y * inv);
    o.w = pack_bf16x2(y[6] * g1.z * inv, y[7] * g1.w * inv);
    *reinterpret_cast<uint4*>(orow + n) = o;
  }
}

// Carves a workspace into consecutive 256-byte aligned pieces.
struct Carve {
  uint8_t* p;
  template <class T>
  T* take(size_t count) {
    T* r = reinterpret_cast<T*>(p);
    p += align256(count * sizeof(T));
    return r;
  }
};

}  // namespace
}  // namespace kda

// Workspace check of an entry point whose arguments are named workspace /
// workspace_bytes: at least ws_need bytes, 16-byte aligned.
#define KDA_F32_COMMON(op, ws_need)                                                                       \
  KDA_CHECK_ARG(workspace && workspace_bytes >= (ws_need), "%s: workspace of %zu bytes required, got %zu", \
                op, static_cast<size_t>(ws_need), workspace_bytes);                                       \
  KDA_CHECK_SUPPORTED(al16(workspace), "%s: workspace must be 16-byte aligned", op)

