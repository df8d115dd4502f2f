// Mamba selective scan (d_state 16, fp32 state).
//
//   h_t = exp(dt_t * A) * h_{t-1} + dt_t * B_t * x_t ;  y_t = C_t . h_t + D x_t
//
// One thread owns one (batch, channel) and keeps its 16 states in registers
// as float2 pairs for the packed f32x2 FMA pipe; the recurrence runs
// sequentially over time with one ex2.approx per (t, channel, state) (A is
// pre-scaled by log2 e) -- the MUFU pipe, not HBM, bounds the north-star size.
// Channels-last inputs (the north-star layout) stream dt / x / B_t / C_t tiles
// through a cp.async shared-memory ring (scan_cl_kernel); other layouts use a
// register-prefetch kernel (scan_kernel) that stages B_t / C_t in shared
// memory and reads dt / x per thread.
//
// When batch * channels is too small to fill the GPU (the reference's 2-D
// case: 256 channels; channels-last tensors with fewer than 4096 channels),
// time is split into chunks scanned in parallel:
//   pass 1: per chunk, the end state from a zero start and sum(dt);
//   pass 2: per (b, d, n), carry states across chunks sequentially
//           (the chunk's total decay is exp(A * sum(dt)));
//   pass 3: per chunk, the scan again from its carried-in state, writing y.
// Chunk summaries live in the caller's workspace.
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace kda {
namespace {

constexpr int kThreads = 128;
constexpr int kTT = 16;  // time steps per tile (one tile of lookahead is prefetched)
constexpr int kState = 16;
constexpr float kLog2e = 1.4426950408889634f;

struct ScanParams {
  const float* dt;
  const void* x;
  const float* A;  // (D, 16)
  const float* Bm;
  const float* Cm;
  const float* Dv;  // (D,) or null
  void* y;
  int64_t batch, L, D;
  int64_t ld_b, ld_t, ld_d;
  int64_t bc_b, bc_t, bc_n;
  int64_t chunk_len;
  int nchunks;
  float* hsum;   // [nchunks][batch][D][16]: pass1 end states / pass2 carried-in states
  float* dtsum;  // [nchunks][batch][D]
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool XBF16>
__device__ __forceinline__ float load_x(const void* x, int64_t off) {
  if (XBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[off]);
  return reinterpret_cast<const float*>(x)[off];
}

// MODE 0: scan from the carried-in state (zero if nchunks == 1) and write y.
// MODE 1: chunk-local scan from zero; write the end state and sum(dt).
template <int MODE, bool XBF16, bool YBF16>
__global__ void __launch_bounds__(kThreads) scan_kernel(const ScanParams p) {
  // B_t / C_t tiles, double buffered: tile i+1 is written while tile i is read
  __shared__ __align__(16) float sB[2][kTT][kState];
  __shared__ __align__(16) float sC[2][kTT][kState];
  const int64_t d = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t b = blockIdx.y;
  const int chunk = blockIdx.z;
  const bool active = d < p.D;
  const int64_t t_begin = chunk * p.chunk_len;
  int64_t t_end = t_begin + p.chunk_len;
  if (t_end > p.L) t_end = p.L;
  const int ntiles = static_cast<int>((t_end - t_begin + kTT - 1) / kTT);

  // states and A (pre-scaled by log2 e) as float2 pairs for the packed f32x2 pipe
  float2 a2[kState / 2], h[kState / 2];
#pragma unroll
  for (int k = 0; k < kState / 2; ++k) {
    a2[k] = active ? make_float2(p.A[d * kState + 2 * k] * kLog2e, p.A[d * kState + 2 * k + 1] * kLog2e)
                   : make_float2(0.f, 0.f);
    h[k] = make_float2(0.f, 0.f);
  }
  if (MODE == 0 && p.nchunks > 1 && active) {
    const float* hs = p.hsum + ((static_cast<int64_t>(chunk) * p.batch + b) * p.D + d) * kState;
#pragma unroll
    for (int k = 0; k < kState / 2; ++k) h[k] = make_float2(hs[2 * k], hs[2 * k + 1]);
  }
  const float dskip = (MODE == 0 && p.Dv && active) ? p.Dv[d] : 0.f;
  float dts = 0.f;
  const int64_t base = b * p.ld_b + d * p.ld_d;
  const float* Bb = p.Bm + b * p.bc_b;
  const float* Cb = p.Cm + b * p.bc_b;

  // per-thread share of one B/C tile: kTT*kState / kThreads = 4 values each
  constexpr int kPer = kTT * kState / kThreads;
  float nb[kPer], nc[kPer];
  float dtv[kTT], xv[kTT], ndt[kTT], nx[kTT];
  auto load_tile = [&](int64_t t0, float (&dd)[kTT], float (&xx)[kTT], float (&bb)[kPer], float (&cc)[kPer]) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = threadIdx.x + i * kThreads;
      const int j = e / kState, n = e % kState;
      const bool in = t0 + j < t_end;
      const int64_t off = (t0 + j) * p.bc_t + n * p.bc_n;
      bb[i] = in ? __ldg(Bb + off) : 0.f;
      cc[i] = (MODE == 0 && in) ? __ldg(Cb + off) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kTT; ++j) {
      const bool in = active && (t0 + j < t_end);
      const int64_t off = base + (t0 + j) * p.ld_t;
      dd[j] = in ? __ldg(p.dt + off) : 0.f;
      xx[j] = in ? load_x<XBF16>(p.x, off) : 0.f;
    }
  };
  auto store_bc = [&](int buf, const float (&bb)[kPer], const float (&cc)[kPer]) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = threadIdx.x + i * kThreads;
      sB[buf][e / kState][e % kState] = bb[i];
      if (MODE == 0) sC[buf][e / kState][e % kState] = cc[i];
    }
  };

  load_tile(t_begin, dtv, xv, nb, nc);
  store_bc(0, nb, nc);
  __syncthreads();
  for (int it = 0; it < ntiles; ++it) {
    const int64_t t0 = t_begin + static_cast<int64_t>(it) * kTT;
    const int buf = it & 1;
    const bool more = it + 1 < ntiles;
    if (more) load_tile(t0 + kTT, ndt, nx, nb, nc);  // in flight during this tile's steps
    const int steps = static_cast<int>((t_end - t0) < kTT ? (t_end - t0) : kTT);
    // Steps past the tile's end see dt = x = 0: exp(0) = 1 and dt*B*x = 0
    // leave the state unchanged, so every tile runs all kTT steps (fully
    // unrolled, register-indexed) and only the stores are predicated.
#pragma unroll
    for (int j = 0; j < kTT; ++j) {
      const float dt = dtv[j];
      const float2 dt2 = make_float2(dt, dt);
      const float dtx = dt * xv[j];
      const float2 dtx2 = make_float2(dtx, dtx);
      const float4* b4 = reinterpret_cast<const float4*>(&sB[buf][j][0]);
      const float4* c4 = reinterpret_cast<const float4*>(&sC[buf][j][0]);
      float2 y2a = make_float2(0.f, 0.f), y2b = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kState / 4; ++q) {
        const float4 bq = b4[q];
        const float2 arg0 = __fmul2_rn(dt2, a2[2 * q]);
        const float2 arg1 = __fmul2_rn(dt2, a2[2 * q + 1]);
        const float2 e0 = make_float2(ex2(arg0.x), ex2(arg0.y));
        const float2 e1 = make_float2(ex2(arg1.x), ex2(arg1.y));
        h[2 * q] = __ffma2_rn(e0, h[2 * q], __fmul2_rn(dtx2, make_float2(bq.x, bq.y)));
        h[2 * q + 1] = __ffma2_rn(e1, h[2 * q + 1], __fmul2_rn(dtx2, make_float2(bq.z, bq.w)));
        if (MODE == 0) {
          const float4 cq = c4[q];
          y2a = __ffma2_rn(make_float2(cq.x, cq.y), h[2 * q], y2a);
          y2b = __ffma2_rn(make_float2(cq.z, cq.w), h[2 * q + 1], y2b);
        }
      }
      if (MODE == 0) {
        const float y = fmaf(dskip, xv[j], (y2a.x + y2a.y) + (y2b.x + y2b.y));
        const int64_t off = base + (t0 + j) * p.ld_t;
        if (active && j < steps) {
          if (YBF16)
            reinterpret_cast<__nv_bfloat16*>(p.y)[off] = __float2bfloat16_rn(y);
          else
            reinterpret_cast<float*>(p.y)[off] = y;
        }
      } else {
        dts += dt;
      }
    }
    if (more) {
      store_bc(buf ^ 1, nb, nc);
#pragma unroll
      for (int j = 0; j < kTT; ++j) {
        dtv[j] = ndt[j];
        xv[j] = nx[j];
      }
    }
    __syncthreads();
  }
  if (MODE == 1 && active) {
    const int64_t idx = (static_cast<int64_t>(chunk) * p.batch + b) * p.D + d;
    float* hs = p.hsum + idx * kState;
#pragma unroll
    for (int k = 0; k < kState / 2; ++k) {
      hs[2 * k] = h[k].x;
      hs[2 * k + 1] = h[k].y;
    }
    p.dtsum[idx] = dts;
  }
}

// ---------------------------------------------------------------------------
// Channels-last scan (the north-star layout, d_inner contiguous): dt / x / B /
// C tiles of kTTA steps stream through a kStagesA-deep cp.async ring in shared
// memory (16-byte copies, zero-filled past the sequence end), so global-load
// latency never stalls the dependent steps.  LPC lanes share a channel's 16
// states (16 / LPC each, as float2 pairs) and combine their partial C . h
// sums by shuffles; CH channels per CTA.  The plan picks by channel count
// (batch x d_inner): 1 lane and 64 channels per CTA from 32768 channels (all
// 16 exponentials of a step independent in one thread), 2 lanes and 32
// channels from 16384, 4 lanes and 32 channels from 4096 (more warps where
// the channels alone leave the SMs nearly empty).  Measured at L4096 D4096
// (ms): batch 8: 0.854 / 0.90 / 1.06 for 1 / 2 / 4 lanes; batch 4: 0.645 /
// 0.593 / 0.661; batch 2: 0.633 / 0.500 / 0.475 (the chunked three-pass scan:
// 0.937); batch 1: 0.633 / 0.490 / 0.412 (chunked: 0.478).  Also measured at
// batch 8 and kept out: the next step's exponentials issued ahead 0.88, MUFU /
// FMA interleaved per state pair 0.89, unpacked scalar math 0.93, 2 / 4 / 8 of
// the 16 exponentials on the FMA pipe 0.93 / 0.98 / 1.07; strides read from
// the parameters rather than derived (below) 0.92.
constexpr int kTTA = 32;      // steps per tile
constexpr int kStagesA = 3;   // ring depth

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int CH, bool XBF16>
struct TileA {
  float dt[kTTA][CH];
  typename std::conditional<XBF16, __nv_bfloat16, float>::type x[kTTA][CH];
  float B[kTTA][kState];
  float C[kTTA][kState];
};

template <int LPC, int CH, bool XBF16, bool YBF16>
__global__ void __launch_bounds__(CH * LPC) scan_cl_kernel(const ScanParams p) {
  constexpr int kThr = CH * LPC;
  constexpr int kNS = kState / LPC;  // states per lane
  constexpr int kH = kNS / 2;        // float2 pairs per lane
  static_assert(kH % 2 == 0, "two pairs per B / C float4");
  extern __shared__ __align__(16) uint8_t smem_a[];
  auto* ring = reinterpret_cast<TileA<CH, XBF16>*>(smem_a);
  const int tid = threadIdx.x;
  const int ch = tid / LPC;
  const int sub = tid % LPC;  // states [kNS sub, kNS sub + kNS)
  const int64_t d0 = static_cast<int64_t>(blockIdx.x) * CH;
  const int64_t d = d0 + ch;
  const int64_t b = blockIdx.y;
  const bool active = d < p.D;
  const int64_t L = p.L;
  const int ntiles = static_cast<int>((L + kTTA - 1) / kTTA);
  // dense channels-last strides, derived here rather than read from p (the
  // derived form compiles to a faster schedule: 0.858 vs 0.92 ms)
  const int64_t ld_t = p.D;
  const int64_t ld_b = L * p.D;
  const float* dtb = p.dt + b * ld_b;
  const uint8_t* xb = reinterpret_cast<const uint8_t*>(p.x) + b * ld_b * (XBF16 ? 2 : 4);
  const float* Bb = p.Bm + b * L * kState;
  const float* Cb = p.Cm + b * L * kState;

  auto issue = [&](int tile) {
    TileA<CH, XBF16>& st = ring[tile % kStagesA];
    const int64_t t0 = static_cast<int64_t>(tile) * kTTA;
    constexpr int kDtChunks = CH * 4 / 16;
    for (int i = tid; i < kTTA * kDtChunks; i += kThr) {
      const int j = i / kDtChunks, c = i % kDtChunks;
      const int64_t t = t0 + j;
      const int64_t col = d0 + c * 4;
      const bool v = t < L && col < p.D;
      cp_async16(&st.dt[j][c * 4], v ? dtb + t * ld_t + col : dtb, v);
    }
    constexpr int kEl = XBF16 ? 2 : 4;
    constexpr int kXChunks = CH * kEl / 16;
    constexpr int kPer = 16 / kEl;
    for (int i = tid; i < kTTA * kXChunks; i += kThr) {
      const int j = i / kXChunks, c = i % kXChunks;
      const int64_t t = t0 + j;
      const int64_t col = d0 + c * kPer;
      const bool v = t < L && col < p.D;
      cp_async16(&st.x[j][c * kPer], v ? xb + (t * ld_t + col) * kEl : xb, v);
    }
    for (int i = tid; i < kTTA * 4; i += kThr) {
      const int j = i / 4, c = i % 4;
      const int64_t t = t0 + j;
      const bool v = t < L;
      cp_async16(&st.B[j][c * 4], v ? Bb + t * kState + c * 4 : Bb, v);
      cp_async16(&st.C[j][c * 4], v ? Cb + t * kState + c * 4 : Cb, v);
    }
  };

  float2 a2[kH], h[kH];
#pragma unroll
  for (int k = 0; k < kH; ++k) {
    const int n = sub * kNS + 2 * k;
    a2[k] = active ? make_float2(p.A[d * kState + n] * kLog2e, p.A[d * kState + n + 1] * kLog2e)
                   : make_float2(0.f, 0.f);
    h[k] = make_float2(0.f, 0.f);
  }
  const float dskip = (p.Dv && active && sub == 0) ? p.Dv[d] : 0.f;

#pragma unroll
  for (int s = 0; s < kStagesA - 1; ++s) {
    if (s < ntiles) issue(s);
    cp_async_commit();
  }
  for (int it = 0; it < ntiles; ++it) {
    if (it + kStagesA - 1 < ntiles) issue(it + kStagesA - 1);
    cp_async_commit();
    cp_async_wait<kStagesA - 1>();
    __syncthreads();
    const TileA<CH, XBF16>& st = ring[it % kStagesA];
    const int64_t t0 = static_cast<int64_t>(it) * kTTA;
#pragma unroll(LPC == 1 ? 2 : 4)
    for (int j = 0; j < kTTA; ++j) {
      const float dt = st.dt[j][ch];
      float xv;
      if (XBF16)
        xv = __bfloat162float(reinterpret_cast<const __nv_bfloat16&>(st.x[j][ch]));
      else
        xv = static_cast<float>(st.x[j][ch]);
      const float2 dt2 = make_float2(dt, dt);
      const float dtx = dt * xv;
      const float2 dtx2 = make_float2(dtx, dtx);
      const float4* b4 = reinterpret_cast<const float4*>(&st.B[j][sub * kNS]);
      const float4* c4 = reinterpret_cast<const float4*>(&st.C[j][sub * kNS]);
      float2 y2a = make_float2(0.f, 0.f), y2b = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < kH / 2; ++q) {
        const float4 bq = b4[q];
        const float4 cq = c4[q];
        const float2 arg0 = __fmul2_rn(dt2, a2[2 * q]);
        const float2 arg1 = __fmul2_rn(dt2, a2[2 * q + 1]);
        const float2 e0 = make_float2(ex2(arg0.x), ex2(arg0.y));
        const float2 e1 = make_float2(ex2(arg1.x), ex2(arg1.y));
        h[2 * q] = __ffma2_rn(e0, h[2 * q], __fmul2_rn(dtx2, make_float2(bq.x, bq.y)));
        h[2 * q + 1] = __ffma2_rn(e1, h[2 * q + 1], __fmul2_rn(dtx2, make_float2(bq.z, bq.w)));
        y2a = __ffma2_rn(make_float2(cq.x, cq.y), h[2 * q], y2a);
        y2b = __ffma2_rn(make_float2(cq.z, cq.w), h[2 * q + 1], y2b);
      }
      float y = (y2a.x + y2a.y) + (y2b.x + y2b.y);
      if (LPC >= 2) y += __shfl_xor_sync(0xffffffffu, y, 1);
      if (LPC >= 4) y += __shfl_xor_sync(0xffffffffu, y, 2);
      y = fmaf(dskip, xv, y);
      const int64_t t = t0 + j;
      if (active && sub == 0 && t < L) {
        const int64_t off = b * ld_b + t * ld_t + d;
        if (YBF16)
          reinterpret_cast<__nv_bfloat16*>(p.y)[off] = __float2bfloat16_rn(y);
        else
          reinterpret_cast<float*>(p.y)[off] = y;
      }
    }
    __syncthreads();  // stage it % kStagesA is refilled by the next iteration
  }
}

// Carry states across chunks: in place, hsum[c] becomes the state entering c.
__global__ void __launch_bounds__(256) carry_kernel(const ScanParams p) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, d, n)
  const int64_t total = p.batch * p.D * kState;
  if (i >= total) return;
  const int64_t n = i % kState;
  const int64_t bd = i / kState;
  const int64_t d = bd % p.D;
  const float a2 = p.A[d * kState + n] * kLog2e;
  float h = 0.f;
  for (int c = 0; c < p.nchunks; ++c) {
    const int64_t idx = static_cast<int64_t>(c) * p.batch * p.D + bd;
    const float hl = p.hsum[idx * kState + n];
    const float decay = ex2(a2 * p.dtsum[idx]);
    p.hsum[idx * kState + n] = h;
    h = fmaf(decay, h, hl);
  }
}

int choose_chunks(int64_t batch, int64_t L, int64_t D) {
  const int64_t chans = batch * D;
  if (chans >= 16384 || L < 256) return 1;
  int64_t want = (32768 + chans - 1) / chans;
  int64_t cap = L / 128;
  if (want > cap) want = cap;
  return static_cast<int>(want < 1 ? 1 : want);
}

template <int MODE>
void launch_scan(const ScanParams& p, bool xb, bool yb, dim3 grid, cudaStream_t st) {
  if (xb) {
    if (yb) scan_kernel<MODE, true, true><<<grid, kThreads, 0, st>>>(p);
    else scan_kernel<MODE, true, false><<<grid, kThreads, 0, st>>>(p);
  } else {
    if (yb) scan_kernel<MODE, false, true><<<grid, kThreads, 0, st>>>(p);
    else scan_kernel<MODE, false, false><<<grid, kThreads, 0, st>>>(p);
  }
}

// The cp.async path needs dense channels-last tensors (dt / x (B, L, D), B / C
// (B, L, 16)) whose starts are 16-byte aligned.
bool cl_layout_ok(const ScanParams& p, bool xbf16) {
  (void)xbf16;
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return p.ld_d == 1 && p.ld_t == p.D && p.ld_b == p.L * p.D && p.bc_n == 1 && p.bc_t == kState &&
         p.bc_b == p.L * kState && p.D % 8 == 0 && al(p.dt) && al(p.x) && al(p.Bm) && al(p.Cm);
}

// One instantiation per kernel variant, so each variant's shared-memory
// opt-in is recorded separately.
template <int LPC, int CH, bool XB, bool YB>
kda_status launch_scan_cl_t(const ScanParams& p, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>((p.D + CH - 1) / CH), static_cast<unsigned>(p.batch), 1);
  constexpr size_t smem = kStagesA * sizeof(TileA<CH, XB>);
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(scan_cl_kernel<LPC, CH, XB, YB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return launch_status("mamba_scan: cudaFuncSetAttribute");
    attr_set[dev].store(true, std::memory_order_release);
  }
  scan_cl_kernel<LPC, CH, XB, YB><<<grid, CH * LPC, smem, st>>>(p);
  return launch_status("mamba_scan");
}

template <int LPC, int CH>
kda_status launch_scan_cl_lc(const ScanParams& p, bool xb, bool yb, cudaStream_t st) {
  if (xb) return yb ? launch_scan_cl_t<LPC, CH, true, true>(p, st) : launch_scan_cl_t<LPC, CH, true, false>(p, st);
  return yb ? launch_scan_cl_t<LPC, CH, false, true>(p, st) : launch_scan_cl_t<LPC, CH, false, false>(p, st);
}

// lanes per channel of the channels-last kernel for this many channels
// (batch x d_inner); 0 = too few channels: the chunked scan instead
int cl_lanes(int64_t chans) { return chans >= 32768 ? 1 : chans >= 16384 ? 2 : chans >= 4096 ? 4 : 0; }

kda_status launch_scan_cl(const ScanParams& p, bool xb, bool yb, cudaStream_t st) {
  switch (cl_lanes(p.batch * p.D)) {
    case 1: return launch_scan_cl_lc<1, 64>(p, xb, yb, st);
    case 2: return launch_scan_cl_lc<2, 32>(p, xb, yb, st);
    default: return launch_scan_cl_lc<4, 32>(p, xb, yb, st);
  }
}

}  // namespace
}  // namespace kda

using namespace kda;

extern "C" size_t kda_mamba_scan_workspace_size(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state) {
  if (batch <= 0 || seqlen <= 0 || d_inner <= 0 || d_state != kState) return 0;
  const int nc = choose_chunks(batch, seqlen, d_inner);
  if (nc <= 1) return 0;
  const size_t per = static_cast<size_t>(nc) * batch * d_inner;
  return ((per * kState * 4 + 255) & ~size_t(255)) + ((per * 4 + 255) & ~size_t(255));
}

extern "C" kda_status kda_mamba_scan(const void* delta, const void* u, const float* a, const float* b, const float* c,
                                     const float* D, void* y, int64_t batch, int64_t seqlen, int64_t d_inner,
                                     int64_t d_state, int64_t ld_b, int64_t ld_t, int64_t ld_d, int64_t bc_ld_b,
                                     int64_t bc_ld_t, int64_t bc_ld_n, int u_bf16, int y_bf16, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  KDA_CHECK_ARG(batch > 0 && batch < 65536 && seqlen > 0 && d_inner > 0,
                "mamba: bad sizes batch=%lld seqlen=%lld d_inner=%lld", (long long)batch, (long long)seqlen,
                (long long)d_inner);
  KDA_CHECK_SUPPORTED(d_state == kState, "mamba: d_state must be 16, got %lld", (long long)d_state);
  KDA_CHECK_ARG(delta && u && a && b && c && y, "mamba: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScanParams p{};
  p.dt = static_cast<const float*>(delta);
  p.x = u;
  p.A = a;
  p.Bm = b;
  p.Cm = c;
  p.Dv = D;
  p.y = y;
  p.batch = batch;
  p.L = seqlen;
  p.D = d_inner;
  p.ld_b = ld_b;
  p.ld_t = ld_t;
  p.ld_d = ld_d;
  p.bc_b = bc_ld_b;
  p.bc_t = bc_ld_t;
  p.bc_n = bc_ld_n;
  // dense channels-last with enough channels: one pass, no workspace
  if (cl_layout_ok(p, u_bf16 != 0) && cl_lanes(batch * d_inner) > 0) {
    p.nchunks = 1;
    p.chunk_len = seqlen;
    return launch_scan_cl(p, u_bf16 != 0, y_bf16 != 0, st);
  }
  const size_t need = kda_mamba_scan_workspace_size(batch, seqlen, d_inner, d_state);
  KDA_CHECK_ARG(need == 0 || (workspace && workspace_bytes >= need),
                "mamba: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  p.nchunks = choose_chunks(batch, seqlen, d_inner);
  p.chunk_len = (seqlen + p.nchunks - 1) / p.nchunks;
  p.chunk_len = (p.chunk_len + kTT - 1) / kTT * kTT;
  p.nchunks = static_cast<int>((seqlen + p.chunk_len - 1) / p.chunk_len);
  const size_t per = static_cast<size_t>(p.nchunks) * batch * d_inner;
  if (p.nchunks > 1) {
    p.hsum = static_cast<float*>(workspace);
    p.dtsum = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((per * kState * 4 + 255) & ~size_t(255)));
  }
  if (p.nchunks == 1 && cl_layout_ok(p, u_bf16 != 0)) return launch_scan_cl(p, u_bf16 != 0, y_bf16 != 0, st);
  const dim3 grid(static_cast<unsigned>((d_inner + kThreads - 1) / kThreads), static_cast<unsigned>(batch),
                  static_cast<unsigned>(p.nchunks));
  if (p.nchunks > 1) {
    launch_scan<1>(p, u_bf16 != 0, y_bf16 != 0, grid, st);
    const int64_t total = batch * d_inner * kState;
    carry_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(p);
  }
  launch_scan<0>(p, u_bf16 != 0, y_bf16 != 0, grid, st);
  return launch_status("mamba_scan");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the chunked scan.
//
// Some callers cannot hand the library a workspace: a host binding (cgo, JNI,
// a plugin) that receives only the input and output buffers from its
// framework and has no way to ask that framework's allocator for more, or a
// caller that must not call cudaMalloc because it can synchronise the device
// and stall work already queued on other streams.  For them the chunk
// summaries live in one fixed array in device memory, created when the
// library is loaded on a GPU and kept until the process exits.
// ---------------------------------------------------------------------------
namespace kda {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB per device
static __device__ __align__(256) float g_mamba_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the scratch array for the current device.  In host code
// `g_mamba_noalloc_scratch` names a host-side stand-in, never the device
// memory, so the address must come from cudaGetSymbolAddress -- once per
// device, with that device current.
kda_status noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* cache[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("mamba_noalloc: cudaGetDevice failed (%s)", cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  std::lock_guard<std::mutex> g(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_mamba_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("mamba_noalloc: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
      return KDA_CUDA_ERROR;
    }
    cache[dev] = static_cast<float*>(p);
  }
  *out = cache[dev];
  return KDA_OK;
}

}  // namespace
}  // namespace kda

extern "C" kda_status kda_mamba_scan_noalloc(const void* delta, const void* u, const float* a, const float* b,
                                             const float* c, const float* D, void* y, int64_t batch, int64_t seqlen,
                                             int64_t d_inner, int64_t d_state, int64_t ld_b, int64_t ld_t,
                                             int64_t ld_d, int64_t bc_ld_b, int64_t bc_ld_t, int64_t bc_ld_n,
                                             int u_bf16, int y_bf16, void* stream) {
  KDA_CHECK_ARG(batch > 0 && batch < 65536 && seqlen > 0 && d_inner > 0,
                "mamba_noalloc: bad sizes batch=%lld seqlen=%lld d_inner=%lld", (long long)batch,
                (long long)seqlen, (long long)d_inner);
  KDA_CHECK_SUPPORTED(d_state == kState, "mamba_noalloc: d_state must be 16, got %lld", (long long)d_state);
  KDA_CHECK_ARG(delta && u && a && b && c && y, "mamba_noalloc: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScanParams p{};
  p.dt = static_cast<const float*>(delta);
  p.x = u;
  p.A = a;
  p.Bm = b;
  p.Cm = c;
  p.Dv = D;
  p.y = y;
  p.batch = batch;
  p.L = seqlen;
  p.D = d_inner;
  p.ld_b = ld_b;
  p.ld_t = ld_t;
  p.ld_d = ld_d;
  p.bc_b = bc_ld_b;
  p.bc_t = bc_ld_t;
  p.bc_n = bc_ld_n;
  // the same one-pass channels-last kernel as kda_mamba_scan: no scratch
  if (cl_layout_ok(p, u_bf16 != 0) && cl_lanes(batch * d_inner) > 0) {
    p.nchunks = 1;
    p.chunk_len = seqlen;
    return launch_scan_cl(p, u_bf16 != 0, y_bf16 != 0, st);
  }
  const size_t need = kda_mamba_scan_workspace_size(batch, seqlen, d_inner, d_state);
  KDA_CHECK_SUPPORTED(need <= kNoAllocScratchBytes,
                      "mamba_noalloc: this shape needs %zu bytes of scratch but the built-in array holds %zu; "
                      "call kda_mamba_scan with a workspace instead",
                      need, kNoAllocScratchBytes);
  float* scratch = nullptr;
  const kda_status ss = noalloc_scratch(&scratch);
  if (ss != KDA_OK) return ss;
  p.nchunks = choose_chunks(batch, seqlen, d_inner);
  p.chunk_len = (seqlen + p.nchunks - 1) / p.nchunks;
  p.chunk_len = (p.chunk_len + kTT - 1) / kTT * kTT;
  p.nchunks = static_cast<int>((seqlen + p.chunk_len - 1) / p.chunk_len);
  const size_t per = static_cast<size_t>(p.nchunks) * batch * d_inner;
  if (p.nchunks > 1) {
    // pass 1 writes every summary before pass 2 reads it: nothing needs clearing
    p.hsum = scratch;
    p.dtsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) +
                                       ((per * kState * 4 + 255) & ~size_t(255)));
  }
  if (p.nchunks == 1 && cl_layout_ok(p, u_bf16 != 0)) return launch_scan_cl(p, u_bf16 != 0, y_bf16 != 0, st);
  const dim3 grid(static_cast<unsigned>((d_inner + kThreads - 1) / kThreads), static_cast<unsigned>(batch),
                  static_cast<unsigned>(p.nchunks));
  if (p.nchunks > 1) {
    launch_scan<1>(p, u_bf16 != 0, y_bf16 != 0, grid, st);
    const int64_t total = batch * d_inner * kState;
    carry_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(p);
  }
  launch_scan<0>(p, u_bf16 != 0, y_bf16 != 0, grid, st);
  return launch_status("mamba_scan_noalloc");
}
