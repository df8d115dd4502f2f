// Bandwidth-bound elementwise operators: SiLU, RoPE apply, AdamW step.
//
// All three are HBM-bound streams (bytes per element >> flops per element).
// Design: 128-bit vector loads with L1 no-allocate / L2 256-byte prefetch
// hints, streaming (evict-first) 128-bit stores, one pass over the data (each
// 256-thread CTA owns a contiguous span; every thread issues all of its loads
// before its first store, so enough bytes are outstanding to cover HBM
// latency).  A scalar kernel handles the ragged tail and pointers that are not
// 16-byte aligned.
#include "common.cuh"

namespace kda {
namespace {

constexpr int kThreads = 256;
constexpr int kCtasPerSm = 8;
constexpr int kUnroll = 4;

__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream(float4* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int grid_for(int64_t work_items) {
  int64_t want = (work_items + kThreads - 1) / kThreads;
  int64_t cap = static_cast<int64_t>(num_sms()) * kCtasPerSm;
  if (want < 1) want = 1;
  return static_cast<int>(want < cap ? want : cap);
}

// ------------------------------------------------------------------ SiLU
__device__ __forceinline__ float4 silu4(float4 v) {
  return make_float4(silu_f32(v.x), silu_f32(v.y), silu_f32(v.z), silu_f32(v.w));
}

// One pass over the data: CTA c handles the kUnroll * kThreads vectors
// starting at c * kUnroll * kThreads (all loads issued before any store).
__global__ void __launch_bounds__(kThreads) silu_vec_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                                            int64_t n4) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (kUnroll * kThreads) + threadIdx.x;
  float4 v[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t i = base + u * kThreads;
    if (i < n4) v[u] = ld_stream(x + i);
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t i = base + u * kThreads;
    if (i < n4) st_stream(y + i, silu4(v[u]));
  }
}

__global__ void silu_scalar_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = silu_f32(x[i]);
}

// ------------------------------------------------------------------ RoPE
// x_in (D, S), cos/sin (D/2, S): thread handles 4 columns of one row pair,
// two such groups per thread (one pass, loads before stores).
__global__ void __launch_bounds__(kThreads) rope_vec_kernel(const float4* __restrict__ x,
                                                            const float4* __restrict__ c,
                                                            const float4* __restrict__ s,
                                                            float4* __restrict__ out, int64_t half_rows,
                                                            int64_t s4) {
  const int64_t total = half_rows * s4;
  const int64_t half_off = half_rows * s4;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (2 * kThreads) + threadIdx.x;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int64_t e = base + u * kThreads;
    if (e >= total) break;
    const float4 x0 = ld_stream(x + e);
    const float4 x1 = ld_stream(x + half_off + e);
    const float4 cv = ld_stream(c + e);
    const float4 sv = ld_stream(s + e);
    float4 o0, o1;
    o0.x = x0.x * cv.x - x1.x * sv.x;
    o0.y = x0.y * cv.y - x1.y * sv.y;
    o0.z = x0.z * cv.z - x1.z * sv.z;
    o0.w = x0.w * cv.w - x1.w * sv.w;
    o1.x = x0.x * sv.x + x1.x * cv.x;
    o1.y = x0.y * sv.y + x1.y * cv.y;
    o1.z = x0.z * sv.z + x1.z * cv.z;
    o1.w = x0.w * sv.w + x1.w * cv.w;
    st_stream(out + e, o0);
    st_stream(out + half_off + e, o1);
  }
}

__global__ void rope_scalar_kernel(const float* __restrict__ x, const float* __restrict__ c,
                                   const float* __restrict__ s, float* __restrict__ out, int64_t half_rows,
                                   int64_t cols) {
  const int64_t total = half_rows * cols;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
    const float x0 = x[e], x1 = x[total + e], cv = c[e], sv = s[e];
    out[e] = x0 * cv - x1 * sv;
    out[total + e] = x0 * sv + x1 * cv;
  }
}

// ----------------------------------------------------------------- AdamW
struct AdamOut {
  float th, m, v;
};
__device__ __forceinline__ AdamOut adam1(float th, float g, float m, float v) {
  const float mt = 0.9f * m + 0.1f * g;
  const float vt = 0.999f * v + 0.001f * g * g;
  const float den = sqrtf(vt * 1000.0f) + 1e-8f;
  AdamOut o;
  o.th = (th - 1e-5f * th) - 0.01f * mt / den;
  o.m = mt;
  o.v = vt;
  return o;
}

template <bool kState>
__global__ void __launch_bounds__(kThreads) adamw_vec_kernel(const float4* __restrict__ th,
                                                             const float4* __restrict__ g, float4* m, float4* v,
                                                             float4* __restrict__ out, int64_t n4) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (2 * kThreads) + threadIdx.x;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int64_t i = base + u * kThreads;
    if (i >= n4) break;
    const float4 t4 = ld_stream(th + i), g4 = ld_stream(g + i);
    const float4 m4 = kState ? m[i] : ld_stream(m + i);
    const float4 v4 = kState ? v[i] : ld_stream(v + i);
    const AdamOut a = adam1(t4.x, g4.x, m4.x, v4.x);
    const AdamOut b = adam1(t4.y, g4.y, m4.y, v4.y);
    const AdamOut c = adam1(t4.z, g4.z, m4.z, v4.z);
    const AdamOut d = adam1(t4.w, g4.w, m4.w, v4.w);
    st_stream(out + i, make_float4(a.th, b.th, c.th, d.th));
    if (kState) {
      st_stream(m + i, make_float4(a.m, b.m, c.m, d.m));
      st_stream(v + i, make_float4(a.v, b.v, c.v, d.v));
    }
  }
}

__global__ void adamw_scalar_kernel(const float* __restrict__ th, const float* __restrict__ g, float* m,
                                    float* v, float* __restrict__ out, int64_t n, int state) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const AdamOut a = adam1(th[i], g[i], m[i], v[i]);
    out[i] = a.th;
    if (state) {
      m[i] = a.m;
      v[i] = a.v;
    }
  }
}

}  // namespace
}  // namespace kda

using namespace kda;

extern "C" kda_status kda_silu_f32(const float* x, float* y, int64_t n, void* stream) {
  KDA_CHECK_ARG(n >= 0, "silu: n = %lld < 0", (long long)n);
  if (n == 0) return KDA_OK;
  KDA_CHECK_ARG(x && y, "silu: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (aligned16(x) && aligned16(y)) {
    const int64_t n4 = n / 4;
    if (n4 > 0)
      silu_vec_kernel<<<static_cast<unsigned>((n4 + kUnroll * kThreads - 1) / (kUnroll * kThreads)), kThreads, 0,
                        st>>>(reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n4);
    const int64_t tail = n - n4 * 4;
    if (tail) silu_scalar_kernel<<<1, 32, 0, st>>>(x + n4 * 4, y + n4 * 4, tail);
  } else {
    silu_scalar_kernel<<<grid_for(n), kThreads, 0, st>>>(x, y, n);
  }
  return launch_status("silu");
}

extern "C" kda_status kda_rope_single_freq_apply_f32(const float* x_in, const float* cos, const float* sin,
                                                     float* out, int64_t d_head, int64_t s, void* stream) {
  KDA_CHECK_ARG(d_head >= 2 && d_head % 2 == 0, "rope: d_head = %lld must be even and >= 2", (long long)d_head);
  KDA_CHECK_ARG(s >= 0, "rope: s = %lld < 0", (long long)s);
  if (s == 0) return KDA_OK;
  KDA_CHECK_ARG(x_in && cos && sin && out, "rope: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t half = d_head / 2;
  if (s % 4 == 0 && aligned16(x_in) && aligned16(cos) && aligned16(sin) && aligned16(out)) {
    const int64_t s4 = s / 4;
    rope_vec_kernel<<<static_cast<unsigned>((half * s4 + 2 * kThreads - 1) / (2 * kThreads)), kThreads, 0, st>>>(
        reinterpret_cast<const float4*>(x_in), reinterpret_cast<const float4*>(cos),
        reinterpret_cast<const float4*>(sin), reinterpret_cast<float4*>(out), half, s4);
  } else {
    rope_scalar_kernel<<<grid_for(half * s), kThreads, 0, st>>>(x_in, cos, sin, out, half, s);
  }
  return launch_status("rope_single_freq_apply");
}

extern "C" kda_status kda_adamw_f32(const float* theta, const float* g, float* m, float* v, float* theta_out,
                                    int64_t n, int update_state, void* stream) {
  KDA_CHECK_ARG(n >= 0, "adamw: n = %lld < 0", (long long)n);
  if (n == 0) return KDA_OK;
  KDA_CHECK_ARG(theta && g && m && v && theta_out, "adamw: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = aligned16(theta) && aligned16(g) && aligned16(m) && aligned16(v) && aligned16(theta_out);
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      auto* t4 = reinterpret_cast<const float4*>(theta);
      auto* g4 = reinterpret_cast<const float4*>(g);
      auto* m4 = reinterpret_cast<float4*>(m);
      auto* v4 = reinterpret_cast<float4*>(v);
      auto* o4 = reinterpret_cast<float4*>(theta_out);
      const unsigned grid = static_cast<unsigned>((n4 + 2 * kThreads - 1) / (2 * kThreads));
      if (update_state)
        adamw_vec_kernel<true><<<grid, kThreads, 0, st>>>(t4, g4, m4, v4, o4, n4);
      else
        adamw_vec_kernel<false><<<grid, kThreads, 0, st>>>(t4, g4, m4, v4, o4, n4);
    }
    done = n4 * 4;
  }
  if (done < n)
    adamw_scalar_kernel<<<grid_for(n - done), kThreads, 0, st>>>(theta + done, g + done, m + done, v + done,
                                                                 theta_out + done, n - done, update_state);
  return launch_status("adamw");
}
