// Backward kernels for training callers of the contractions and attention:
// rmsnorm_matmul, swiglu and gqa_full gradients on the tcgen05 engine.
#include "gemm.cuh"

KDA_DEFINE_ERROR_WORD(gemm_bwd)
static unsigned* gemm_err_word() { return kda_err_ptr_gemm_bwd(); }

#include "gemm_host.cuh"

using namespace kda;

// --------------------------------------------------- rmsnorm_matmul backward
// Gradients of out = a @ w, a = x * r * g, r = 1 / sqrt(mean_k x^2 + eps):
//   dA = dy @ w^T (fp32)        dw = a^T @ dy          dg_k = sum_m dA_mk xn_mk
//   dx = r (dA g - xn c),  xn = x r,  c = mean_k(dA_k g_k xn_k)
// Both products run on the tcgen05 engine (w transposed once into the
// workspace so dy @ w^T is an MN-major-B GEMM; a^T @ dy is the
// transpose_matmul kernel on the recomputed bf16 a, the forward's operand);
// dx comes from one row kernel, dg from a column kernel over row chunks and
// a fixed-order sum of the chunks (deterministic, no atomics).
namespace kda {
namespace {
constexpr int kDgRows = 32;  // rows per column-partial of dg

// One warp per row: r from x, c from dA, g and xn, then dx (bf16); r is
// kept for the dg kernel.  K % 8 == 0.
__global__ void __launch_bounds__(256) rms_backward_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const float* __restrict__ dA,
                                                                const float* __restrict__ g, float eps,
                                                                __nv_bfloat16* __restrict__ dx,
                                                                float* __restrict__ r_out, int64_t M, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * K;
  const float* dr = dA + row * K;
  float ss = 0.f, sd = 0.f;  // sum x^2, sum dA g x
  for (int k = lane * 8; k < K; k += 256) {
    float a[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(xr + k), a);
    const float4 d0 = *reinterpret_cast<const float4*>(dr + k), d1 = *reinterpret_cast<const float4*>(dr + k + 4);
    float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    if (g) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + k), g1 = *reinterpret_cast<const float4*>(g + k + 4);
      d[0] *= g0.x, d[1] *= g0.y, d[2] *= g0.z, d[3] *= g0.w, d[4] *= g1.x, d[5] *= g1.y, d[6] *= g1.z, d[7] *= g1.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(a[i], a[i], ss);
      sd = fmaf(d[i], a[i], sd);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    sd += __shfl_xor_sync(0xffffffffu, sd, o);
  }
  const float r = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
  const float c = sd * r / static_cast<float>(K);  // mean_k(dA g xn)
  if (lane == 0) r_out[row] = r;
  for (int k = lane * 8; k < K; k += 256) {
    float a[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(xr + k), a);
    const float4 d0 = *reinterpret_cast<const float4*>(dr + k), d1 = *reinterpret_cast<const float4*>(dr + k + 4);
    float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    if (g) {
      const float4 g0 = *reinterpret_cast<const float4*>(g + k), g1 = *reinterpret_cast<const float4*>(g + k + 4);
      d[0] *= g0.x, d[1] *= g0.y, d[2] *= g0.z, d[3] *= g0.w, d[4] *= g1.x, d[5] *= g1.y, d[6] *= g1.z, d[7] *= g1.w;
    }
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = r * (d[i] - a[i] * r * c);
    uint4 pk;
    pk.x = pack_bf16x2(o[0], o[1]);
    pk.y = pack_bf16x2(o[2], o[3]);
    pk.z = pack_bf16x2(o[4], o[5]);
    pk.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(dx + row * K + k) = pk;
  }
}

// The same per-row math with one 256-thread CTA per row held in registers
// (NV chunks of 8 columns per thread, K = 2048 NV): x, dA and g are read
// from HBM once, every load issued before the first use; the two row sums
// are reduced through shared memory.
template <int NV>
__global__ void __launch_bounds__(256) rms_backward_rows_cta_kernel(const __nv_bfloat16* __restrict__ x,
                                                                    const float* __restrict__ dA,
                                                                    const float* __restrict__ g, float eps,
                                                                    __nv_bfloat16* __restrict__ dx,
                                                                    float* __restrict__ r_out, int K) {
  __shared__ float red[2][8];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * K;
  const float* dr = dA + row * K;
  float a[NV][8], d[NV][8];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int k = (v * 256 + threadIdx.x) * 8;
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(xr + k)), a[v]);
    const float4 d0 = __ldg(reinterpret_cast<const float4*>(dr + k)), d1 = __ldg(reinterpret_cast<const float4*>(dr + k + 4));
    d[v][0] = d0.x, d[v][1] = d0.y, d[v][2] = d0.z, d[v][3] = d0.w;
    d[v][4] = d1.x, d[v][5] = d1.y, d[v][6] = d1.z, d[v][7] = d1.w;
  }
  if (g) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int k = (v * 256 + threadIdx.x) * 8;
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(g + k)), g1 = __ldg(reinterpret_cast<const float4*>(g + k + 4));
      d[v][0] *= g0.x, d[v][1] *= g0.y, d[v][2] *= g0.z, d[v][3] *= g0.w;
      d[v][4] *= g1.x, d[v][5] *= g1.y, d[v][6] *= g1.z, d[v][7] *= g1.w;
    }
  }
  float ss = 0.f, sd = 0.f;  // sum x^2, sum dA g x
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(a[v][i], a[v][i], ss);
      sd = fmaf(d[v][i], a[v][i], sd);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    sd += __shfl_xor_sync(0xffffffffu, sd, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = ss;
    red[1][warp] = sd;
  }
  __syncthreads();
  ss = 0.f;
  sd = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) {  // every thread sums the warps' parts in the same order
    ss += red[0][w];
    sd += red[1][w];
  }
  const float r = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
  const float c = sd * r / static_cast<float>(K);  // mean_k(dA g xn)
  if (threadIdx.x == 0) r_out[row] = r;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int k = (v * 256 + threadIdx.x) * 8;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = r * (d[v][i] - a[v][i] * r * c);
    uint4 pk;
    pk.x = pack_bf16x2(o[0], o[1]);
    pk.y = pack_bf16x2(o[2], o[3]);
    pk.z = pack_bf16x2(o[4], o[5]);
    pk.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(dx + row * K + k) = pk;
  }
}

// part[chunk][k] = sum over the chunk's kDgRows rows of dA_mk * x_mk * r_m;
// four columns per thread.  grid (ceil(K/4/256), chunks): 32-row chunks give
// the GPU several CTAs per SM, and a full chunk's loads are issued in groups of
// eight rows before they are summed (in row order).
__global__ void __launch_bounds__(256) dg_partial_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const float* __restrict__ dA, const float* __restrict__ r,
                                                         float* __restrict__ part, int64_t M, int K) {
  const int k = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (k >= K) return;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kDgRows;
  const int64_t m1 = m0 + kDgRows < M ? m0 + kDgRows : M;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  auto add_row = [&](const uint2 xv, const float4 d, const float rm) {
    const __nv_bfloat162 x01 = *reinterpret_cast<const __nv_bfloat162*>(&xv.x);
    const __nv_bfloat162 x23 = *reinterpret_cast<const __nv_bfloat162*>(&xv.y);
    s0 = fmaf(d.x, __low2float(x01) * rm, s0);
    s1 = fmaf(d.y, __high2float(x01) * rm, s1);
    s2 = fmaf(d.z, __low2float(x23) * rm, s2);
    s3 = fmaf(d.w, __high2float(x23) * rm, s3);
  };
  int64_t m = m0;
  for (; m + 8 <= m1; m += 8) {
    uint2 xv[8];
    float4 d[8];
    float rm[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[i] = __ldg(reinterpret_cast<const uint2*>(x + (m + i) * K + k));
      d[i] = __ldg(reinterpret_cast<const float4*>(dA + (m + i) * K + k));
      rm[i] = __ldg(r + m + i);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) add_row(xv[i], d[i], rm[i]);
  }
  for (; m < m1; ++m)
    add_row(*reinterpret_cast<const uint2*>(x + m * K + k), *reinterpret_cast<const float4*>(dA + m * K + k), r[m]);
  *reinterpret_cast<float4*>(part + static_cast<int64_t>(blockIdx.y) * K + k) = make_float4(s0, s1, s2, s3);
}

// dg[k] = sum of the chunks' partials, in chunk order (loads issued eight
// chunks ahead of the sum).
__global__ void __launch_bounds__(256) dg_sum_kernel(const float* __restrict__ part, float* __restrict__ dg, int chunks,
                                                     int K) {
  const int k = blockIdx.x * 256 + threadIdx.x;
  if (k >= K) return;
  float s = 0.f;
  int c = 0;
  for (; c + 8 <= chunks; c += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __ldg(part + static_cast<int64_t>(c + i) * K + k);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
  }
  for (; c < chunks; ++c) s += part[static_cast<int64_t>(c) * K + k];
  dg[k] = s;
}
}  // namespace
}  // namespace kda

extern "C" size_t kda_rmsnorm_matmul_backward_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  const size_t m = M, k = K, n = N, chunks = (m + kDgRows - 1) / kDgRows;
  (void)n;
  // a (bf16), dA (fp32), r (fp32), dg partials (fp32)
  return align256(m * k * 2) + align256(m * k * 4) + align256(m * 4) + align256(chunks * k * 4);
}

extern "C" kda_status kda_rmsnorm_matmul_backward_bf16(const void* dy, const void* x, const void* w, const float* g,
                                                       float eps, void* dx, void* dw, float* dg, int64_t M,
                                                       int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                                                       void* stream) {
  const char* op = "rmsnorm_matmul_backward";
  KDA_TRY(check_dims(op, M, K, N));
  KDA_CHECK_ARG(dy && x && w && dx && dw, "%s: null pointer", op);
  KDA_CHECK_ARG(!g == !dg, "%s: dg is written exactly when g is given", op);
  KDA_CHECK_ARG(eps >= 0.f, "%s: eps must be >= 0", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "%s: K (%lld) and N (%lld) must be multiples of 8", op,
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(dy) && al16(x) && al16(w) && al16(dx) && al16(dw) && (!g || al16(g)) &&
                          (!dg || al16(dg)),
                      "%s: pointers must be 16-byte aligned", op);
  KDA_F32_COMMON(op, kda_rmsnorm_matmul_backward_workspace_size(M, K, N));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<uint8_t*>(workspace)};
  __nv_bfloat16* a = c.take<__nv_bfloat16>(static_cast<size_t>(M) * K);
  float* dA = c.take<float>(static_cast<size_t>(M) * K);
  float* r = c.take<float>(static_cast<size_t>(M));
  const int chunks = cdiv(M, kDgRows);
  float* part = c.take<float>(static_cast<size_t>(chunks) * K);
  // the forward's GEMM operand, recomputed: a = bf16(x r g)
  launch_rms_prep<false>(static_cast<const __nv_bfloat16*>(x), nullptr, g, eps, a, static_cast<int>(M),
                         static_cast<int>(K), st);
  KDA_TRY(launch_status("rms_prep_kernel"));
  // dA (M,K) fp32 = dy (M,N) @ w^T (N,K): w (K,N) is that product's K-major
  // B operand as stored (rows = output columns, contraction contiguous)
  {
    CUtensorMap ta, tb, to;
    const bool pair = M > gemm::BM && N >= 256 && K > 128;
    KDA_TRY(tmap2(&ta, dy, N, M, N, 128));
    KDA_TRY(tmap2(&tb, w, N, K, N, pair ? 128 : 256));
    KDA_TRY(tmap_out2_f32(&to, dA, K, M, K));
    Params p = base_params(M, K, N, 256, pair);
    p.out = dA;
    kda_status s_;
    if (pair)
      s_ = gemm::launch<256, false, false, gemm::EPI_F32OUT, false, gemm::B_SINGLE, 6, true>(ta, tb, ta, tb, to, p,
                                                                                            gemm_err_word(), st);
    else
      s_ = gemm::launch<256, false, false, gemm::EPI_F32OUT, false, gemm::B_SINGLE, 4>(ta, tb, ta, tb, to, p,
                                                                                      gemm_err_word(), st);
    KDA_TRY(s_);
  }
  // dw (K,N) = a^T @ dy: a stored (M,K) is the MN-major lhs of transpose_matmul
  KDA_TRY(kda_transpose_matmul_bf16(a, dy, dw, K, M, N, stream));
  {
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    auto* dxb = static_cast<__nv_bfloat16*>(dx);
    const unsigned rows = static_cast<unsigned>(M);
    if (K == 2048)
      rms_backward_rows_cta_kernel<1><<<rows, 256, 0, st>>>(xb, dA, g, eps, dxb, r, static_cast<int>(K));
    else if (K == 4096)
      rms_backward_rows_cta_kernel<2><<<rows, 256, 0, st>>>(xb, dA, g, eps, dxb, r, static_cast<int>(K));
    else if (K == 8192)
      rms_backward_rows_cta_kernel<4><<<rows, 256, 0, st>>>(xb, dA, g, eps, dxb, r, static_cast<int>(K));
    else
      rms_backward_rows_kernel<<<static_cast<unsigned>(cdiv(M, 8)), 256, 0, st>>>(xb, dA, g, eps, dxb, r, M,
                                                                                  static_cast<int>(K));
    KDA_TRY(launch_status("rms_backward_rows_kernel"));
  }
  if (g) {
    dg_partial_kernel<<<dim3(static_cast<unsigned>(cdiv(K / 4, 256)), static_cast<unsigned>(chunks)), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), dA, r, part, M, static_cast<int>(K));
    dg_sum_kernel<<<static_cast<unsigned>(cdiv(K, 256)), 256, 0, st>>>(part, dg, chunks, static_cast<int>(K));
    KDA_TRY(launch_status("dg_kernels"));
  }
  return KDA_OK;
}

// ----------------------------------------------------------- swiglu backward
// Gradients of out = h @ w_down, h = silu(g) u, g = x @ w_gate, u = x @ w_up:
//   dh = dout @ w_down^T; dg = dh u silu'(g); du = dh silu(g)
//   dw_down = h^T dout; dw_gate = x^T dg; dw_up = x^T du;
//   dx = dg @ w_gate^T + du @ w_up^T   (ONE K-extended GEMM over 2 d_ff)
// g and u are recomputed (two GEMMs) unless the forward kept them
// (kda_swiglu_gu_bf16 / kda_swiglu_backward_saved_bf16); the weights are read
// as stored (K-major B operands of dh and dx); the x^T / h^T products are the
// transpose_matmul kernel.  bf16 storage,
// fp32 accumulation and fp32 elementwise math.
namespace kda {
namespace {
// h, dg, du from g, u, dh (bf16, 8 per thread).
__global__ void __launch_bounds__(256) swiglu_bwd_elem_kernel(const __nv_bfloat16* __restrict__ g,
                                                              const __nv_bfloat16* __restrict__ u,
                                                              const __nv_bfloat16* __restrict__ dh,
                                                              __nv_bfloat16* __restrict__ h,
                                                              __nv_bfloat16* __restrict__ dg,
                                                              __nv_bfloat16* __restrict__ du, int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  float gv[8], uv[8], dv[8], ho[8], go[8], uo[8];
  unpack_bf16x8(reinterpret_cast<const uint4*>(g)[i], gv);
  unpack_bf16x8(reinterpret_cast<const uint4*>(u)[i], uv);
  unpack_bf16x8(reinterpret_cast<const uint4*>(dh)[i], dv);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float s = 1.0f / (1.0f + expf(-gv[q]));
    const float sg = gv[q] * s;
    ho[q] = sg * uv[q];
    go[q] = dv[q] * uv[q] * s * (1.0f + gv[q] * (1.0f - s));
    uo[q] = dv[q] * sg;
  }
  uint4 a, b, c;
  a.x = pack_bf16x2(ho[0], ho[1]), a.y = pack_bf16x2(ho[2], ho[3]), a.z = pack_bf16x2(ho[4], ho[5]),
  a.w = pack_bf16x2(ho[6], ho[7]);
  b.x = pack_bf16x2(go[0], go[1]), b.y = pack_bf16x2(go[2], go[3]), b.z = pack_bf16x2(go[4], go[5]),
  b.w = pack_bf16x2(go[6], go[7]);
  c.x = pack_bf16x2(uo[0], uo[1]), c.y = pack_bf16x2(uo[2], uo[3]), c.z = pack_bf16x2(uo[4], uo[5]),
  c.w = pack_bf16x2(uo[6], uo[7]);
  reinterpret_cast<uint4*>(h)[i] = a;
  reinterpret_cast<uint4*>(dg)[i] = b;
  reinterpret_cast<uint4*>(du)[i] = c;
}

// h = silu(g) * u from the bf16 g, u (8 per thread; the same arithmetic as
// swiglu_bwd_elem_kernel's h, so forward and backward agree bit for bit).
__global__ void __launch_bounds__(256) swiglu_h_kernel(const __nv_bfloat16* __restrict__ g,
                                                       const __nv_bfloat16* __restrict__ u,
                                                       __nv_bfloat16* __restrict__ h, int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  float gv[8], uv[8], ho[8];
  unpack_bf16x8(reinterpret_cast<const uint4*>(g)[i], gv);
  unpack_bf16x8(reinterpret_cast<const uint4*>(u)[i], uv);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float s = 1.0f / (1.0f + expf(-gv[q]));
    ho[q] = gv[q] * s * uv[q];
  }
  uint4 a;
  a.x = pack_bf16x2(ho[0], ho[1]), a.y = pack_bf16x2(ho[2], ho[3]), a.z = pack_bf16x2(ho[4], ho[5]),
  a.w = pack_bf16x2(ho[6], ho[7]);
  reinterpret_cast<uint4*>(h)[i] = a;
}

}  // namespace
}  // namespace kda

namespace kda {
namespace {

kda_status swiglu_check(const char* op, int64_t M, int64_t K, int64_t N, std::initializer_list<const void*> ptrs) {
  KDA_TRY(check_dims(op, M, K, N));
  for (const void* q : ptrs) KDA_CHECK_ARG(q, "%s: null pointer", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "%s: K (%lld) and N (%lld) must be multiples of 8", op,
                      (long long)K, (long long)N);
  for (const void* q : ptrs) KDA_CHECK_SUPPORTED(al16(q), "%s: pointers must be 16-byte aligned", op);
  return KDA_OK;
}

// Workspace of the backward given g and u: dh, h, dg, du (M x F), bf16.
size_t swiglu_backward_core_bytes(int64_t M, int64_t K, int64_t N) {
  (void)K;
  const size_t m = M, f = N;
  return 4 * align256(m * f * 2);
}

// out (M,N) bf16 = A (M,K) @ B^T with B stored (N,K) -- B^T's K-major form,
// read as stored (no transpose pass).
kda_status gemm_bt(const void* A, const void* Bnk, void* out, int64_t M, int64_t K, int64_t N, cudaStream_t st) {
  const bool pair = N > 128 && M > gemm::BM && K >= 256;
  const int bn = N <= 128 ? 128 : 256;
  CUtensorMap ta, tb, to;
  KDA_TRY(tmap2(&ta, A, K, M, K, 128));
  KDA_TRY(tmap2(&tb, Bnk, K, N, K, pair ? 128 : bn));
  KDA_TRY(tmap_out2(&to, out, N, M, N));
  Params p = base_params(M, N, K, bn, pair);
  p.out = out;
  unsigned* err = gemm_err_word();
  if (bn == 128)
    return gemm::launch<128, false, false, gemm::EPI_BF16, false, gemm::B_SINGLE, 6>(ta, tb, ta, tb, to, p, err, st);
  if (pair)
    return gemm::launch<256, false, false, gemm::EPI_BF16, false, gemm::B_SINGLE, 6, true>(ta, tb, ta, tb, to, p, err,
                                                                                          st);
  return gemm::launch<256, false, false, gemm::EPI_BF16, false, gemm::B_SINGLE, 4>(ta, tb, ta, tb, to, p, err, st);
}

// dx, dw_up, dw_down, dw_gate given g = x w_gate and u = x w_up (bf16, M x F).
kda_status swiglu_backward_core(const void* dout, const void* x, const void* w_up, const void* w_down,
                                const void* w_gate, const __nv_bfloat16* g, const __nv_bfloat16* u, void* dx,
                                void* dw_up, void* dw_down, void* dw_gate, int64_t M, int64_t K, int64_t N, Carve& c,
                                cudaStream_t st) {
  const int64_t F = N;
  const size_t mf = static_cast<size_t>(M) * F;
  __nv_bfloat16* dh = c.take<__nv_bfloat16>(mf);
  __nv_bfloat16* h = c.take<__nv_bfloat16>(mf);
  __nv_bfloat16* dg = c.take<__nv_bfloat16>(mf);
  __nv_bfloat16* du = c.take<__nv_bfloat16>(mf);
  KDA_TRY(gemm_bt(dout, w_down, dh, M, K, F, st));           // dh (M,F) = dout (M,K) @ w_down^T (K,F)
  const int64_t n8 = static_cast<int64_t>(mf / 8);
  swiglu_bwd_elem_kernel<<<static_cast<unsigned>(cdiv(n8, 256)), 256, 0, st>>>(g, u, dh, h, dg, du, n8);
  KDA_TRY(launch_status("swiglu_bwd_elem_kernel"));
  KDA_TRY(kda_transpose_matmul_bf16(h, dout, dw_down, F, M, K, st));   // h^T (F,M) @ dout (M,K)
  KDA_TRY(kda_transpose_matmul_bf16(x, dg, dw_gate, K, M, F, st));     // x^T (K,M) @ dg (M,F)
  KDA_TRY(kda_transpose_matmul_bf16(x, du, dw_up, K, M, F, st));       // x^T (K,M) @ du (M,F)
  // dx (M,K) = [dg | du] @ [w_gate^T ; w_up^T]: w_gate, w_up (K,F) are the
  // K-major B operands as stored
  const bool pair = M > gemm::BM;
  CUtensorMap ta, ta2, tb, tb2, to;
  KDA_TRY(tmap2(&ta, dg, F, M, F, 128));
  KDA_TRY(tmap2(&ta2, du, F, M, F, 128));
  KDA_TRY(tmap2(&tb, w_gate, F, K, F, pair ? 128 : 256));
  KDA_TRY(tmap2(&tb2, w_up, F, K, F, pair ? 128 : 256));
  KDA_TRY(tmap_out2(&to, dx, K, M, K));
  Params p = base_params(M, K, F, 256, pair);
  p.k_blocks2 = cdiv(F, gemm::BK);
  p.out = dx;
  if (pair)
    return gemm::launch<256, false, false, gemm::EPI_BF16, false, gemm::B_KEXT, 6, true>(ta, tb, ta2, tb2, to, p,
                                                                                         gemm_err_word(), st);
  return gemm::launch<256, false, false, gemm::EPI_BF16, false, gemm::B_KEXT, 4>(ta, tb, ta2, tb2, to, p,
                                                                                 gemm_err_word(), st);
}

}  // namespace
}  // namespace kda

extern "C" size_t kda_swiglu_backward_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  // g and u (M x F, bf16), then the backward proper
  return 2 * align256(static_cast<size_t>(M) * N * 2) + kda::swiglu_backward_core_bytes(M, K, N);
}

extern "C" kda_status kda_swiglu_backward_bf16(const void* dout, const void* x, const void* w_up, const void* w_down,
                                               const void* w_gate, void* dx, void* dw_up, void* dw_down,
                                               void* dw_gate, int64_t M, int64_t K, int64_t N, void* workspace,
                                               size_t workspace_bytes, void* stream) {
  const char* op = "swiglu_backward";
  KDA_TRY(kda::swiglu_check(op, M, K, N, {dout, x, w_up, w_down, w_gate, dx, dw_up, dw_down, dw_gate}));
  KDA_F32_COMMON(op, kda_swiglu_backward_workspace_size(M, K, N));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<uint8_t*>(workspace)};
  const size_t mf = static_cast<size_t>(M) * N;
  __nv_bfloat16* g = c.take<__nv_bfloat16>(mf);
  __nv_bfloat16* u = c.take<__nv_bfloat16>(mf);
  KDA_TRY(plain_gemm(x, w_gate, g, M, K, N, st));
  KDA_TRY(plain_gemm(x, w_up, u, M, K, N, st));
  return kda::swiglu_backward_core(dout, x, w_up, w_down, w_gate, g, u, dx, dw_up, dw_down, dw_gate, M, K, N, c, st);
}

extern "C" size_t kda_swiglu_gu_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return align256(static_cast<size_t>(M) * N * 2);  // h
}

extern "C" kda_status kda_swiglu_gu_bf16(const void* x, const void* w_up, const void* w_down, const void* w_gate,
                                         void* out, void* g, void* u, int64_t M, int64_t K, int64_t N, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  const char* op = "swiglu_gu";
  KDA_TRY(kda::swiglu_check(op, M, K, N, {x, w_up, w_down, w_gate, out, g, u}));
  KDA_F32_COMMON(op, kda_swiglu_gu_workspace_size(M, K, N));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __nv_bfloat16* h = static_cast<__nv_bfloat16*>(workspace);
  KDA_TRY(plain_gemm(x, w_gate, g, M, K, N, st));
  KDA_TRY(plain_gemm(x, w_up, u, M, K, N, st));
  const int64_t n8 = M * N / 8;
  swiglu_h_kernel<<<static_cast<unsigned>(cdiv(n8, 256)), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(u), h, n8);
  KDA_TRY(launch_status("swiglu_h_kernel"));
  return plain_gemm(h, w_down, out, M, N, K, st);
}

extern "C" size_t kda_swiglu_backward_saved_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return kda::swiglu_backward_core_bytes(M, K, N);
}

extern "C" kda_status kda_swiglu_backward_saved_bf16(const void* dout, const void* x, const void* w_up,
                                                     const void* w_down, const void* w_gate, const void* g,
                                                     const void* u, void* dx, void* dw_up, void* dw_down, void* dw_gate,
                                                     int64_t M, int64_t K, int64_t N, void* workspace,
                                                     size_t workspace_bytes, void* stream) {
  const char* op = "swiglu_backward_saved";
  KDA_TRY(kda::swiglu_check(op, M, K, N, {dout, x, w_up, w_down, w_gate, g, u, dx, dw_up, dw_down, dw_gate}));
  KDA_F32_COMMON(op, kda_swiglu_backward_saved_workspace_size(M, K, N));
  Carve c{static_cast<uint8_t*>(workspace)};
  return kda::swiglu_backward_core(dout, x, w_up, w_down, w_gate, static_cast<const __nv_bfloat16*>(g),
                                   static_cast<const __nv_bfloat16*>(u), dx, dw_up, dw_down, dw_gate, M, K, N, c,
                                   static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------- gqa_full backward
// Gradients of out_h = softmax(q_h k_g^T * scale [+ causal mask]) v_g, query
// head h in kv group g, given dout in the reference order (B, QH, S, D):
//   P = softmax(S), S = q_h k_g^T scale ; dP = dout_h v_g^T ;
//   dS = P (dP - rowsum(P dP)) scale ; dq_h = dS k_g ; dk_g = sum_h dS^T q_h ;
//   dv_g = sum_h P^T dout_h
// The forward reruns for every query row's log2-sum-exp (and out, for
// rowsum(P dP) = rowsum(dout * out)); the rest is one flash-style kernel
// (csrc/attn_bwd.cu) per call: P and dS never leave shared memory.
namespace kda {
namespace {
// di[row] = sum_d dout[row][d] * o[row][d] (rows of D = 128 bf16, fp32 sum):
// the attention backward's rowsum(P * dP) = dout . out for every query row.
// One warp per row, all its loads issued first.
__global__ void __launch_bounds__(256) rowdot_kernel(const __nv_bfloat16* __restrict__ a,
                                                     const __nv_bfloat16* __restrict__ b, float* __restrict__ out,
                                                     int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  // 128 values per row: lane l holds 4 of them (8 bytes)
  const uint2 va = reinterpret_cast<const uint2*>(a + row * 128)[lane];
  const uint2 vb = reinterpret_cast<const uint2*>(b + row * 128)[lane];
  const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&va);
  const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&vb);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 fa = __bfloat1622float2(pa[i]), fb = __bfloat1622float2(pb[i]);
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[row] = acc;
}

}  // namespace
}  // namespace kda

namespace kda {
namespace {

// Workspace of the backward proper (everything after the forward): di, the
// fp32 dq scratch and, with RoPE, the table, rotated q and k, and dq, dk
// before the inverse rotation.
size_t gqa_backward_core_bytes(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D, float rope_theta) {
  const size_t b = B, s = S, qh = QH, kh = KH, d = D;
  size_t n = align256(b * qh * s * 4) + align256(attn_backward_scratch_bytes(B, S, QH));
  if (rope_theta > 0.f)
    n += align256(s * (d / 2) * 8) + 2 * align256(b * s * qh * d * 2) + 2 * align256(b * s * kh * d * 2);
  return n;
}

// Shape, pointer and alignment checks shared by both backward entry points.
kda_status gqa_backward_check(const char* op, const void* dout, const void* q, const void* k, const void* v,
                              const void* dq, const void* dk, const void* dv, int64_t B, int64_t S, int64_t QH,
                              int64_t KH, int64_t D) {
  KDA_CHECK_ARG(B > 0 && S > 0 && QH > 0 && KH > 0 && QH % KH == 0 && B * KH < 65536,
                "%s: bad shape B=%lld S=%lld QH=%lld KH=%lld", op, (long long)B, (long long)S, (long long)QH,
                (long long)KH);
  KDA_CHECK_ARG(dout && q && k && v && dq && dk && dv, "%s: null pointer", op);
  KDA_CHECK_SUPPORTED(D == 128, "%s: head_dim must be 128 (got %lld)", op, (long long)D);
  KDA_CHECK_SUPPORTED(S % 8 == 0 && S < (1 << 20), "%s: S (%lld) must be a multiple of 8", op, (long long)S);
  KDA_CHECK_SUPPORTED(al16(dout) && al16(q) && al16(k) && al16(v) && al16(dq) && al16(dk) && al16(dv),
                      "%s: pointers must be 16-byte aligned", op);
  return KDA_OK;
}

// The backward given the forward's output O (the reference order
// (B, QH, S, D), like dout) and its rows' log2-sum-exp: di = rowsum(dout * O),
// then the flash-style kernel on q and k (rotated first with RoPE, dq and dk
// rotated back at the end).  Takes its buffers from `c`.
kda_status gqa_backward_core(const void* dout, const void* q, const void* k, const void* v, const __nv_bfloat16* O,
                             const float* lse, void* dq, void* dk, void* dv, int64_t B, int64_t S, int64_t QH,
                             int64_t KH, int64_t D, int causal, float rope_theta, Carve& c, cudaStream_t st) {
  float* di = c.take<float>(static_cast<size_t>(B) * QH * S);
  float* dq32 = c.take<float>(attn_backward_scratch_bytes(B, S, QH) / 4);
  const bool rope = rope_theta > 0.f;
  rowdot_kernel<<<static_cast<unsigned>(cdiv(B * QH * S, 8)), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(dout), O, di, B * QH * S);
  KDA_TRY(launch_status("rowdot_kernel"));
  const __nv_bfloat16* qsrc = static_cast<const __nv_bfloat16*>(q);
  const __nv_bfloat16* ksrc = static_cast<const __nv_bfloat16*>(k);
  __nv_bfloat16* dq_t = static_cast<__nv_bfloat16*>(dq);
  __nv_bfloat16* dk_t = static_cast<__nv_bfloat16*>(dk);
  float2* tab = nullptr;
  if (rope) {
    // the gradients w.r.t. the rotated q and k, rotated back at the end
    const size_t nq = static_cast<size_t>(B) * S * QH * D, nk = static_cast<size_t>(B) * S * KH * D;
    tab = c.take<float2>(static_cast<size_t>(S) * (D / 2));
    __nv_bfloat16* qr = c.take<__nv_bfloat16>(nq);
    __nv_bfloat16* kr = c.take<__nv_bfloat16>(nk);
    dq_t = c.take<__nv_bfloat16>(nq);
    dk_t = c.take<__nv_bfloat16>(nk);
    KDA_TRY(rope_table(tab, S, rope_theta, st));
    KDA_TRY(rope_rotate_rows(qsrc, qr, tab, B * S * QH, S, QH, false, st));
    KDA_TRY(rope_rotate_rows(ksrc, kr, tab, B * S * KH, S, KH, false, st));
    qsrc = qr;
    ksrc = kr;
  }
  KDA_TRY(attn_backward_flash(qsrc, ksrc, static_cast<const __nv_bfloat16*>(v),
                              static_cast<const __nv_bfloat16*>(dout), lse, di, dq_t, dk_t,
                              static_cast<__nv_bfloat16*>(dv), dq32, B, S, QH, KH, causal != 0, st));
  if (rope) {
    KDA_TRY(rope_rotate_rows(dq_t, static_cast<__nv_bfloat16*>(dq), tab, B * S * QH, S, QH, true, st));
    KDA_TRY(rope_rotate_rows(dk_t, static_cast<__nv_bfloat16*>(dk), tab, B * S * KH, S, KH, true, st));
  }
  return KDA_OK;
}

}  // namespace
}  // namespace kda

extern "C" size_t kda_gqa_full_backward_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                                       float rope_theta) {
  if (B <= 0 || S <= 0 || QH <= 0 || KH <= 0 || D <= 0 || QH % KH) return 0;
  const size_t b = B, s = S, qh = QH, d = D;
  // the forward's output (B, QH, S, D), its rows' log2-sum-exp (B, QH, S)
  // fp32, its own workspace, then the backward proper
  return align256(b * qh * s * d * 2) + align256(b * qh * s * 4) +
         align256(kda_gqa_full_workspace_size(B, S, QH, KH, D, rope_theta)) +
         kda::gqa_backward_core_bytes(B, S, QH, KH, D, rope_theta);
}

extern "C" kda_status kda_gqa_full_backward_bf16(const void* dout, const void* q, const void* k, const void* v,
                                                 void* dq, void* dk, void* dv, int64_t B, int64_t S, int64_t QH,
                                                 int64_t KH, int64_t D, int causal, float rope_theta, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
  const char* op = "gqa_full_backward";
  KDA_TRY(kda::gqa_backward_check(op, dout, q, k, v, dq, dk, dv, B, S, QH, KH, D));
  KDA_F32_COMMON(op, kda_gqa_full_backward_workspace_size(B, S, QH, KH, D, rope_theta));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<uint8_t*>(workspace)};
  __nv_bfloat16* O = c.take<__nv_bfloat16>(static_cast<size_t>(B) * QH * S * D);
  float* lse = c.take<float>(static_cast<size_t>(B) * QH * S);
  const size_t fws_bytes = kda_gqa_full_workspace_size(B, S, QH, KH, D, rope_theta);
  uint8_t* fws = c.take<uint8_t>(fws_bytes);
  // the forward (same causal mask and RoPE) gives out, in dout's (B, QH, S, D)
  // order, and every query row's log2-sum-exp
  KDA_TRY(gqa_forward(q, k, v, O, B, S, QH, KH, D, causal, rope_theta, 0, fws, fws_bytes, lse, st));
  return kda::gqa_backward_core(dout, q, k, v, O, lse, dq, dk, dv, B, S, QH, KH, D, causal, rope_theta, c, st);
}

extern "C" size_t kda_gqa_full_backward_saved_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                                             float rope_theta) {
  if (B <= 0 || S <= 0 || QH <= 0 || KH <= 0 || D <= 0 || QH % KH) return 0;
  return kda::gqa_backward_core_bytes(B, S, QH, KH, D, rope_theta);
}

extern "C" kda_status kda_gqa_full_backward_saved_bf16(const void* dout, const void* q, const void* k, const void* v,
                                                       const void* out, const float* lse, void* dq, void* dk, void* dv,
                                                       int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                                       int causal, float rope_theta, void* workspace,
                                                       size_t workspace_bytes, void* stream) {
  const char* op = "gqa_full_backward_saved";
  KDA_TRY(kda::gqa_backward_check(op, dout, q, k, v, dq, dk, dv, B, S, QH, KH, D));
  KDA_CHECK_ARG(out && lse, "%s: null out or lse", op);
  KDA_CHECK_SUPPORTED(al16(out) && al16(lse), "%s: out and lse must be 16-byte aligned", op);
  KDA_F32_COMMON(op, kda_gqa_full_backward_saved_workspace_size(B, S, QH, KH, D, rope_theta));
  Carve c{static_cast<uint8_t*>(workspace)};
  return kda::gqa_backward_core(dout, q, k, v, static_cast<const __nv_bfloat16*>(out), lse, dq, dk, dv, B, S, QH,
                                KH, D, causal, rope_theta, c, static_cast<cudaStream_t>(stream));
}

