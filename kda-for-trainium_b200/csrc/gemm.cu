// bf16 contraction entry points built on the tcgen05 GEMM engine (gemm.cuh):
// matmul, transpose_matmul, bmm, bmm_softmax, rmsnorm_matmul,
// add_rmsnorm_matmul, matmul_add_rmsnorm, swiglu, lora (the RMS pre-pass
// kernels are in gemm_host.cuh, the row-norm kernels here).
#include "gemm.cuh"

KDA_DEFINE_ERROR_WORD(gemm)
static unsigned* gemm_err_word() { return kda_err_ptr_gemm(); }

#include "gemm_host.cuh"

using namespace kda;

extern "C" kda_status kda_matmul_bf16(const void* lhs, const void* rhs, void* out, int64_t M, int64_t K, int64_t N,
                                      void* stream) {
  KDA_TRY(check_dims("matmul", M, K, N));
  KDA_CHECK_ARG(lhs && rhs && out, "matmul: null pointer");
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "matmul: K (%lld) and N (%lld) must be multiples of 8",
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(lhs) && al16(rhs) && al16(out), "matmul: pointers must be 16-byte aligned");
  return plain_gemm(lhs, rhs, out, M, K, N, static_cast<cudaStream_t>(stream));
}

extern "C" kda_status kda_transpose_matmul_bf16(const void* lhs, const void* rhs, void* out, int64_t M, int64_t K,
                                                int64_t N, void* stream) {
  KDA_TRY(check_dims("transpose_matmul", M, K, N));
  KDA_CHECK_ARG(lhs && rhs && out, "transpose_matmul: null pointer");
  KDA_CHECK_SUPPORTED(M % 8 == 0 && N % 8 == 0, "transpose_matmul: M (%lld) and N (%lld) must be multiples of 8",
                      (long long)M, (long long)N);
  KDA_CHECK_SUPPORTED(al16(lhs) && al16(rhs) && al16(out), "transpose_matmul: pointers must be 16-byte aligned");
  CUtensorMap ta, tb;
  KDA_TRY(tmap2(&ta, lhs, M, K, M, 64));  // lhs (K, M): MN-major A
  KDA_TRY(tmap2(&tb, rhs, N, K, N, 64));
  CUtensorMap to;
  KDA_TRY(tmap_out2(&to, out, N, M, N));
  if (M > gemm::BM) {
    Params p = base_params(M, N, K, 256, true);
    p.out = out;
    return gemm::launch<256, true, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 6, true>(
        ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
  }
  Params p = base_params(M, N, K, 256);
  p.out = out;
  return gemm::launch<256, true, true, gemm::EPI_BF16, false, gemm::B_SINGLE, 4>(
      ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
}

extern "C" kda_status kda_bmm_bf16(const void* lhs, const void* rhs, void* out, int64_t batch, int64_t M, int64_t K,
                                   int64_t N, void* stream) {
  KDA_TRY(check_dims("bmm", M, K, N));
  KDA_CHECK_ARG(batch > 0 && batch < 65536, "bmm: bad batch %lld", (long long)batch);
  KDA_CHECK_ARG(lhs && rhs && out, "bmm: null pointer");
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "bmm: K (%lld) and N (%lld) must be multiples of 8", (long long)K,
                      (long long)N);
  KDA_CHECK_SUPPORTED(al16(lhs) && al16(rhs) && al16(out), "bmm: pointers must be 16-byte aligned");
  CUtensorMap ta, tb;
  KDA_TRY(tmap3(&ta, lhs, K, M, K, batch, M * K, 128));
  KDA_TRY(tmap3(&tb, rhs, N, K, N, batch, K * N, 64));
  CUtensorMap to;
  KDA_TRY(tmap_out3(&to, out, N, M, N, batch, M * N));
  // K = 64-class batches are output-bound: single-CTA tiles keep the epilogue
  // free of the pair's cross-CTA handshake
  const bool pair = M > gemm::BM && K >= 256;
  Params p = base_params(M, N, K, 256, pair);
  p.batch = static_cast<int>(batch);
  p.out = out;
  p.out_bstride = M * N;
  if (pair)
    return gemm::launch<256, false, true, gemm::EPI_BF16, true, gemm::B_SINGLE, 6, true>(
        ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
  return gemm::launch<256, false, true, gemm::EPI_BF16, true, gemm::B_SINGLE, 4>(
      ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
}

// Workspace: the normalised activations (M x K bf16), then the GEMM's tail
// split (fp32 partial tiles of the last wave, and their counters).
extern "C" size_t kda_rmsnorm_matmul_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0) return 0;
  const TailPlan t = tail_plan(M, K, N);
  return align256(static_cast<size_t>(M) * K * 2) + t.part_bytes + t.cnt_bytes;
}

static kda_status rms_then_gemm(const char* op, const void* x, const void* z, const void* w, const float* g, float eps,
                                void* out, int64_t M, int64_t K, int64_t N, void* ws, size_t ws_bytes,
                                void* stream) {
  KDA_TRY(check_dims(op, M, K, N));
  KDA_CHECK_ARG(x && w && out, "%s: null pointer", op);
  KDA_CHECK_ARG(eps >= 0.f, "%s: eps must be >= 0", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "%s: K (%lld) and N (%lld) must be multiples of 8", op,
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(x) && al16(w) && al16(out) && (!z || al16(z)) && (!g || al16(g)),
                      "%s: pointers must be 16-byte aligned", op);
  const size_t need = kda_rmsnorm_matmul_workspace_size(M, K, N);
  KDA_CHECK_ARG(ws && ws_bytes >= need, "%s: workspace of %zu bytes required, got %zu", op, need, ws_bytes);
  KDA_CHECK_SUPPORTED(al16(ws), "%s: workspace must be 16-byte aligned", op);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* a = static_cast<__nv_bfloat16*>(ws);
  const TailPlan tail = tail_plan(M, K, N);
  uint8_t* tail_ws = static_cast<uint8_t*>(ws) + align256(static_cast<size_t>(M) * K * 2);
  unsigned* tail_cnt = tail.parts > 1 ? reinterpret_cast<unsigned*>(tail_ws + tail.part_bytes) : nullptr;
  // encode the GEMM's tensor maps first: once the short pre-pass is queued,
  // only the GEMM launch itself stands between it and the GEMM
  PlainGemm gm;
  KDA_TRY(plan_plain_gemm(gm, a, w, out, M, K, N, &tail, tail_ws));
  // the pre-pass also zeroes the tail counters
  const int nz = tail.parts > 1 ? 2 * tail.tiles : 0;
  if (z)
    launch_rms_prep<true>(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(z), g, eps, a,
                          static_cast<int>(M), static_cast<int>(K), st, tail_cnt, nz);
  else
    launch_rms_prep<false>(static_cast<const __nv_bfloat16*>(x), nullptr, g, eps, a, static_cast<int>(M),
                           static_cast<int>(K), st, tail_cnt, nz);
  KDA_TRY(launch_status("rms_prep_kernel"));
  return launch_plain_gemm(gm, st, /*pdl=*/true);
}

extern "C" kda_status kda_rmsnorm_matmul_bf16(const void* x, const void* w, const float* g, float eps, void* out,
                                              int64_t M, int64_t K, int64_t N, void* workspace,
                                              size_t workspace_bytes, void* stream) {
  return rms_then_gemm("rmsnorm_matmul", x, nullptr, w, g, eps, out, M, K, N, workspace, workspace_bytes, stream);
}

extern "C" size_t kda_add_rmsnorm_matmul_workspace_size(int64_t M, int64_t K, int64_t N) {
  return kda_rmsnorm_matmul_workspace_size(M, K, N);
}

extern "C" kda_status kda_add_rmsnorm_matmul_bf16(const void* x, const void* w, float eps, const void* z,
                                                  const float* g, void* out, int64_t M, int64_t K, int64_t N,
                                                  void* workspace, size_t workspace_bytes, void* stream) {
  KDA_CHECK_ARG(z && g, "add_rmsnorm_matmul: null pointer");
  return rms_then_gemm("add_rmsnorm_matmul", x, z, w, g, eps, out, M, K, N, workspace, workspace_bytes, stream);
}

extern "C" size_t kda_matmul_add_rmsnorm_workspace_size(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  // per-row sums of squares, the tail split's counters (both zeroed by one
  // memset), its fp32 partials
  const TailPlan t = tail_plan(M, K, N);
  size_t n = align256(static_cast<size_t>(M) * 4);
  if (t.parts > 1) n += t.cnt_bytes + t.part_bytes;
  return n;
}

// y = x @ w + z is written once, as bf16, straight into `out` by the GEMM
// epilogue together with fp32 per-row sums of squares of y; a second light
// pass scales each row in place by g / sqrt(mean(y^2) + eps).
extern "C" kda_status kda_matmul_add_rmsnorm_bf16(const void* x, const void* w, float eps, const void* z,
                                                  const float* g, void* out, int64_t M, int64_t K, int64_t N,
                                                  void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = "matmul_add_rmsnorm";
  KDA_TRY(check_dims(op, M, K, N));
  KDA_CHECK_ARG(x && w && z && g && out, "%s: null pointer", op);
  KDA_CHECK_ARG(eps >= 0.f, "%s: eps must be >= 0", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "%s: K (%lld) and N (%lld) must be multiples of 8", op,
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(x) && al16(w) && al16(z) && al16(g) && al16(out), "%s: pointers must be 16-byte aligned",
                      op);
  const size_t need = kda_matmul_add_rmsnorm_workspace_size(M, K, N);
  KDA_CHECK_ARG(workspace && workspace_bytes >= need, "%s: workspace of %zu bytes required, got %zu", op, need,
                workspace_bytes);
  KDA_CHECK_SUPPORTED(al16(workspace), "%s: workspace must be 16-byte aligned", op);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* rowsq = static_cast<float*>(workspace);
  const bool pair = M > gemm::BM && K >= 256;
  // the last partial wave of pair tiles split along K (as the plain GEMM does)
  const TailPlan tail = pair ? tail_plan(M, K, N) : TailPlan{};
  const size_t rows_bytes = align256(static_cast<size_t>(M) * 4);
  uint8_t* tail_ws = static_cast<uint8_t*>(workspace) + rows_bytes;
  const size_t zero_bytes = rows_bytes + (tail.parts > 1 ? tail.cnt_bytes : 0);
  if (cudaMemsetAsync(rowsq, 0, zero_bytes, st) != cudaSuccess) return launch_status(op);
  CUtensorMap ta, tb, to;
  KDA_TRY(tmap2(&ta, x, K, M, K, 128));
  KDA_TRY(tmap2(&tb, w, N, K, N, 64));
  KDA_TRY(tmap_out2(&to, out, N, M, N));
  Params p = base_params(M, N, K, 256, pair);
  p.out = out;
  p.z = static_cast<const __nv_bfloat16*>(z);
  p.ldz = N;
  p.rowsq = rowsq;
  if (pair && tail.parts > 1) {
    p.tail_parts = tail.parts;
    p.tail_first = tail.first;
    p.tail_kb = tail.kb;
    p.tail_cnt = reinterpret_cast<unsigned*>(tail_ws);
    p.tail_part = reinterpret_cast<float*>(tail_ws + tail.cnt_bytes);
    KDA_TRY((gemm::launch<256, false, true, gemm::EPI_RESID_BF16, false, gemm::B_SINGLE, 6, true, false, true>(
        ta, tb, ta, tb, to, p, gemm_err_word(), st)));
  } else if (pair)
    KDA_TRY((gemm::launch<256, false, true, gemm::EPI_RESID_BF16, false, gemm::B_SINGLE, 6, true>(
        ta, tb, ta, tb, to, p, gemm_err_word(), st)));
  else
    KDA_TRY((gemm::launch<256, false, true, gemm::EPI_RESID_BF16, false, gemm::B_SINGLE, 4>(
        ta, tb, ta, tb, to, p, gemm_err_word(), st)));
  auto* o = static_cast<__nv_bfloat16*>(out);
  const unsigned g2 = static_cast<unsigned>((M + 1) / 2);
  switch (N % 2048 == 0 ? N / 2048 : 0) {
    case 1: rownorm2_inplace_kernel<1><<<g2, 256, 0, st>>>(o, rowsq, g, eps, static_cast<int>(M)); break;
    case 2: rownorm2_inplace_kernel<2><<<g2, 256, 0, st>>>(o, rowsq, g, eps, static_cast<int>(M)); break;
    case 4: rownorm2_inplace_kernel<4><<<g2, 256, 0, st>>>(o, rowsq, g, eps, static_cast<int>(M)); break;
    default:
      rownorm_inplace_kernel<<<static_cast<unsigned>(M), 256, 0, st>>>(o, rowsq, g, eps, static_cast<int>(N));
  }
  return launch_status("rownorm_inplace_kernel");
}

extern "C" size_t kda_swiglu_workspace_size(int64_t M, int64_t K, int64_t N) {
  (void)K;
  return (M > 0 && N > 0) ? align256(static_cast<size_t>(M) * N * 2) : 0;
}

extern "C" kda_status kda_swiglu_bf16(const void* x, const void* w_up, const void* w_down, const void* w_gate,
                                      void* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  const char* op = "swiglu";
  KDA_TRY(check_dims(op, M, K, N));
  KDA_CHECK_ARG(x && w_up && w_down && w_gate && out, "%s: null pointer", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "%s: K (%lld) and N (%lld) must be multiples of 8", op,
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(x) && al16(w_up) && al16(w_down) && al16(w_gate) && al16(out),
                      "%s: pointers must be 16-byte aligned", op);
  const size_t need = kda_swiglu_workspace_size(M, K, N);
  KDA_CHECK_ARG(workspace && workspace_bytes >= need, "%s: workspace of %zu bytes required, got %zu", op, need,
                workspace_bytes);
  KDA_CHECK_SUPPORTED(al16(workspace), "%s: workspace must be 16-byte aligned", op);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* h = workspace;
  CUtensorMap ta, tg, tu;
  KDA_TRY(tmap2(&ta, x, K, M, K, 128));
  KDA_TRY(tmap2(&tg, w_gate, N, K, N, 64));
  KDA_TRY(tmap2(&tu, w_up, N, K, N, 64));
  CUtensorMap th;
  KDA_TRY(tmap_out2(&th, h, N, M, N));
  PlainGemm down;  // encoded now: the down GEMM is launched right after the up/gate GEMM
  KDA_TRY(plan_plain_gemm(down, h, w_down, out, M, N, K));
  // 128 h columns per tile: gate|up pair in 256 accumulator columns (in CTA
  // pairs rank 0 loads the gate columns and rank 1 the up columns)
  if (M > gemm::BM) {
    Params p = base_params(M, N, K, 128, true);
    p.out = h;
    KDA_TRY((gemm::launch<256, false, true, gemm::EPI_SWIGLU, false, gemm::B_DUAL, 6, true>(
        ta, tg, ta, tu, th, p, gemm_err_word(), st)));
  } else {
    Params p = base_params(M, N, K, 128);
    p.out = h;
    KDA_TRY((gemm::launch<256, false, true, gemm::EPI_SWIGLU, false, gemm::B_DUAL, 4>(ta, tg, ta, tu, th, p,
                                                                                      gemm_err_word(), st)));
  }
  return launch_plain_gemm(down, st, /*pdl=*/true);
}

// t = x @ a has only ceil(M/128) output tiles when R <= 128 (32 at M = 4096):
// split its K over up to 8 parts so that the tiles x parts fill the GPU's 148
// SMs, each part at least 8 k-blocks, the parts dividing the k-blocks evenly.
// A pure function of the shape (the workspace size depends on it).
static int lora_k_split(int64_t M, int64_t K, int64_t R) {
  constexpr int kSms = 148;
  if (R > 128) return 1;
  const int64_t tiles = cdiv(M, gemm::BM);
  const int64_t kb = cdiv(K, gemm::BK);
  for (int s = 8; s >= 2; --s)
    if (kb % s == 0 && kb / s >= 8 && tiles * s <= kSms) return s;
  return 1;
}

// t = bf16(sum over parts of the fp32 partials), 8 elements per thread.
__global__ void __launch_bounds__(256) splitk_sum_bf16_kernel(const float* __restrict__ part, int parts,
                                                              int64_t n8, __nv_bfloat16* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  float4 a = reinterpret_cast<const float4*>(part)[2 * i];
  float4 b = reinterpret_cast<const float4*>(part)[2 * i + 1];
  for (int s = 1; s < parts; ++s) {
    const float4 c = reinterpret_cast<const float4*>(part + s * n8 * 8)[2 * i];
    const float4 d = reinterpret_cast<const float4*>(part + s * n8 * 8)[2 * i + 1];
    a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
    b.x += d.x; b.y += d.y; b.z += d.z; b.w += d.w;
  }
  reinterpret_cast<uint4*>(out)[i] =
      make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
}

extern "C" size_t kda_lora_workspace_size(int64_t M, int64_t K, int64_t N, int64_t R) {
  (void)N;
  if (M <= 0 || R <= 0) return 0;
  // t (bf16), then the fp32 partials of a split t = x @ a
  const int ks = lora_k_split(M, K, R);
  return align256(static_cast<size_t>(M) * R * 2) + (ks > 1 ? static_cast<size_t>(ks) * M * R * 4 : 0);
}

extern "C" kda_status kda_lora_bf16(const void* x, const void* w, const void* a, const void* b, void* out, int64_t M,
                                    int64_t K, int64_t N, int64_t R, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  const char* op = "lora";
  KDA_TRY(check_dims(op, M, K, N));
  KDA_CHECK_ARG(R > 0 && R <= 4096, "%s: bad rank R=%lld", op, (long long)R);
  KDA_CHECK_ARG(x && w && a && b && out, "%s: null pointer", op);
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0 && R % 8 == 0, "%s: K, N and R must be multiples of 8", op);
  KDA_CHECK_SUPPORTED(al16(x) && al16(w) && al16(a) && al16(b) && al16(out), "%s: pointers must be 16-byte aligned",
                      op);
  const size_t need = kda_lora_workspace_size(M, K, N, R);
  KDA_CHECK_ARG(workspace && workspace_bytes >= need, "%s: workspace of %zu bytes required, got %zu", op, need,
                workspace_bytes);
  KDA_CHECK_SUPPORTED(al16(workspace), "%s: workspace must be 16-byte aligned", op);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* t = workspace;
  // t = x @ a (M, R), kept in bf16
  const int ks = lora_k_split(M, K, R);
  if (ks > 1) {
    // split K: fp32 partials per part, then their sum as bf16
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256(static_cast<size_t>(M) * R * 2));
    CUtensorMap tx1, ta1;
    KDA_TRY(tmap2(&tx1, x, K, M, K, 128));
    KDA_TRY(tmap2(&ta1, a, R, K, R, 64));
    Params p1 = base_params(M, R, K, 128);
    p1.k_blocks /= ks;
    p1.k_split = ks;
    p1.out = part;
    KDA_TRY((gemm::launch<128, false, true, gemm::EPI_F32, false, gemm::B_SINGLE, 6>(tx1, ta1, tx1, ta1, tx1, p1,
                                                                                     gemm_err_word(), st)));
    const int64_t n8 = M * R / 8;
    splitk_sum_bf16_kernel<<<static_cast<unsigned>(cdiv(n8, 256)), 256, 0, st>>>(part, ks, n8,
                                                                                 static_cast<__nv_bfloat16*>(t));
    KDA_TRY(launch_status("splitk_sum_bf16_kernel"));
  } else {
    KDA_TRY(plain_gemm(x, a, t, M, K, R, st));
  }
  // out = [x | t] @ [w ; b]: one accumulator, K-extended by R
  CUtensorMap tx, tw, tt, tb;
  KDA_TRY(tmap2(&tx, x, K, M, K, 128));
  KDA_TRY(tmap2(&tw, w, N, K, N, 64));
  KDA_TRY(tmap2(&tt, t, R, M, R, 128));
  KDA_TRY(tmap2(&tb, b, N, R, N, 64));
  CUtensorMap to;
  KDA_TRY(tmap_out2(&to, out, N, M, N));
  const bool pair = M > gemm::BM;
  Params p = base_params(M, N, K, 256, pair);
  p.k_blocks2 = cdiv(R, gemm::BK);
  p.out = out;
  if (pair)
    return gemm::launch<256, false, true, gemm::EPI_BF16, false, gemm::B_KEXT, 6, true>(tx, tw, tt, tb, to, p,
                                                                                        gemm_err_word(), st);
  return gemm::launch<256, false, true, gemm::EPI_BF16, false, gemm::B_KEXT, 4>(tx, tw, tt, tb, to, p,
                                                                                gemm_err_word(), st);
}

extern "C" kda_status kda_bmm_softmax_bf16(const void* lhs, const void* rhs, void* out, int64_t batch, int64_t M,
                                           int64_t K, int64_t N, void* stream) {
  KDA_TRY(check_dims("bmm_softmax", M, K, N));
  KDA_CHECK_ARG(batch > 0 && batch < 65536, "bmm_softmax: bad batch %lld", (long long)batch);
  KDA_CHECK_ARG(lhs && rhs && out, "bmm_softmax: null pointer");
  KDA_CHECK_SUPPORTED(K % 8 == 0 && N % 8 == 0, "bmm_softmax: K (%lld) and N (%lld) must be multiples of 8",
                      (long long)K, (long long)N);
  KDA_CHECK_SUPPORTED(al16(lhs) && al16(rhs) && al16(out), "bmm_softmax: pointers must be 16-byte aligned");
  CUtensorMap ta, tb;
  KDA_TRY(tmap3(&ta, lhs, K, M, K, batch, M * K, 128));
  KDA_TRY(tmap3(&tb, rhs, N, K, N, batch, K * N, 64));
  CUtensorMap to;
  KDA_TRY(tmap_out3(&to, out, N, M, N, batch, M * N));
  Params p = base_params(M, N, K, 256);
  p.batch = static_cast<int>(batch);
  p.out = out;
  p.out_bstride = M * N;
  // two or more column tiles: split each row block's columns over a CTA pair
  if (p.n_tiles >= 2)
    return gemm::launch<256, false, true, gemm::EPI_SOFTMAX, true, gemm::B_SINGLE, 3, false, true>(
        ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
  return gemm::launch<256, false, true, gemm::EPI_SOFTMAX, true, gemm::B_SINGLE, 3>(
      ta, tb, ta, tb, to, p, gemm_err_word(), static_cast<cudaStream_t>(stream));
}
