/*
 * kda.h -- C ABI of the kda-b200 fused-operator library (libkda.so, sm_100a).
 *
 * One entry point per operator of the reference's NKIBench operator set
 * (Jerry2423/kda-for-trainium).  Each replaces the reference's per-operator
 * numpy `forward(...)` / NKI `kernel(...)` pair: arguments keep the forward's
 * parameter names and order, in natural (untiled) row-major layout, followed
 * by sizes, an optional caller-owned workspace, and the CUDA stream.
 * Around them: fp32-accuracy variants of the contractions (`*_f32`), the
 * training-side neighbours of the path (backward kernels, a multi-tensor
 * AdamW, a fused ZeRO-1 step over NVLink with its CUDA IPC helpers).
 *
 * Conventions
 *   - All pointers are device pointers owned by the caller.  bf16 tensors are
 *     passed as `const void*` (raw bf16 storage); fp32 tensors as float*.
 *   - Calls are asynchronous and stream-ordered on `stream` (a cudaStream_t,
 *     passed as void*; NULL = legacy default stream).  No call synchronises
 *     the device or allocates memory (kda_ipc_open maps a peer's existing
 *     allocation).  Calls are reentrant: concurrent calls
 *     on different streams or devices are safe when they do not share output
 *     or workspace buffers.
 *   - Every entry point returns a kda_status; no C++ exception crosses the
 *     ABI.  kda_last_error() gives the calling thread's detail message.
 *   - Kernels bound every internal wait; a wait that expires writes a code to
 *     a device error word that kda_device_error() reads after the stream is
 *     synchronised.
 *   - Ops that need scratch memory take (workspace, workspace_bytes); the
 *     required size comes from the matching *_workspace_size() query.
 */
#ifndef KDA_H_
#define KDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_ABI_VERSION 1

typedef enum kda_status {
  KDA_OK = 0,
  KDA_INVALID_ARG = 1,  /* null pointer, bad dimension, too-small workspace */
  KDA_UNSUPPORTED = 2,  /* shape / alignment outside the kernel's contract   */
  KDA_CUDA_ERROR = 3,   /* launch or driver failure (cudaGetLastError)       */
  KDA_TIMEOUT = 4       /* a bounded device wait expired (kda_device_error)  */
} kda_status;

/* ------------------------------------------------------------- library -- */
int kda_abi_version(void);
const char* kda_status_string(kda_status s);
/* Detail message of the last non-OK status returned on this thread. */
const char* kda_last_error(void);
/* Reads (and with clear != 0 resets) the OR of the device error words of the
 * current device.  *word == 0 means no kernel reported an expired wait.
 * Synchronous with respect to the device (cudaMemcpyFromSymbol). */
kda_status kda_device_error(unsigned* word, int clear);

/* ------------------------------------------------------ elementwise ops -- */

/* silu: y = x / (1 + exp(-x)), fp32, n elements.
 * Replaces silu forward(x) (prompts/_gen_prompts.py:19-33) and the NKI kernel
 * workspaces/silu/runs/silu_v3_s7.py:31-71. */
kda_status kda_silu_f32(const float* x, float* y, int64_t n, void* stream);

/* rope_single_freq_apply: half-split rotation over the leading axis.
 * x_in (d_head, s) row-major, cos/sin (d_head/2, s), out (d_head, s):
 *   out[:h] = x0*cos - x1*sin ; out[h:] = x0*sin + x1*cos   (h = d_head/2)
 * Replaces rope_single_freq_apply forward(x_in, cos, sin)
 * (workspaces/rope_single_freq_apply/runs/rope_v1.py:5-8, kernel :33). */
kda_status kda_rope_single_freq_apply_f32(const float* x_in, const float* cos, const float* sin, float* out,
                                          int64_t d_head, int64_t s, void* stream);

/* adamw: one AdamW step with the reference constants (lr 0.01, beta1 0.9,
 * beta2 0.999, weight decay 1e-5, eps 1e-8, bias-correction 1000 on v):
 *   m' = .9m + .1g ; v' = .999v + .001g^2 ;
 *   theta_out = theta - 1e-5 theta - .01 m'/(sqrt(1000 v') + 1e-8)
 * If update_state != 0, m and v are overwritten with m', v' (in place).
 * Replaces adamw forward(theta, g, m, v) (prompts/_gen_prompts.py:227-228,
 * workspaces/adamw/runs/adamw_v1.py:5-11; kernel adamw_v2_ch1824.py:51). */
kda_status kda_adamw_f32(const float* theta, const float* g, float* m, float* v, float* theta_out, int64_t n,
                         int update_state, void* stream);

/* adamw_multi: the AdamW step over a list of `count` fp32 tensors, in place
 * (theta, m, v updated; g read), one launch per 48 tensors.  Decoupled weight
 * decay and bias correction at `step` (>= 1):
 *   m' = b1 m + (1-b1) g ; v' = b2 v + (1-b2) g^2 ;
 *   theta' = (theta - lr wd theta) - lr/(1-b1^step) m' / (sqrt(v'/(1-b2^step)) + eps)
 * Hyperparameters in double.  lr 1e-3, betas (0.9, 0.999), eps 1e-8, wd 1e-2,
 * step 1 is exactly the adamw forward above (workspaces/adamw/runs/adamw_v1.py:5-11),
 * applied to many tensors at once: the multi-tensor form of the step that
 * follows it in training. */
kda_status kda_adamw_multi_f32(float* const* theta, const float* const* g, float* const* m, float* const* v,
                               const int64_t* n, int count, double lr, double beta1, double beta2, double eps,
                               double weight_decay, int64_t step, void* stream);

/* CUDA IPC for the ZeRO-1 step: export a device pointer as (handle, offset
 * into its allocation), open a peer's export in this process (mapped with
 * peer access; no multicast), close it again.  The handle is
 * kda_ipc_handle_size() bytes.  No reference counterpart: the reference has
 * no multi-device code (the plumbing of adamw's training-step neighbour). */
size_t kda_ipc_handle_size(void);
kda_status kda_ipc_export(const void* ptr, void* handle, int64_t* offset);
kda_status kda_ipc_open(const void* handle, int64_t offset, void** ptr);
kda_status kda_ipc_close(void* ptr, int64_t offset);

/* zero1_adamw: one fused ZeRO-1 step for this rank's shard [shard_off,
 * shard_off + shard_len) of flat fp32 buffers replicated on `world` ranks
 * (<= 8): g = (1/world) sum_r grads[r][shard] (peer loads), AdamW as
 * kda_adamw_multi_f32 on params[rank][shard] with this rank's moments m, v
 * (shard_len elements), and the new values stored into params[r][shard] of
 * every rank (peer stores).  grads / params hold every rank's buffer address
 * in this process (its own, and kda_ipc_open'ed peers).  shard_off and
 * shard_len multiples of 4, all buffers 16-byte aligned.  The caller orders
 * the step: every rank's gradients complete before any rank launches, and no
 * rank touches its buffers again until every rank's launch has completed
 * (e.g. a one-element all-reduce on the stream before and after).  The
 * reduce-scatter -> adamw -> all-gather around the adamw forward
 * (workspaces/adamw/runs/adamw_v1.py:5-11) as one kernel. */
kda_status kda_zero1_adamw_f32(const float* const* grads, float* const* params, int world, int rank,
                               int64_t shard_off, int64_t shard_len, float* m, float* v, double lr, double beta1,
                               double beta2, double eps, double weight_decay, int64_t step, void* stream);

/* ------------------------------------------------------ selective scan -- */

/* mamba: h_t = exp(dt_t * A) h_{t-1} + dt_t B_t x_t ; y_t = C_t . h_t + D x_t
 * fp32 state (h_0 = 0), d_state == 16.
 * Batched channels-last layout: delta (dt) and u (x) are (batch, seqlen,
 * d_inner) with element (b,t,d) at b*ld_b + t*ld_t + d*ld_d (element
 * strides); a (A) is (d_inner, 16) contiguous; b (B) and c (C) are
 * (batch, seqlen, 16) with element (b,t,n) at b*bc_ld_b + t*bc_ld_t + n*bc_ld_n;
 * D is (d_inner,) or NULL; y has the strides of delta.
 * u_bf16 != 0: u is bf16 storage, else fp32.  y_bf16 != 0: y is bf16, else fp32.
 * The reference's 2-D form -- delta, u (C, M); a (C, S); b, c (S, M) -- is
 * batch 1, ld_t = 1, ld_d = M, bc_ld_t = 1, bc_ld_n = M.
 * When batch * d_inner is too small to fill the GPU, time is split into
 * chunks scanned in parallel; their summaries need the workspace that
 * kda_mamba_scan_workspace_size() reports (0 bytes when no chunking is used).
 * Replaces mamba forward(delta, u, a, b, c) (workspaces/mamba/docs/
 * draft-phase1.md:22-29; kernel workspaces/mamba/runs/mamba_v4_s4unroll.py:8). */
size_t kda_mamba_scan_workspace_size(int64_t batch, int64_t seqlen, int64_t d_inner, int64_t d_state);
kda_status kda_mamba_scan(const void* delta, const void* u, const float* a, const float* b, const float* c,
                          const float* D, void* y, int64_t batch, int64_t seqlen, int64_t d_inner,
                          int64_t d_state, int64_t ld_b, int64_t ld_t, int64_t ld_d, int64_t bc_ld_b,
                          int64_t bc_ld_t, int64_t bc_ld_n, int u_bf16, int y_bf16, void* workspace,
                          size_t workspace_bytes, void* stream);

/* mamba_scan_noalloc: the same scan as kda_mamba_scan, for callers that
 * cannot allocate device memory -- a host binding that is handed only the
 * input and output buffers by its framework, or code that must not call
 * cudaMalloc because it can synchronise the device.  It has no counterpart in
 * the reference.  When the time axis is split into chunks, the chunk summaries
 * go to a fixed 1 MiB array that every GPU loading the library holds until
 * the process exits; shapes needing more (kda_mamba_scan_workspace_size() >
 * 1 MiB) are rejected with KDA_UNSUPPORTED.  The first call on each device
 * looks up that array's device address (cudaGetSymbolAddress), so make it
 * before any stream capture.  All calls share the array: calls that overlap
 * on the GPU (other streams, other threads) race and must be serialised by
 * the caller.  No memory is allocated or freed.  Arguments as kda_mamba_scan
 * without the workspace. */
kda_status kda_mamba_scan_noalloc(const void* delta, const void* u, const float* a, const float* b,
                                  const float* c, const float* D, void* y, int64_t batch, int64_t seqlen,
                                  int64_t d_inner, int64_t d_state, int64_t ld_b, int64_t ld_t, int64_t ld_d,
                                  int64_t bc_ld_b, int64_t bc_ld_t, int64_t bc_ld_n, int u_bf16, int y_bf16,
                                  void* stream);

/* ---------------------------------------------------------- contractions --
 * bf16 operands, fp32 accumulation in tensor memory (tcgen05), bf16 output
 * unless stated.  Row strides must be multiples of 16 bytes (TMA), and the
 * base pointers 16-byte aligned. */

/* matmul: out (M,N) = lhs (M,K) @ rhs (K,N).
 * Replaces matmul forward(lhs, rhs) (workspaces/matmul/runs/offline_bf16_split_sim.py:137-139;
 * kernel workspaces/matmul/runs/matmul_v3_bf16_split.py:11). */
kda_status kda_matmul_bf16(const void* lhs, const void* rhs, void* out, int64_t M, int64_t K, int64_t N,
                           void* stream);

/* matmul, fp32 in / fp32 out at fp32 accuracy on the bf16 tensor core: each
 * operand is split into bf16 hi + lo (in the workspace) and
 * out = hi.hi + hi.lo + lo.hi is accumulated in fp32 -- the reference's
 * bf16 split of fp32 operands (workspaces/matmul/runs/matmul_v3_bf16_split.py:14-24;
 * forward workspaces/matmul/runs/offline_bf16_split_sim.py:137-139). */
size_t kda_matmul_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_matmul_f32(const float* lhs, const float* rhs, float* out, int64_t M, int64_t K, int64_t N,
                          void* workspace, size_t workspace_bytes, void* stream);

/* transpose_matmul: out (M,N) = lhs^T @ rhs, lhs stored (K,M).
 * Replaces transpose_matmul forward(lhs, rhs)
 * (workspaces/transpose_matmul/runs/offline_bf16_split_sim.py:101-104; kernel
 * workspaces/transpose_matmul/runs/tmm_v3_mblk16_bf16_split.py:11). */
kda_status kda_transpose_matmul_bf16(const void* lhs, const void* rhs, void* out, int64_t M, int64_t K,
                                     int64_t N, void* stream);

/* transpose_matmul, fp32 in / fp32 out at fp32 accuracy: the bf16 hi + lo
 * split of kda_matmul_f32 with lhs (K,M) read MN-major
 * (workspaces/transpose_matmul/runs/tmm_v3_mblk16_bf16_split.py:11, the
 * reference's bf16-split kernel; forward
 * workspaces/transpose_matmul/runs/offline_bf16_split_sim.py:101-104). */
size_t kda_transpose_matmul_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_transpose_matmul_f32(const float* lhs, const float* rhs, float* out, int64_t M, int64_t K,
                                    int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* bmm: out[b] (M,N) = lhs[b] (M,K) @ rhs[b] (K,N), b < batch.
 * Replaces bmm forward(lhs, rhs) (workspaces/bmm/runs/offline_bf16_split_sim.py:102-117;
 * kernel workspaces/bmm/runs/bmm_v2.py:11). */
kda_status kda_bmm_bf16(const void* lhs, const void* rhs, void* out, int64_t batch, int64_t M, int64_t K,
                        int64_t N, void* stream);

/* bmm, fp32 in / fp32 out at fp32 accuracy: both operands split into bf16
 * hi + lo once for the whole batch, then one three-pass GEMM per entry
 * (forward workspaces/bmm/runs/offline_bf16_split_sim.py:102-104, whose
 * bf16-split product it reproduces). */
size_t kda_bmm_f32_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t N);
kda_status kda_bmm_f32(const float* lhs, const float* rhs, float* out, int64_t batch, int64_t M, int64_t K,
                       int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* bmm_softmax: out[b] = softmax over the last axis of lhs[b] @ rhs[b]
 * (max-shifted, fp32 scores and statistics, bf16 out).
 * Replaces bmm_softmax forward(lhs, rhs) (prompts/_gen_prompts.py:170-177;
 * kernel workspaces/bmm_softmax/runs/bmm_softmax_v4.py:11-27). */
kda_status kda_bmm_softmax_bf16(const void* lhs, const void* rhs, void* out, int64_t batch, int64_t M,
                                int64_t K, int64_t N, void* stream);

/* bmm_softmax, fp32 in / fp32 out at fp32 accuracy: kda_bmm_f32, then a
 * max-shifted fp32 row softmax in place (the spec's fp32 forward,
 * prompts/_gen_prompts.py:170-177). */
size_t kda_bmm_softmax_f32_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t N);
kda_status kda_bmm_softmax_f32(const float* lhs, const float* rhs, float* out, int64_t batch, int64_t M, int64_t K,
                               int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* rmsnorm_matmul: out = (x / sqrt(mean_k x^2 + eps) * g) @ w ; g may be NULL
 * (the reference: no gamma, eps = 0).  x (M,K), w (K,N), g (K,) fp32.
 * Replaces rmsnorm_matmul forward(x, w)
 * (workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:83-93; kernel
 * workspaces/rmsnorm_matmul/runs/rmsnorm_matmul_v4_bf16_split.py:11). */
size_t kda_rmsnorm_matmul_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_rmsnorm_matmul_bf16(const void* x, const void* w, const float* g, float eps, void* out, int64_t M,
                                   int64_t K, int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* rmsnorm_matmul, fp32 x / w / out at fp32 accuracy: a row kernel normalises
 * x in fp32 and writes the bf16 hi + lo split of the normalised rows, then the
 * three-pass split GEMM (the reference forward in fp32,
 * workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:83-93, and its
 * bf16-split kernel workspaces/rmsnorm_matmul/runs/rmsnorm_matmul_v4_bf16_split.py:11). */
size_t kda_rmsnorm_matmul_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_rmsnorm_matmul_f32(const float* x, const float* w, const float* g, float eps, float* out, int64_t M,
                                  int64_t K, int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* rmsnorm_matmul backward: the gradients of out = a @ w, a = x r g,
 * r = 1 / sqrt(mean_k x^2 + eps), given dy (M,N):
 *   dx (M,K) bf16 = r (dA g - xn mean_k(dA g xn)),  xn = x r,  dA = dy @ w^T (fp32)
 *   dw (K,N) bf16 = a^T @ dy  (a recomputed as the forward's bf16 operand)
 *   dg (K,)  fp32 = sum_m dA xn  (written iff g is given; deterministic order)
 * dy, x, w bf16; g fp32 or NULL.  The training-side caller of rmsnorm_matmul
 * forward (workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:83-93); the
 * reference has no backward (its operators are forward-only). */
size_t kda_rmsnorm_matmul_backward_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_rmsnorm_matmul_backward_bf16(const void* dy, const void* x, const void* w, const float* g, float eps,
                                            void* dx, void* dw, float* dg, int64_t M, int64_t K, int64_t N,
                                            void* workspace, size_t workspace_bytes, void* stream);

/* add_rmsnorm_matmul: a = x + z ; out = (a / sqrt(mean_k a^2 + eps) * g) @ w.
 * x, z (M,K) bf16, w (K,N) bf16, g (K,) fp32.
 * Replaces add_rmsnorm_matmul forward(x, w, eps, z, g)
 * (workspaces/add_rmsnorm_matmul/runs/offline_bf16_split_sim.py:97-106; kernel
 * workspaces/add_rmsnorm_matmul/runs/add_rmsnorm_matmul_v3_bf16_split.py:9). */
size_t kda_add_rmsnorm_matmul_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_add_rmsnorm_matmul_bf16(const void* x, const void* w, float eps, const void* z, const float* g,
                                       void* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* add_rmsnorm_matmul, fp32 x / z / w / out at fp32 accuracy (as
 * kda_rmsnorm_matmul_f32 on a = x + z;
 * workspaces/add_rmsnorm_matmul/runs/offline_bf16_split_sim.py:97-106). */
size_t kda_add_rmsnorm_matmul_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_add_rmsnorm_matmul_f32(const float* x, const float* w, float eps, const float* z, const float* g,
                                      float* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* matmul_add_rmsnorm: y = x @ w + z ; out = y * g / sqrt(mean_n y^2 + eps).
 * x (M,K), w (K,N), z (M,N) bf16; g (N,) fp32; out (M,N) bf16.
 * Replaces matmul_add_rmsnorm forward(x, w, eps, z, g)
 * (workspaces/matmul_add_rmsnorm/runs/offline_bf16_split_sim.py:111-115; kernel
 * workspaces/matmul_add_rmsnorm/runs/matmul_add_rmsnorm_v2_bf16_split.py:9). */
size_t kda_matmul_add_rmsnorm_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_matmul_add_rmsnorm_bf16(const void* x, const void* w, float eps, const void* z, const float* g,
                                       void* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* matmul_add_rmsnorm, fp32 in / out at fp32 accuracy: the three-pass split
 * GEMM writes x @ w into out, a row kernel adds z and normalises in place
 * (workspaces/matmul_add_rmsnorm/runs/offline_bf16_split_sim.py:111-115). */
size_t kda_matmul_add_rmsnorm_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_matmul_add_rmsnorm_f32(const float* x, const float* w, float eps, const float* z, const float* g,
                                      float* out, int64_t M, int64_t K, int64_t N, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* swiglu: out (M,K) = (silu(x @ w_gate) * (x @ w_up)) @ w_down.
 * x (M,K), w_up / w_gate (K,N), w_down (N,K), all bf16; the intermediate h
 * (M,N) is stored once in the workspace as bf16.
 * Replaces swiglu forward(x, w_up, w_down, w_gate)
 * (workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97; kernel
 * workspaces/swiglu/runs/swiglu_v3_mblock.py:47). */
size_t kda_swiglu_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_swiglu_bf16(const void* x, const void* w_up, const void* w_down, const void* w_gate, void* out,
                           int64_t M, int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                           void* stream);

/* swiglu, fp32 in / out at fp32 accuracy: [gate | up] in one three-pass GEMM
 * (fp32, in the workspace), h = silu(gate) * up in fp32 written as its bf16
 * hi + lo split, then h @ w_down (the reference forward with its fp32 h,
 * workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97). */
size_t kda_swiglu_f32_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_swiglu_f32(const float* x, const float* w_up, const float* w_down, const float* w_gate, float* out,
                          int64_t M, int64_t K, int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/* swiglu backward: the gradients of out = (silu(x w_gate) * (x w_up)) w_down
 * given dout (M,K): dx (M,K), dw_up / dw_gate (K,N), dw_down (N,K), all bf16
 * (fp32 accumulation; g = x w_gate and u = x w_up recomputed; N is d_ff):
 *   dh = dout w_down^T ; dg = dh u silu'(g) ; du = dh silu(g)
 *   dw_down = h^T dout ; dw_gate = x^T dg ; dw_up = x^T du ; dx = dg w_gate^T + du w_up^T
 * The training-side caller of swiglu forward
 * (workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97); the reference has no
 * backward. */
size_t kda_swiglu_backward_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_swiglu_backward_bf16(const void* dout, const void* x, const void* w_up, const void* w_down,
                                    const void* w_gate, void* dx, void* dw_up, void* dw_down, void* dw_gate,
                                    int64_t M, int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* swiglu forward of a training step: out as kda_swiglu_bf16 computes it, but
 * unfused -- g = x w_gate and u = x w_up (bf16, M x N) are written to the
 * caller's buffers, h = silu(g) * u (from the bf16 g, u) goes through the
 * workspace (kda_swiglu_gu_workspace_size()) into out = h w_down -- so that
 * kda_swiglu_backward_saved_bf16 need not recompute g and u.  Same reference
 * forward as kda_swiglu_bf16 (workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97);
 * the reference keeps no activations, so no counterpart for g and u. */
size_t kda_swiglu_gu_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_swiglu_gu_bf16(const void* x, const void* w_up, const void* w_down, const void* w_gate, void* out,
                              void* g, void* u, int64_t M, int64_t K, int64_t N, void* workspace,
                              size_t workspace_bytes, void* stream);

/* swiglu backward from the saved g and u of kda_swiglu_gu_bf16: the same
 * gradients as kda_swiglu_backward_bf16 without its two recomputing GEMMs
 * (smaller workspace, kda_swiglu_backward_saved_workspace_size()).  Same
 * reference caller as kda_swiglu_backward_bf16. */
size_t kda_swiglu_backward_saved_workspace_size(int64_t M, int64_t K, int64_t N);
kda_status kda_swiglu_backward_saved_bf16(const void* dout, const void* x, const void* w_up, const void* w_down,
                                          const void* w_gate, const void* g, const void* u, void* dx, void* dw_up,
                                          void* dw_down, void* dw_gate, int64_t M, int64_t K, int64_t N,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* lora: out (M,N) = x @ w + (x @ a) @ b ; x (M,K), w (K,N), a (K,R), b (R,N).
 * The low-rank product t = x @ a (M,R) is kept in the workspace as bf16 and
 * accumulated into the same tensor-memory accumulator as x @ w; for R <= 128
 * the workspace also holds the fp32 partials of a K-split t = x @ a.
 * Replaces lora forward(x, w, a, b)
 * (workspaces/lora/runs/offline_lora_bf16_split_sim.py:175-180; kernel
 * workspaces/lora/runs/lora_v3_bf16_split.py:11). */
size_t kda_lora_workspace_size(int64_t M, int64_t K, int64_t N, int64_t R);
kda_status kda_lora_bf16(const void* x, const void* w, const void* a, const void* b, void* out, int64_t M,
                         int64_t K, int64_t N, int64_t R, void* workspace, size_t workspace_bytes, void* stream);

/* lora, fp32 in / out at fp32 accuracy: t = x @ a in fp32, then one
 * three-pass GEMM of [x | t] @ [w ; b] over K + R (the reference forward,
 * workspaces/lora/runs/offline_lora_bf16_split_sim.py:175-180, with its fp32 t).
 * R must be a multiple of 8. */
size_t kda_lora_f32_workspace_size(int64_t M, int64_t K, int64_t N, int64_t R);
kda_status kda_lora_f32(const float* x, const float* w, const float* a, const float* b, float* out, int64_t M,
                        int64_t K, int64_t N, int64_t R, void* workspace, size_t workspace_bytes, void* stream);

/* gqa_full: grouped-query attention, head_dim 128.
 * q (B,S,QH,128), k/v (B,S,KH,128) bf16 (row-major, [B,S,H,D]); query head
 * h reads kv head h / (QH/KH).  out = softmax(q k^T / sqrt(128) [+causal
 * mask]) v, fp32 softmax / accumulation, bf16 out.
 * rope_theta > 0 applies the half-split rotary embedding (angle =
 * pos * rope_theta^(-2i/128)) to q and k first; rope_theta <= 0 disables it.
 * out_bshd != 0 writes out as (B,S,QH,128); 0 writes the reference order
 * (B,QH,S,128).  The workspace (kda_gqa_full_workspace_size() bytes,
 * 16-byte aligned, always required) receives a transposed copy of v and, with
 * RoPE, the rotated q and k.
 * Replaces gqa_full forward(q, k, v)
 * (workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124; kernel
 * workspaces/gqa_full/runs/gqa_full_v7a_exp_from_psum.py:16). */
size_t kda_gqa_full_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D, float rope_theta);
kda_status kda_gqa_full_bf16(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S,
                             int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd,
                             void* workspace, size_t workspace_bytes, void* stream);

/* gqa_full, fp32 q / k / v / out at fp32 accuracy, head by head: fp32 scores
 * from a three-pass split GEMM, a max-shifted fp32 row softmax (scale
 * 1/sqrt(D), optional causal mask) that writes the probabilities' split,
 * then P @ v_h.  Any D that is a multiple of 32; S a multiple of 8; no RoPE
 * (rope_theta must be <= 0).  The workspace holds the split q, k (transposed
 * per head), v and one head's scores and probabilities
 * (workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124). */
size_t kda_gqa_full_f32_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D);
kda_status kda_gqa_full_f32(const float* q, const float* k, const float* v, float* out, int64_t B, int64_t S,
                            int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd,
                            void* workspace, size_t workspace_bytes, void* stream);

/* gqa_full with the row statistics the backward needs: the same forward as
 * kda_gqa_full_bf16 (same workspace) that also writes lse [B][QH][S] fp32,
 * each query row's log2-sum-exp of the scaled scores (16-byte aligned).
 * The training-side forward of gqa_full forward(q, k, v)
 * (workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124); the
 * reference has no backward, so no counterpart for lse. */
kda_status kda_gqa_full_lse_bf16(const void* q, const void* k, const void* v, void* out, float* lse, int64_t B,
                                 int64_t S, int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta,
                                 int out_bshd, void* workspace, size_t workspace_bytes, void* stream);

/* gqa_full backward: the gradients of gqa_full (head_dim 128) given
 * dout in the reference order (B,QH,S,128) bf16: dq (B,S,QH,128) and dk, dv
 * (B,S,KH,128), bf16.  The forward runs again first (its output and each
 * row's log2-sum-exp into the workspace); di = rowsum(dout * out); then one
 * flash-style kernel per (batch, kv head, 128-key block) walks the query
 * blocks with P and dS only in shared memory:
 *   P = 2^(q k^T log2e / sqrt(128) - lse) [causal: 0 for keys after the query];
 *   dS = P (dout v^T - di) ; dq = dS k / sqrt(128) ; dk = dS^T q / sqrt(128) ;
 *   dv = P^T dout
 * rope_theta > 0: the forward's RoPE -- the backward runs on the rotated q, k
 * (recomputed in the workspace) and rotates dq, dk back by the negated angle.
 * S a multiple of 8.  The training-side caller of gqa_full forward
 * (workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124); the
 * reference has no backward. */
size_t kda_gqa_full_backward_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                            float rope_theta);
kda_status kda_gqa_full_backward_bf16(const void* dout, const void* q, const void* k, const void* v, void* dq,
                                      void* dk, void* dv, int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                      int causal, float rope_theta, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* gqa_full backward from a saved forward: as kda_gqa_full_backward_bf16, but
 * the forward's output `out` (reference order (B,QH,S,128) bf16, as written by
 * kda_gqa_full_lse_bf16 with out_bshd = 0) and its lse (B,QH,S fp32) are
 * passed in instead of recomputed -- the backward of a training step whose
 * forward kept them.  Smaller workspace (kda_gqa_full_backward_saved_
 * workspace_size()).  Same reference caller as kda_gqa_full_backward_bf16. */
size_t kda_gqa_full_backward_saved_workspace_size(int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D,
                                                  float rope_theta);
kda_status kda_gqa_full_backward_saved_bf16(const void* dout, const void* q, const void* k, const void* v,
                                            const void* out, const float* lse, void* dq, void* dk, void* dv,
                                            int64_t B, int64_t S, int64_t QH, int64_t KH, int64_t D, int causal,
                                            float rope_theta, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_H_ */
