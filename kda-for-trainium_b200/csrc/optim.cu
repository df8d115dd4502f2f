// The optimizer step around the adamw operator: a multi-tensor AdamW (one
// launch updates a list of parameter tensors and their moments in place) and a
// ZeRO-1 step that fuses the gradient reduce-scatter, the AdamW update of this
// rank's shard and the parameter all-gather into one kernel over NVLink peer
// memory (CUDA IPC mappings of every rank's flat gradient and parameter
// buffers).  Peer access is plain loads and stores: no multicast, no device
// spin-waits -- the host orders the step with stream-ordered collectives.
#include <climits>
#include <cmath>
#include <cstring>

#include "common.cuh"

#define KDA_TRY(expr)            \
  do {                           \
    kda_status _s = (expr);      \
    if (_s != KDA_OK) return _s; \
  } while (0)

namespace kda {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;                              // float4s per thread per block
constexpr int64_t kChunk = int64_t(kThreads) * kVecPerThread * 4;  // elements per block
constexpr int kMaxTensors = 48;
constexpr int kMaxPeers = 8;

// AdamW with decoupled weight decay and bias correction, the scalars folded on
// the host in double:  c1 = 1 - beta1, c2 = 1 - beta2, wdlr = lr * wd,
// step_size = lr / (1 - beta1^t), bc2 = 1 / (1 - beta2^t).  The expression
// order is the reference's (workspaces/adamw/runs/adamw_v1.py:5-11 spec):
// theta' = (theta - wdlr * theta) - step_size * m' / (sqrt(v' * bc2) + eps).
struct AdamHp {
  float b1, c1, b2, c2, wdlr, step_size, bc2, eps;
};

struct Upd {
  float th, m, v;
};
__device__ __forceinline__ Upd adam_step(const AdamHp& h, float th, float g, float m, float v) {
  Upd o;
  o.m = h.b1 * m + h.c1 * g;
  o.v = h.b2 * v + h.c2 * g * g;
  const float den = sqrtf(o.v * h.bc2) + h.eps;
  o.th = (th - h.wdlr * th) - h.step_size * o.m / den;
  return o;
}

struct MultiArgs {
  float* th[kMaxTensors];
  const float* g[kMaxTensors];
  float* m[kMaxTensors];
  float* v[kMaxTensors];
  int64_t n[kMaxTensors];
  int block0[kMaxTensors + 1];  // first block of each tensor; block0[count] = grid size
  int count;
  AdamHp hp;
};

__device__ __forceinline__ bool al16d(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One block = kChunk consecutive elements of one tensor.
__global__ void __launch_bounds__(kThreads) adamw_multi_kernel(const __grid_constant__ MultiArgs a) {
  const int b = blockIdx.x;
  int lo = 0, hi = a.count - 1;  // last t with block0[t] <= b
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.block0[mid] <= b) lo = mid; else hi = mid - 1;
  }
  const int t = lo;
  float* th = a.th[t];
  const float* g = a.g[t];
  float* m = a.m[t];
  float* v = a.v[t];
  const int64_t n = a.n[t];
  const int64_t start = static_cast<int64_t>(b - a.block0[t]) * kChunk;
  const int64_t end = start + kChunk < n ? start + kChunk : n;
  if (al16d(th) && al16d(g) && al16d(m) && al16d(v)) {
    const int64_t full4 = end / 4;  // float4s wholly inside [0, end)
#pragma unroll
    for (int u = 0; u < kVecPerThread; ++u) {
      const int64_t i4 = start / 4 + u * kThreads + threadIdx.x;
      if (i4 >= full4) break;
      const float4 t4 = reinterpret_cast<const float4*>(th)[i4];
      const float4 g4 = reinterpret_cast<const float4*>(g)[i4];
      const float4 m4 = reinterpret_cast<const float4*>(m)[i4];
      const float4 v4 = reinterpret_cast<const float4*>(v)[i4];
      const Upd x = adam_step(a.hp, t4.x, g4.x, m4.x, v4.x);
      const Upd y = adam_step(a.hp, t4.y, g4.y, m4.y, v4.y);
      const Upd z = adam_step(a.hp, t4.z, g4.z, m4.z, v4.z);
      const Upd w = adam_step(a.hp, t4.w, g4.w, m4.w, v4.w);
      reinterpret_cast<float4*>(th)[i4] = make_float4(x.th, y.th, z.th, w.th);
      reinterpret_cast<float4*>(m)[i4] = make_float4(x.m, y.m, z.m, w.m);
      reinterpret_cast<float4*>(v)[i4] = make_float4(x.v, y.v, z.v, w.v);
    }
    // the tensor's last 1-3 elements (only in its last block)
    const int64_t i = full4 * 4 + threadIdx.x;
    if (i >= start && i < end) {
      const Upd x = adam_step(a.hp, th[i], g[i], m[i], v[i]);
      th[i] = x.th, m[i] = x.m, v[i] = x.v;
    }
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += kThreads) {
      const Upd x = adam_step(a.hp, th[i], g[i], m[i], v[i]);
      th[i] = x.th, m[i] = x.m, v[i] = x.v;
    }
  }
}

struct ZeroArgs {
  const float* grad[kMaxPeers];  // every rank's flat gradient buffer (this rank's own included)
  float* param[kMaxPeers];       // every rank's flat parameter buffer
  float* m;                      // this rank's moments for its shard (local)
  float* v;
  int64_t off, len;              // this rank's shard [off, off + len) of the flat buffers
  int world, rank;
  float grad_scale;              // 1 / world: the reduce-scatter averages
  AdamHp hp;
};

// ZeRO-1 step for this rank's shard: g = scale * sum_r grad_r[off + i] (peer
// loads, ranks summed in order 0..world-1), AdamW on param_rank / m / v, the
// new parameter stored into every rank's buffer (peer stores).  off and len
// are multiples of 4 and every buffer is 16-byte aligned (checked on the host).
__global__ void __launch_bounds__(kThreads) zero1_adamw_kernel(const __grid_constant__ ZeroArgs a) {
  const int64_t n4 = a.len / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i4 = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i4 < n4; i4 += stride) {
    const int64_t e4 = a.off / 4 + i4;
    float4 gs = reinterpret_cast<const float4*>(a.grad[0])[e4];
    for (int r = 1; r < a.world; ++r) {
      const float4 q = reinterpret_cast<const float4*>(a.grad[r])[e4];
      gs.x += q.x, gs.y += q.y, gs.z += q.z, gs.w += q.w;
    }
    gs.x *= a.grad_scale, gs.y *= a.grad_scale, gs.z *= a.grad_scale, gs.w *= a.grad_scale;
    const float4 t4 = reinterpret_cast<const float4*>(a.param[a.rank])[e4];
    const float4 m4 = reinterpret_cast<const float4*>(a.m)[i4];
    const float4 v4 = reinterpret_cast<const float4*>(a.v)[i4];
    const Upd x = adam_step(a.hp, t4.x, gs.x, m4.x, v4.x);
    const Upd y = adam_step(a.hp, t4.y, gs.y, m4.y, v4.y);
    const Upd z = adam_step(a.hp, t4.z, gs.z, m4.z, v4.z);
    const Upd w = adam_step(a.hp, t4.w, gs.w, m4.w, v4.w);
    reinterpret_cast<float4*>(a.m)[i4] = make_float4(x.m, y.m, z.m, w.m);
    reinterpret_cast<float4*>(a.v)[i4] = make_float4(x.v, y.v, z.v, w.v);
    const float4 nt = make_float4(x.th, y.th, z.th, w.th);
    for (int r = 0; r < a.world; ++r) reinterpret_cast<float4*>(a.param[r])[e4] = nt;
  }
  // make the peer stores visible system-wide before the host's next
  // stream-ordered collective tells the other ranks this step is done
  __threadfence_system();
}

// Hyperparameters arrive in double (as a Python optimizer holds them), so
// 1 - beta and the bias corrections are exact before the one rounding to fp32.
kda_status make_hp(AdamHp* h, double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step) {
  KDA_CHECK_ARG(step >= 1, "adamw: step (%lld) must be >= 1", (long long)step);
  KDA_CHECK_ARG(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0, "adamw: betas must lie in [0, 1)");
  KDA_CHECK_ARG(lr >= 0.0 && eps >= 0.0 && weight_decay >= 0.0, "adamw: lr, eps and weight_decay must be >= 0");
  h->b1 = static_cast<float>(beta1);
  h->b2 = static_cast<float>(beta2);
  h->c1 = static_cast<float>(1.0 - beta1);
  h->c2 = static_cast<float>(1.0 - beta2);
  h->wdlr = static_cast<float>(lr * weight_decay);
  h->step_size = static_cast<float>(lr / (1.0 - std::pow(beta1, static_cast<double>(step))));
  h->bc2 = static_cast<float>(1.0 / (1.0 - std::pow(beta2, static_cast<double>(step))));
  h->eps = static_cast<float>(eps);
  return KDA_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuMemGetAddressRange through the runtime's driver entry point (the library
// does not link libcuda).
typedef CUresult (*addr_range_fn)(CUdeviceptr*, size_t*, CUdeviceptr);
addr_range_fn get_addr_range() {
  // resolved once; a function-local static's initialisation is thread-safe
  static const addr_range_fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<addr_range_fn>(p);
    return static_cast<addr_range_fn>(nullptr);
  }();
  return fn;
}

}  // namespace
}  // namespace kda

using namespace kda;

extern "C" kda_status kda_adamw_multi_f32(float* const* theta, const float* const* g, float* const* m,
                                          float* const* v, const int64_t* n, int count, double lr, double beta1,
                                          double beta2, double eps, double weight_decay, int64_t step,
                                          void* stream) {
  KDA_CHECK_ARG(count >= 0, "adamw_multi: count = %d < 0", count);
  if (count == 0) return KDA_OK;
  KDA_CHECK_ARG(theta && g && m && v && n, "adamw_multi: null list");
  MultiArgs a{};
  KDA_TRY(make_hp(&a.hp, lr, beta1, beta2, eps, weight_decay, step));
  for (int i = 0; i < count; ++i) {
    KDA_CHECK_ARG(n[i] >= 0, "adamw_multi: tensor %d has %lld elements", i, (long long)n[i]);
    KDA_CHECK_ARG(n[i] == 0 || (theta[i] && g[i] && m[i] && v[i]), "adamw_multi: null pointer in tensor %d", i);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int i = 0;
  while (i < count) {
    // pack up to kMaxTensors non-empty tensors (and < 2^31 blocks) into one launch
    int k = 0;
    int64_t blocks = 0;
    for (; i < count && k < kMaxTensors; ++i) {
      if (n[i] == 0) continue;
      const int64_t nb = (n[i] + kChunk - 1) / kChunk;
      if (k > 0 && blocks + nb > INT32_MAX) break;
      KDA_CHECK_SUPPORTED(nb <= INT32_MAX, "adamw_multi: tensor %d too large", i);
      a.th[k] = theta[i];
      a.g[k] = g[i];
      a.m[k] = m[i];
      a.v[k] = v[i];
      a.n[k] = n[i];
      a.block0[k] = static_cast<int>(blocks);
      blocks += nb;
      ++k;
    }
    if (k == 0) break;
    a.count = k;
    a.block0[k] = static_cast<int>(blocks);
    adamw_multi_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(a);
    KDA_TRY(launch_status("adamw_multi_kernel"));
  }
  return KDA_OK;
}

extern "C" size_t kda_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" kda_status kda_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  KDA_CHECK_ARG(ptr && handle && offset, "ipc_export: null pointer");
  addr_range_fn range = get_addr_range();
  KDA_CHECK_SUPPORTED(range != nullptr, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("ipc_export: pointer is not device memory");
    return KDA_INVALID_ARG;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    set_error("ipc_export: cudaIpcGetMemHandle failed (%s)", cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return KDA_OK;
}

extern "C" kda_status kda_ipc_open(const void* handle, int64_t offset, void** ptr) {
  KDA_CHECK_ARG(handle && ptr && offset >= 0, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("ipc_open: cudaIpcOpenMemHandle failed (%s)", cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  *ptr = static_cast<uint8_t*>(base) + offset;
  return KDA_OK;
}

extern "C" kda_status kda_ipc_close(void* ptr, int64_t offset) {
  KDA_CHECK_ARG(ptr && offset >= 0, "ipc_close: bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (e != cudaSuccess) {
    set_error("ipc_close: cudaIpcCloseMemHandle failed (%s)", cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  return KDA_OK;
}

extern "C" kda_status kda_zero1_adamw_f32(const float* const* grads, float* const* params, int world, int rank,
                                          int64_t shard_off, int64_t shard_len, float* m, float* v, double lr,
                                          double beta1, double beta2, double eps, double weight_decay, int64_t step,
                                          void* stream) {
  KDA_CHECK_ARG(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "zero1_adamw: bad world/rank %d/%d",
                world, rank);
  KDA_CHECK_ARG(shard_off >= 0 && shard_len >= 0, "zero1_adamw: bad shard [%lld, +%lld)", (long long)shard_off,
                (long long)shard_len);
  KDA_CHECK_SUPPORTED(shard_off % 4 == 0 && shard_len % 4 == 0,
                      "zero1_adamw: shard offset and length must be multiples of 4");
  KDA_CHECK_ARG(grads && params && m && v, "zero1_adamw: null pointer");
  ZeroArgs a{};
  KDA_TRY(make_hp(&a.hp, lr, beta1, beta2, eps, weight_decay, step));
  for (int r = 0; r < world; ++r) {
    KDA_CHECK_ARG(grads[r] && params[r], "zero1_adamw: null buffer for rank %d", r);
    KDA_CHECK_SUPPORTED(al16(grads[r]) && al16(params[r]), "zero1_adamw: rank %d buffers must be 16-byte aligned", r);
    a.grad[r] = grads[r];
    a.param[r] = params[r];
  }
  KDA_CHECK_SUPPORTED(al16(m) && al16(v), "zero1_adamw: moments must be 16-byte aligned");
  if (shard_len == 0) return KDA_OK;
  a.m = m;
  a.v = v;
  a.off = shard_off;
  a.len = shard_len;
  a.world = world;
  a.rank = rank;
  a.grad_scale = 1.0f / static_cast<float>(world);
  const int64_t n4 = shard_len / 4;
  int64_t grid = (n4 + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;  // grid-stride beyond 8 CTAs per SM
  if (grid > cap) grid = cap;
  zero1_adamw_kernel<<<static_cast<unsigned>(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("zero1_adamw_kernel");
}
