// Shared device helpers for the kda-b200 kernels (sm_100a only).
//
// Hand-written inline PTX for the Blackwell data path: mbarriers, TMA bulk
// tensor copies, and the tcgen05 tensor-core / tensor-memory instructions.
// Every wait on an mbarrier is bounded in time: on expiry the waiting thread
// records a code in the translation unit's device error word and returns
// false, so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "kda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "kda-b200 kernels are written for sm_100a only"
#endif

namespace kda {

// Upper bound for any single mbarrier wait inside a kernel (nanoseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Device error codes written to the per-translation-unit error word.
enum : unsigned {
  kErrNone = 0,
  kErrWaitFull = 1,      // consumer gave up waiting for a TMA stage
  kErrWaitEmpty = 2,     // producer gave up waiting for a free stage
  kErrWaitAccum = 3,     // epilogue gave up waiting for the accumulator
  kErrWaitAccumFree = 4, // MMA issuer gave up waiting for a free accumulator
  kErrWaitDrain = 5,     // teardown gave up waiting for in-flight work
  kErrWaitPeer = 6,      // gave up waiting for another CTA's result
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// One arrival per warp once every lane has reached this point: __syncwarp
// orders the lanes' earlier shared-memory writes (each lane fences them to the
// async proxy first where an MMA or TMA reads them) and TMEM reads (each lane
// waited for them and issued tcgen05.fence::before_thread_sync) before lane
// 0's release-arrive.  The barrier then counts warps, not threads: 32 times
// fewer arrivals on the barrier's shared word.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31u) == 0u)
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `code` in *err) if the limit expires, or if another
// thread already recorded an error.  The error word (a global load of several
// hundred cycles) and the timer are polled only every 16th try: a phase that
// completes while the thread sits in that load would otherwise be seen late,
// and the waits of the pipelined kernels are on their critical path.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = 0;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0u) {
      if (*reinterpret_cast<volatile unsigned*>(err) != 0u) return false;
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        atomicCAS(err, 0u, code);
        return false;
      }
    }
  }
}

// Programmatic dependent launch.  pdl_trigger(): this CTA allows a kernel
// launched after it with programmatic stream serialization to start (the
// dependent launches once every CTA of this grid has triggered or exited).
// pdl_wait(): block until the preceding grid has completed and its memory
// operations are visible; a no-op when the kernel was launched normally.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Rendezvous of two warps (64 threads, both block) on named barrier ID;
// returns the AND of every participating thread's `ok`.  Used to hand work
// from a warp that waits on mbarriers to the warp that issues tcgen05.mma:
// a shared-memory access (an mbarrier wait included) from the issuing thread
// stalls behind its queued MMAs and idles the tensor core, a named barrier
// does not.  Both warps must execute the same number of these calls.
template <int ID>
__device__ __forceinline__ bool go_barrier64(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, 64, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(ok ? 1u : 0u), "n"(ID)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// Non-tensor bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on an mbarrier of this CTA.
__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// TMA bulk tensor stores (shared -> global), bulk-group completion.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most one committed group may still be reading its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ----------------------------------------------------------------- tcgen05
// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1").
//   K-major:  rows of 128 B, 8-row groups at `sbo` bytes, lbo unused (16 B).
//   MN-major: 64-element MN atoms at `lbo` bytes, 8-row K groups at `sbo`.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                              // D format: f32
         | (1u << 7)                            // A format: bf16
         | (1u << 10)                           // B format: bf16
         | (static_cast<uint32_t>(a_mn_major) << 15) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Whole-warp TMEM allocation; writes the TMEM base address to *dst (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base_lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns store (registers -> TMEM), mirror of the load above.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool elect_one_lane() { return (threadIdx.x & 31u) == 0u; }

// ------------------------------------------------------- CTA pairs (clusters)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 8-byte store into another CTA's shared memory (shared::cluster address).
__device__ __forceinline__ void st_cluster_f32x2(uint32_t cluster_addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(cluster_addr), "f"(a), "f"(b) : "memory");
}
// Bounded wait whose acquire covers writes that other CTAs of the cluster
// made before their release-arrive on this barrier.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned* err, unsigned code) {
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 15u) == 15u) {
      if (*reinterpret_cast<volatile unsigned*>(err) != 0u) return false;
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        atomicCAS(err, 0u, code);
        return false;
      }
    }
  }
}
// TMA load by either CTA of a pair whose completion bytes go to `bar_cluster`
// (the leader CTA's barrier, a shared::cluster address); the data lands in the issuing CTA only.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` (same offset) in every CTA of `mask` once this thread's
// issued pair MMAs are done.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void unpack_bf16x8(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// 2^x on the MUFU pipe (PTX ex2.approx.ftz.f32).
// max of three floats in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair of floats on the FMA / integer pipes only (no MUFU), so
// exponential-heavy loops can split their work between both pipes.
// x = n + f with n = rint(x) -- adding 1.5 * 2^23 leaves n in the low
// mantissa bits of t -- and f = x - n in [-0.5, 0.5]; 2^f comes from a
// degree-3 minimax fit of 2^f on [-0.5, 0.5] (coefficients fitted for this
// library; max relative error 7.5e-5 in fp32 for x in [-125, 8], checked by a
// float32 emulation in the tests), and 2^n is applied by adding n to the
// exponent field:
// (bits(t) << 23) equals (n << 23) modulo 2^32 because bits(1.5 * 2^23) has
// its low 22 bits clear.  x below -126 is clamped (result ~1.2e-38, zero for
// softmax weights).  For values rounded to bf16 (relative step 3.9e-3) right
// after, such as softmax weights.
__device__ __forceinline__ float2 exp2_poly2_lp(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 q = make_float2(0.0551716610789299f, 0.0551716610789299f);
  q = __ffma2_rn(q, f, make_float2(0.2426111400127411f, 0.2426111400127411f));
  q = __ffma2_rn(q, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  q = __ffma2_rn(q, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
  const uint32_t rx = __float_as_uint(q.x) + (__float_as_uint(t.x) << 23);
  const uint32_t ry = __float_as_uint(q.y) + (__float_as_uint(t.y) << 23);
  return make_float2(__uint_as_float(rx), __uint_as_float(ry));
}


}  // namespace kda

// ------------------------------------------------------------- host helpers
namespace kda {

// Thread-local message describing the last non-OK status of this thread.
void set_error(const char* fmt, ...);

#define KDA_CHECK_ARG(cond, ...)           \
  do {                                     \
    if (!(cond)) {                         \
      ::kda::set_error(__VA_ARGS__);       \
      return KDA_INVALID_ARG;              \
    }                                      \
  } while (0)

#define KDA_CHECK_SUPPORTED(cond, ...)     \
  do {                                     \
    if (!(cond)) {                         \
      ::kda::set_error(__VA_ARGS__);       \
      return KDA_UNSUPPORTED;              \
    }                                      \
  } while (0)

kda_status launch_status(const char* what);

int num_sms();

// Per-translation-unit device error words; each TU registers a reader.
typedef cudaError_t (*err_reader_fn)(unsigned* out, int clear);
void register_err_reader(err_reader_fn fn);

// 2-D / 3-D bf16 TMA descriptors with 128-byte swizzle (zero fill out of
// bounds).  dims/strides are innermost-first; strides in bytes (dims >= 1).
kda_status make_tmap_bf16(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box);
// Same with an explicit swizzle (CU_TENSOR_MAP_SWIZZLE_*).
kda_status make_tmap_bf16_sw(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);
kda_status make_tmap_f32_sw(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// RoPE table (S x 64 float2 cos/sin, angle = pos * theta^(-2i/128)) and the
// half-split rotation of [rows][128] bf16 rows at position (row / H) % S;
// inverse rotates by the negated angle.  Defined with the attention kernels.
kda_status rope_table(float2* tab, int64_t S, float theta, cudaStream_t st);
kda_status rope_rotate_rows(const __nv_bfloat16* x, __nv_bfloat16* out, const float2* tab, int64_t rows, int64_t S,
                            int64_t H, bool inverse, cudaStream_t st);

// The gqa_full forward (attention.cu), which also writes each query row's
// log2-sum-exp of the scaled scores into lse [B][QH][S] when lse is not null
// (the attention backward recomputes P from it).
// Flash-style attention backward (csrc/attn_bwd.cu): fp32 dq scratch bytes,
// and the kernel given rotated q, k (RoPE), dout (B, QH, S, 128), the
// forward's per-row lse and di = rowsum(dout * out).
size_t attn_backward_scratch_bytes(int64_t B, int64_t S, int64_t QH);
kda_status attn_backward_flash(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                               const __nv_bfloat16* dout, const float* lse, const float* di, __nv_bfloat16* dq,
                               __nv_bfloat16* dk, __nv_bfloat16* dv, float* dq32, int64_t B, int64_t S, int64_t QH,
                               int64_t KH, bool causal, cudaStream_t st);
kda_status gqa_forward(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S, int64_t QH,
                       int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd, void* workspace,
                       size_t workspace_bytes, float* lse, cudaStream_t st);

}  // namespace kda

// Define a per-TU device error word plus its host reader.
#define KDA_DEFINE_ERROR_WORD(tag)                                                     \
  static __device__ unsigned g_kda_err_##tag;                                          \
  static cudaError_t kda_read_err_##tag(unsigned* out, int clear) {                    \
    cudaError_t e = cudaMemcpyFromSymbol(out, g_kda_err_##tag, sizeof(unsigned));      \
    if (e == cudaSuccess && clear) {                                                   \
      unsigned z = 0;                                                                  \
      e = cudaMemcpyToSymbol(g_kda_err_##tag, &z, sizeof(unsigned));                   \
    }                                                                                  \
    return e;                                                                          \
  }                                                                                    \
  static unsigned* kda_err_ptr_##tag() {                                               \
    static std::atomic<unsigned*> cache[64] = {};                                      \
    int dev = 0;                                                                       \
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;    \
    unsigned* p = cache[dev].load(std::memory_order_acquire);                          \
    if (!p) {                                                                          \
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_kda_err_##tag) !=       \
          cudaSuccess)                                                                 \
        return nullptr;                                                                \
      cache[dev].store(p, std::memory_order_release);                                  \
    }                                                                                  \
    return p;                                                                          \
  }                                                                                    \
  static struct kda_err_reg_##tag {                                                    \
    kda_err_reg_##tag() { ::kda::register_err_reader(&kda_read_err_##tag); }           \
  } kda_err_reg_instance_##tag;
