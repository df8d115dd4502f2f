// Library-level C ABI: status strings, error messages, the device error
// words, and host-side TMA descriptor encoding.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace kda {

static thread_local char t_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

kda_status launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return KDA_CUDA_ERROR;
  }
  return KDA_OK;
}

int num_sms() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

static std::mutex& readers_mu() {
  static std::mutex m;
  return m;
}
static std::vector<err_reader_fn>& readers() {
  static std::vector<err_reader_fn> v;
  return v;
}
void register_err_reader(err_reader_fn fn) {
  std::lock_guard<std::mutex> g(readers_mu());
  readers().push_back(fn);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly (it loads on machines without a GPU).
typedef CUresult (*encode_tiled_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static encode_tiled_fn get_encode() {
  static encode_tiled_fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<encode_tiled_fn>(p);
  });
  return fn;
}

kda_status make_tmap_bf16(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides_bytes, const uint32_t* box) {
  return make_tmap_bf16_sw(out, base, rank, dims, strides_bytes, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

static kda_status make_tmap_sw(CUtensorMap* out, CUtensorMapDataType dt, const void* base, int rank,
                               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                               CUtensorMapSwizzle swizzle);
kda_status make_tmap_bf16_sw(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  return make_tmap_sw(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box, swizzle);
}
kda_status make_tmap_f32_sw(CUtensorMap* out, const void* base, int rank, const uint64_t* dims,
                            const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  return make_tmap_sw(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rank, dims, strides_bytes, box, swizzle);
}
static kda_status make_tmap_sw(CUtensorMap* out, CUtensorMapDataType dt, const void* base, int rank,
                               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                               CUtensorMapSwizzle swizzle) {
  encode_tiled_fn enc = get_encode();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable (driver entry point lookup failed)");
    return KDA_CUDA_ERROR;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
    set_error("TMA base pointer %p is not 16-byte aligned", base);
    return KDA_UNSUPPORTED;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i > 0) {
      if (strides_bytes[i - 1] % 16 != 0) {
        set_error("TMA stride %llu bytes is not a multiple of 16", (unsigned long long)strides_bytes[i - 1]);
        return KDA_UNSUPPORTED;
      }
      gstride[i - 1] = strides_bytes[i - 1];
    }
  }
  CUresult r = enc(out, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                   gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    return KDA_UNSUPPORTED;
  }
  return KDA_OK;
}

}  // namespace kda

extern "C" {

int kda_abi_version(void) { return KDA_ABI_VERSION; }

const char* kda_status_string(kda_status s) {
  switch (s) {
    case KDA_OK: return "KDA_OK";
    case KDA_INVALID_ARG: return "KDA_INVALID_ARG";
    case KDA_UNSUPPORTED: return "KDA_UNSUPPORTED";
    case KDA_CUDA_ERROR: return "KDA_CUDA_ERROR";
    case KDA_TIMEOUT: return "KDA_TIMEOUT";
  }
  return "KDA_UNKNOWN_STATUS";
}

const char* kda_last_error(void) { return kda::t_err; }

kda_status kda_device_error(unsigned* word, int clear) {
  if (!word) {
    kda::set_error("kda_device_error: null output pointer");
    return KDA_INVALID_ARG;
  }
  unsigned acc = 0;
  std::vector<kda::err_reader_fn> rs;
  {
    std::lock_guard<std::mutex> g(kda::readers_mu());
    rs = kda::readers();
  }
  for (auto fn : rs) {
    unsigned w = 0;
    cudaError_t e = fn(&w, clear);
    if (e != cudaSuccess) {
      kda::set_error("kda_device_error: %s", cudaGetErrorString(e));
      return KDA_CUDA_ERROR;
    }
    acc |= w;
  }
  *word = acc;
  if (acc != 0) {
    kda::set_error("a kernel reported an expired wait (device error word 0x%x)", acc);
    return KDA_TIMEOUT;
  }
  return KDA_OK;
}

}  // extern "C"
