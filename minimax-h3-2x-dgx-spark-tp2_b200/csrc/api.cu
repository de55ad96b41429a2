// Host-side plumbing of the C ABI: error strings, the per-device status word that bounded device waits write,
// TMA descriptor encoding through the runtime's driver entry point, and small device queries.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"

namespace h3b {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
  return H3B_ECUDA;
}

static constexpr int kMaxDevices = 64;
static int* g_status[kMaxDevices] = {nullptr};
static std::mutex g_status_mu;
static uint64_t g_timeout_ns = 4000000000ull;

int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_status[dev] = p;
  }
  return g_status[dev];
}

uint64_t wait_timeout_ns() { return g_timeout_ns; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// dims/strides innermost first; strides_bytes has rank-1 entries (dimension 1..rank-1)
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return fail(H3B_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box),
                  elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(H3B_ECUDA, "cuTensorMapEncodeTiled failed (%d): rank %u dims %llu x %llu", static_cast<int>(r), rank,
                (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 1));
  return H3B_OK;
}

int num_sms() {
  static int cached[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace h3b

extern "C" {

int h3b_abi_version(void) { return 4; }

const char* h3b_status_string(int status) {
  switch (status) {
    case H3B_OK: return "ok";
    case H3B_EINVAL: return "invalid argument";
    case H3B_EALIGN: return "unsupported alignment";
    case H3B_EUNSUPPORTED: return "unsupported configuration";
    case H3B_ECUDA: return "CUDA error";
    case H3B_ETIMEOUT: return "device wait timed out";
    case H3B_ERANGE: return "value out of range for the requested path";
    default: return "unknown status";
  }
}

const char* h3b_last_error(void) { return h3b::g_last_error; }

int h3b_device_status(void) {
  int* w = h3b::device_status_word();
  if (w == nullptr) return h3b::fail(H3B_ECUDA, "no device status word");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return h3b::cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return h3b::cuda_fail(e, "reading the device status word");
  if (v != 0) {
    cudaMemset(w, 0, sizeof(int));
    cudaDeviceSynchronize();
    h3b::set_error("device status word held %d (%s)", v, h3b_status_string(v));
  }
  return v;
}

int h3b_set_wait_timeout_ns(uint64_t ns) {
  if (ns < 1000000ull) return h3b::fail(H3B_EINVAL, "wait timeout below 1 ms");
  h3b::g_timeout_ns = ns;
  return H3B_OK;
}

}  // extern "C"
