// Flash attention with a bf16 v for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: plugins whose host framework owns every byte of device memory
// and exposes no allocator to them, and processes that must not allocate after start-up (real-time services with a
// fixed memory plan).  h3b_flash_attn_fwd_bf16v needs, for a bf16 v, an f16 copy of v and control words that its
// caller allocates, and a device status word that the library allocates on first use.  h3b_flash_attn_fwd_noalloc
// needs none of them: the f16 copy of v, the control words and a status word of its own live in one file-scope
// device array, g_scratch, of fixed size (H3B_NOALLOC_SCRATCH_BYTES).  Every GPU that loads the library holds that
// array until the process exits.
//
// Per call (all on the caller's stream), exactly as h3b_flash_attn_fwd_bf16v: clear the control words, convert the
// valid rows of v to f16 into the array (raising the range flag if a finite value overflows f16), run the f16 P.V
// attention kernel unless the flag is set, and only if it is set, convert again with a power-of-two scale per
// (head, column) and run the f16 P.V kernel on that copy.  The result is therefore always computed.  A device-side wait that gives up is recorded in the array's status
// word, which stays set (and makes later calls on that device skip their work) until h3b_noalloc_status() reads and
// clears it.
#include <mutex>

#include "common.cuh"

namespace h3b {
namespace attn {
// attention.cu: the bf16-v attention with caller-supplied scratch
int bf16v_with_scratch(const char* who, const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                       int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o, int64_t o_tok,
                       int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv, int32_t heads, int32_t head_dim,
                       float scale, int64_t max_v16, int (*scratch)(void** v16, void** ctl, int** status),
                       cudaStream_t st);
}  // namespace attn

namespace noalloc {

// control words first (the attention's: range flag at +0, column maxima from +16; this file's status word at +4,
// in the bytes the attention leaves alone), then the f16 copy of v
constexpr int64_t kControlBytes = H3B_NOALLOC_CTL_BYTES;
static_assert(kControlBytes % 256 == 0 && kControlBytes >= H3B_ATTN_CTL_BYTES(H3B_NOALLOC_MAX_HEADS),
              "control area");
constexpr int64_t kMaxVElems = H3B_NOALLOC_MAX_V_ELEMS;
constexpr int64_t kScratchBytes = kControlBytes + 2 * kMaxVElems;
static_assert(kScratchBytes == H3B_NOALLOC_SCRATCH_BYTES, "scratch size must match the header");

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

struct DeviceState {
  unsigned char* base = nullptr;  // device address of g_scratch on that device
};
static DeviceState g_state[64];
static std::mutex g_mu;

// Once per device, with that device current: the array's device address (host code may not use the symbol itself).
static int setup(int dev, unsigned char** base) {
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_state[dev];
  if (st.base == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "flash_attn_noalloc: cudaGetSymbolAddress(g_scratch)");
    st.base = static_cast<unsigned char*>(ptr);
  }
  *base = st.base;
  return H3B_OK;
}

static int current_device(const char* who, int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, who);
  if (*dev < 0 || *dev >= 64) return fail(H3B_EUNSUPPORTED, "%s: device index %d", who, *dev);
  return H3B_OK;
}

}  // namespace noalloc
}  // namespace h3b

// the array's parts on the current device (looked up on the first call there)
static int noalloc_scratch(void** v16, void** ctl, int** status) {
  using namespace h3b::noalloc;
  int dev = 0;
  int rc = current_device("flash_attn_noalloc: cudaGetDevice", &dev);
  if (rc) return rc;
  unsigned char* base = nullptr;
  rc = setup(dev, &base);
  if (rc) return rc;
  *ctl = base;
  *status = reinterpret_cast<int*>(base + 4);
  *v16 = base + kControlBytes;
  return H3B_OK;
}

extern "C" int h3b_flash_attn_fwd_noalloc(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                          int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o,
                                          int64_t o_tok, int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                          int32_t heads, int32_t head_dim, float scale, h3b_stream_t stream) {
  return h3b::attn::bf16v_with_scratch("flash_attn_noalloc", q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, o,
                                       o_tok, o_head, s_q, s_kv, valid_kv, heads, head_dim, scale,
                                       h3b::noalloc::kMaxVElems, noalloc_scratch,
                                       reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_noalloc_status(void) {
  using namespace h3b::noalloc;
  int dev = 0;
  int rc = current_device("noalloc_status: cudaGetDevice", &dev);
  if (rc) return rc;
  unsigned char* base = nullptr;
  rc = setup(dev, &base);
  if (rc) return rc;
  // the calls whose status this reads may run on any stream of the device
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return h3b::cuda_fail(e, "noalloc_status: cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, base + 4, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return h3b::cuda_fail(e, "noalloc_status: reading the status word");
  if (v != 0) {
    e = cudaMemset(base + 4, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return h3b::cuda_fail(e, "noalloc_status: clearing the status word");
    h3b::set_error("noalloc status word held %d (%s)", v, h3b_status_string(v));
  }
  return v;
}
