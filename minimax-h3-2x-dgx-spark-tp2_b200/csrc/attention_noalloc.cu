// Flash attention with a bf16 v for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: plugins whose host framework owns every byte of device memory
// and exposes no allocator to them, and processes that must not allocate after start-up (real-time services with a
// fixed memory plan).  The regular entry point h3b_flash_attn_fwd
// needs, for a bf16 v, an f16 copy of v that its caller allocates, and a device status word that the library
// allocates on first use.  h3b_flash_attn_fwd_noalloc needs neither: the f16 copy of v, the overflow flag and the
// status word live in one file-scope device array, g_scratch, of fixed size (H3B_NOALLOC_SCRATCH_BYTES).  Every
// GPU that loads the library holds that array until the process exits.
//
// Per call (all on the caller's stream): clear the two control words, convert v to f16 into the array (raising the
// flag if a finite value overflows f16), run the f16 P.V attention kernel unless the flag is set, then the bf16 P.V
// kernel only if it is set.  The result is therefore always computed, with f16 P.V whenever v fits.
#define H3B_ATTENTION_KERNEL_ONLY
#include "attention.cu"

#include <mutex>

namespace h3b {
namespace noalloc {

// control words (range flag, status word) in the first 256 bytes, then the f16 copy of v
constexpr int64_t kControlBytes = 256;
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

// v [s_kv, heads, 128] bf16 (strided) -> out [s_kv, heads, 128] f16 contiguous; flag = 1 on a finite overflow
__global__ void v_to_f16_kernel(const uint16_t* __restrict__ v, int64_t s_kv, int heads, int64_t v_tok,
                                int64_t v_head, uint16_t* __restrict__ out, int32_t* flag) {
  const int64_t total = s_kv * heads * 16;  // 16-byte granules of 8 elements
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t & 15, th = t >> 4;
    const int64_t h = th % heads, tok = th / heads;
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(v + tok * v_tok + h * v_head) + c);
    uint32_t w[4] = {x.x, x.y, x.z, x.w};
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = __uint_as_float(w[i] << 16), b = __uint_as_float(w[i] & 0xFFFF0000u);
      bad |= (fabsf(a) > 65504.0f && isfinite(a)) || (fabsf(b) > 65504.0f && isfinite(b));
      __half2 hv = __floats2half2_rn(a, b);
      w[i] = *reinterpret_cast<uint32_t*>(&hv);
    }
    if (bad) atomicExch(flag, 1);
    reinterpret_cast<uint4*>(out)[t] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace noalloc
}  // namespace h3b

extern "C" int h3b_flash_attn_fwd_noalloc(const void* q, int64_t q_tok, int64_t q_head, const void* k, int64_t k_tok,
                                          int64_t k_head, const void* v, int64_t v_tok, int64_t v_head, void* o,
                                          int64_t o_tok, int64_t o_head, int64_t s_q, int64_t s_kv, int64_t valid_kv,
                                          int32_t heads, int32_t head_dim, float scale, h3b_stream_t stream) {
  using namespace h3b::attn;
  using namespace h3b::noalloc;
  if (s_q < 0 || s_kv <= 0 || heads <= 0)
    return fail(H3B_EINVAL, "flash_attn_noalloc: s_q %lld s_kv %lld heads %d", (long long)s_q, (long long)s_kv, heads);
  if (head_dim != 128) return fail(H3B_EUNSUPPORTED, "flash_attn_noalloc: head_dim %d (only 128)", head_dim);
  if (valid_kv < 0) valid_kv = s_kv;
  if (valid_kv == 0 || valid_kv > s_kv)
    return fail(H3B_EINVAL, "flash_attn_noalloc: valid_kv %lld of %lld", (long long)valid_kv, (long long)s_kv);
  if (s_kv * static_cast<int64_t>(heads) * 128 > kMaxVElems)
    return fail(H3B_EUNSUPPORTED,
                "flash_attn_noalloc: s_kv * heads * 128 = %lld exceeds the fixed scratch of %lld f16 elements "
                "(s_kv * heads <= %lld); use h3b_flash_attn_fwd",
                (long long)(s_kv * heads * 128), (long long)kMaxVElems, (long long)(kMaxVElems / 128));
  if (s_q == 0) return H3B_OK;
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return fail(H3B_EINVAL, "flash_attn_noalloc: null pointer");
  if (heads > 65535 || s_q > (1ll << 31) - 1) return fail(H3B_EUNSUPPORTED, "flash_attn_noalloc: size limits");
  const int64_t strides[8] = {q_tok, q_head, k_tok, k_head, v_tok, v_head, o_tok, o_head};
  for (int64_t s : strides)
    if (s <= 0 || s % 8) return fail(H3B_EALIGN, "flash_attn_noalloc: token/head strides must be positive multiples of 8");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o)) & 15u)
    return fail(H3B_EALIGN, "flash_attn_noalloc: q, k, v, o must be 16-byte aligned");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "flash_attn_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(H3B_EUNSUPPORTED, "flash_attn_noalloc: device index %d", dev);
  unsigned char* base = nullptr;
  int rc = setup(dev, &base);
  if (rc) return rc;
  int32_t* flag = reinterpret_cast<int32_t*>(base);
  int* status = reinterpret_cast<int*>(base + 4);
  uint16_t* v16 = reinterpret_cast<uint16_t*>(base + kControlBytes);

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the array keeps the previous call's contents: the flag and the status word must start at zero
  e = cudaMemsetAsync(base, 0, 8, st);
  if (e != cudaSuccess) return cuda_fail(e, "flash_attn_noalloc: clearing the control words");
  const int64_t granules = s_kv * heads * 16;
  int64_t blocks = (granules + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  if (blocks > cap) blocks = cap;
  v_to_f16_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(static_cast<const uint16_t*>(v), s_kv, heads, v_tok,
                                                              v_head, v16, flag);
  H3B_CHECK_LAUNCH("flash_attn_noalloc: v conversion launch");

  Params p{};
  p.s_q = s_q;
  p.s_kv = s_kv;
  p.valid_kv = valid_kv;
  p.heads = heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = static_cast<uint16_t*>(o);
  p.o_tok = o_tok;
  p.o_head = o_head;
  p.range_flag = flag;
  p.wc.status = status;
  p.wc.timeout = wait_timeout_ns();
  p.range_mode = 1;  // f16 P.V unless v overflowed f16
  rc = launch_attention(q, q_tok, q_head, k, k_tok, k_head, v16, static_cast<int64_t>(heads) * 128, 128, true, p, st);
  if (rc) return rc;
  p.range_mode = 2;  // bf16 P.V only if it did
  rc = launch_attention(q, q_tok, q_head, k, k_tok, k_head, v, v_tok, v_head, false, p, st);
  if (rc) return rc;
  return H3B_OK;
}
