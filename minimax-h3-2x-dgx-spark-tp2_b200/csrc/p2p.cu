// Peer memory for the Ulysses P2P exchange: CUDA IPC allocations shared between the ranks of one NVSwitch box, and
// the epoch flag signal/wait kernel that orders one rank's peer stores before the other ranks' reads.  No multicast
// object is ever created (plain cudaMalloc + cudaIpc*), so a rank that dies leaves no NVLink multicast binding.
#include <string.h>

#include "common.cuh"

namespace h3b {
namespace p2p {

struct FlagPtrs {
  int32_t* peer[H3B_MAX_RANKS];
};

__global__ void signal_wait_kernel(const __grid_constant__ FlagPtrs peers, int32_t* mine, int ws, int rank, int epoch, WaitCtl wc) {
  const int t = threadIdx.x;
  if (t < ws) {
    __threadfence_system();  // everything this stream wrote before (peer stores included) before the flag
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(peers.peer[t] + rank), "r"(epoch) : "memory");
  }
  __syncthreads();
  if (t < ws) {
    const uint64_t t0 = globaltimer();
    int32_t v = 0;
    while (true) {
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine + t) : "memory");
      // epochs only grow: wrap-safe "v >= epoch" in 32-bit serial-number arithmetic
      if (static_cast<int32_t>(static_cast<uint32_t>(v) - static_cast<uint32_t>(epoch)) >= 0) break;
      if (status_bad(wc)) break;
      if (globaltimer() - t0 > wc.timeout) {
        record_status(wc, H3B_ETIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

}  // namespace p2p
}  // namespace h3b

using namespace h3b;

extern "C" {

int h3b_p2p_alloc(size_t bytes, void** ptr, h3b_ipc_handle* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return fail(H3B_EINVAL, "p2p_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "p2p_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  // the zeros must land before any peer can see the handle and store into the buffer
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) {
      static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(handle->bytes), "IPC handle size");
      memcpy(handle->bytes, &h, sizeof(h));
      *ptr = p;
      return H3B_OK;
    }
  }
  cudaFree(p);
  return cuda_fail(e, "p2p_alloc: memset / IPC handle");
}

int h3b_p2p_open(const h3b_ipc_handle* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(H3B_EINVAL, "p2p_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "p2p_open: cudaIpcOpenMemHandle");
  return H3B_OK;
}

int h3b_p2p_close(void* peer_ptr) {
  if (peer_ptr == nullptr) return H3B_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "p2p_close: cudaIpcCloseMemHandle");
  return H3B_OK;
}

int h3b_p2p_free(void* ptr) {
  if (ptr == nullptr) return H3B_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "p2p_free: cudaFree");
  return H3B_OK;
}

int h3b_p2p_signal_wait(int32_t* const* peer_flags, int32_t* my_flags, int32_t ws, int32_t rank, int32_t epoch,
                        h3b_stream_t stream) {
  if (peer_flags == nullptr || my_flags == nullptr || ws < 1 || ws > H3B_MAX_RANKS || rank < 0 || rank >= ws)
    return fail(H3B_EINVAL, "p2p_signal_wait: ws %d rank %d", ws, rank);
  p2p::FlagPtrs f{};
  for (int i = 0; i < ws; ++i) {
    if (peer_flags[i] == nullptr) return fail(H3B_EINVAL, "p2p_signal_wait: null flag pointer for rank %d", i);
    f.peer[i] = peer_flags[i];
  }
  WaitCtl wc{device_status_word(), wait_timeout_ns()};
  if (wc.status == nullptr) return fail(H3B_ECUDA, "p2p_signal_wait: device status word");
  p2p::signal_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, my_flags, ws, rank, epoch, wc);
  H3B_CHECK_LAUNCH("p2p_signal_wait launch");
  return H3B_OK;
}

}  // extern "C"
