// Peer memory for the tensor-parallel exchange between the GPUs of one node.
//
// Each rank allocates its exchange buffers with w8a8_peer_alloc and publishes
// the 64-byte CUDA IPC handle; the host side carries the handles to the other
// ranks (the Python layer uses torch.distributed.all_gather_object) and each
// rank maps its peers' buffers with w8a8_peer_open. Kernels then load and store
// peer memory directly over NVLink: plain 16-byte loads and stores, no TMA and
// no multicast on peer memory anywhere.
//
// Ordering between GPUs uses flag words: w8a8_peer_signal, enqueued after the
// kernels whose stores must be seen, waits for them (programmatic dependent
// launch) and then publishes `value` into one flag word on each listed GPU with
// a system-scope fence and release store; w8a8_peer_wait, enqueued before the
// kernels that read, spins with system-scope acquire loads until n flag words
// of this GPU reach `value`. The wait is bounded: after ~2 s of SM clock it
// records an error code in the device error word and returns, so a peer that
// never signals cannot hang the GPU. Flag values only grow (one epoch counter
// per exchange step), so flags never need resetting.
#include <string.h>

#include "common.cuh"
#include "runtime.cuh"

namespace w8a8 {

constexpr int kMaxPeers = 8;

struct SignalArgs {
  uint32_t *flag[kMaxPeers];
  int n;
  uint32_t value;
};

struct WaitArgs {
  const uint32_t *flags;
  int n;
  uint32_t value;
  int *err;
};

__global__ void peer_signal_kernel(SignalArgs a) {
  pdl_wait();  // the producing kernels have completed
  pdl_launch_dependents();
  const int i = threadIdx.x;
  if (i < a.n) {
    asm volatile("fence.sc.sys;" ::: "memory");
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flag[i]), "r"(a.value) : "memory");
  }
}

__global__ void peer_wait_kernel(WaitArgs a) {
  pdl_wait();
  const int i = threadIdx.x;
  if (i < a.n) {
    const uint32_t *f = a.flags + i;
    long long t0 = clock64();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if ((int32_t)(v - a.value) >= 0) break;  // wrap-safe "v >= value"
      if (clock64() - t0 > kWaitLimitCycles) {
        report_error(a.err, 0x1301);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  pdl_launch_dependents();
}

}  // namespace w8a8

using namespace w8a8;

extern "C" int w8a8_peer_alloc(size_t bytes, void **ptr, void *ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return W8A8_ERR_INVALID;
  *ptr = nullptr;
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return W8A8_ERR_NOMEM;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return W8A8_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return W8A8_OK;
}

extern "C" int w8a8_peer_open(const void *ipc_handle, void **ptr) {
  if (!ipc_handle || !ptr) return W8A8_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void *p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return W8A8_ERR_CUDA;
  }
  *ptr = p;
  return W8A8_OK;
}

extern "C" int w8a8_peer_close(void *ptr) {
  if (!ptr) return W8A8_ERR_INVALID;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? W8A8_OK : W8A8_ERR_CUDA;
}

extern "C" int w8a8_peer_free(void *ptr) {
  if (!ptr) return W8A8_ERR_INVALID;
  return cudaFree(ptr) == cudaSuccess ? W8A8_OK : W8A8_ERR_CUDA;
}

extern "C" int w8a8_peer_copy(void *dst, const void *src, size_t bytes, void *stream) {
  if (bytes == 0) return W8A8_OK;
  if (!dst || !src) return W8A8_ERR_INVALID;
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream) ==
                 cudaSuccess
             ? W8A8_OK
             : W8A8_ERR_CUDA;
}

extern "C" int w8a8_peer_signal(uint32_t *const *flags, int n, uint32_t value, void *stream) {
  if (!flags || n <= 0 || n > kMaxPeers) return W8A8_ERR_INVALID;
  SignalArgs a = {};
  for (int i = 0; i < n; ++i) {
    if (!flags[i] || ((uintptr_t)flags[i] & 3)) return W8A8_ERR_INVALID;
    a.flag[i] = flags[i];
  }
  a.n = n;
  a.value = value;
  int st;
  if (!device_ctx(&st)) return st;
  launch_pdl(peer_signal_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, a);
  return check_launch("peer_signal");
}

extern "C" int w8a8_peer_wait(const uint32_t *flags, int n, uint32_t value, void *stream) {
  if (!flags || n <= 0 || n > 32 || ((uintptr_t)flags & 3)) return W8A8_ERR_INVALID;
  int st;
  DeviceCtx *c = device_ctx(&st);
  if (!c) return st;
  WaitArgs a = {flags, n, value, c->err};
  launch_pdl(peer_wait_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, a);
  return check_launch("peer_wait");
}
