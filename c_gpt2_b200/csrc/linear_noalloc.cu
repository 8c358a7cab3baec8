// Fixed-scratch variant of the fused W8A8 linear layer.
//
// w8a8_linear splits a few-token GEMM over K when its operands rule out the
// cluster kernel (unaligned output rows, N not a multiple of 4, ...), and that
// split needs an int32 workspace for the partial sums, which its caller
// allocates. Some callers cannot: a host program that sizes all device memory
// once at start-up and may not allocate in its token loop (gpt2.c allocates
// every buffer in allocate_weights_gpu and nowhere else), a plugin whose host
// owns the device allocator, or a code path that must not pay cudaMalloc's
// implicit device synchronisation. w8a8_linear_noalloc serves them from a
// scratch array compiled into this library instead.
//
// The scratch is a file-scope __device__ array of W8A8_NOALLOC_SCRATCH_BYTES
// (4 MiB): every GPU that loads the library holds it until the process exits.
// Its device address is looked up once per device, on the first call made
// with that device current, so that first call must come before any stream
// capture. Only calls whose dispatch ends in the split-K kernel touch the
// scratch; each of those clears the bytes it uses (the [M][N] partial sums and
// one arrival counter per output tile must start at zero) and refuses shapes
// that need more than the array holds. Every other shape (one token, the
// token-major prefill GEMM, the cluster GEMM) runs exactly as w8a8_linear
// without a workspace. All calls share the array and it keeps the last call's
// contents; calls whose GPU work overlaps (different streams, or different
// host threads on one device) race on it and must be serialised by the caller.
#include "common.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

static __device__ __align__(256) unsigned char g_noalloc_scratch[W8A8_NOALLOC_SCRATCH_BYTES];

static void *g_noalloc_ptr[64];

// Device address of the scratch array for the current device (host code may
// not use the symbol itself: on the host it names a stand-in, not device
// memory).
static int noalloc_scratch(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return W8A8_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return W8A8_OK;
}

}  // namespace w8a8

using namespace w8a8;

extern "C" int w8a8_linear_noalloc(const int8_t *Xq, const float *sX, int M, int K,
                                   const int8_t *W, const float *sW, const gpt2_bf16_t *bias,
                                   int N, int epilogue, const gpt2_bf16_t *R, int64_t ldr,
                                   gpt2_bf16_t *Y, int64_t ldy, void *stream) {
  if (M == 0 || N == 0) return W8A8_OK;
  if (M < 0 || N < 0) return W8A8_ERR_INVALID;
  void *scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != W8A8_OK) return st;
  const size_t need = linear_workspace_used(Xq, sX, M, K, W, sW, bias, N, epilogue, R, ldr, Y, ldy);
  if (need == 0)  // the chosen kernel reads no workspace
    return w8a8_linear(Xq, sX, M, K, W, sW, bias, N, epilogue, R, ldr, Y, ldy, nullptr, 0,
                       stream);
  if (need > (size_t)W8A8_NOALLOC_SCRATCH_BYTES) return W8A8_ERR_UNSUPPORTED;
  // The split-K reduction adds into the partial sums and counts arrivals from
  // zero. The kernel leaves both at zero again, but a call that stopped early
  // (a device error) may not have.
  if (cudaMemsetAsync(scratch, 0, need, (cudaStream_t)stream) != cudaSuccess)
    return W8A8_ERR_CUDA;
  return w8a8_linear(Xq, sX, M, K, W, sW, bias, N, epilogue, R, ldr, Y, ldy, scratch, need,
                     stream);
}
