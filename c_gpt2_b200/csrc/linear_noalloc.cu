// Fixed-scratch variant of the fused W8A8 linear layer.
//
// w8a8_linear splits small (decode-sized) GEMMs over K and needs an int32
// workspace for the partial sums, which its caller allocates. Some callers
// cannot: a host program that sizes all device memory once at start-up and
// may not allocate in its token loop (gpt2.c allocates every buffer in
// allocate_weights_gpu and nowhere else), a plugin whose host owns the device
// allocator, or a code path that must not pay cudaMalloc's implicit device
// synchronisation. w8a8_linear_noalloc serves them from a scratch array
// compiled into this library instead.
//
// The scratch is a file-scope __device__ array of W8A8_NOALLOC_SCRATCH_BYTES
// (4 MiB): every GPU that loads the library holds it until the process exits.
// Its device address is looked up once per device, on the first call made
// with that device current, so that first call must come before any stream
// capture. All calls share the array and it keeps the last call's contents,
// so each call clears the part the split-K reduction needs zeroed; calls whose
// GPU work overlaps (different streams, or different host threads on one
// device) race on it and must be serialised by the caller.
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
  // The scratch holds the [M][N] int32 partial sums plus one ticket per tile.
  const size_t need = linear_workspace_bytes(M, N);
  if (need > (size_t)W8A8_NOALLOC_SCRATCH_BYTES) return W8A8_ERR_UNSUPPORTED;
  void *scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != W8A8_OK) return st;
  // The split-K reduction adds into the scratch and counts tickets from zero.
  if (cudaMemsetAsync(scratch, 0, need, (cudaStream_t)stream) != cudaSuccess)
    return W8A8_ERR_CUDA;
  return w8a8_linear(Xq, sX, M, K, W, sW, bias, N, epilogue, R, ldr, Y, ldy, scratch, need,
                     stream);
}
