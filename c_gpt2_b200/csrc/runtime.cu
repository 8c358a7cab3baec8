// Per-device state, status strings and the device error word.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "runtime.cuh"

namespace w8a8 {

// One error word per device. Kernels record the first failure here (bounded
// wait expired, shape check failed) instead of trapping.
__device__ int g_device_error;

static DeviceCtx g_ctx[64];

// The CUDA error of the calling thread's last failed launch.
static thread_local cudaError_t g_last_cuda_error = cudaSuccess;
void note_cuda_error(cudaError_t e) { g_last_cuda_error = e; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn g_encode = nullptr;

static int resolve_encoder() {
  if (g_encode) return W8A8_OK;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return W8A8_ERR_CUDA;
  g_encode = (EncodeTiledFn)fn;
  return W8A8_OK;
}

DeviceCtx *device_ctx(int *status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    if (status) *status = W8A8_ERR_CUDA;
    return nullptr;
  }
  DeviceCtx *c = &g_ctx[dev];
  if (!c->ready) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      if (status) *status = W8A8_ERR_CUDA;
      return nullptr;
    }
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) {
      if (status) *status = W8A8_ERR_CUDA;
      return nullptr;
    }
    int st = resolve_encoder();
    if (st != W8A8_OK) {
      if (status) *status = st;
      return nullptr;
    }
    c->sm_count = sms;
    c->err = (int *)p;
    c->ready = 1;
  }
  if (status) *status = W8A8_OK;
  return c;
}

int make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, uint64_t rows,
                 uint64_t cols, uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 int swizzle_bytes) {
  if (!g_encode && resolve_encoder() != W8A8_OK) return W8A8_ERR_CUDA;
  if (!aligned16(base) || (row_pitch_bytes & 15u) || rows == 0 || cols == 0)
    return W8A8_ERR_INVALID;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? W8A8_OK : W8A8_ERR_INVALID;
}

int make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, uint64_t planes,
                 uint64_t rows, uint64_t cols, uint64_t row_pitch_bytes,
                 uint64_t plane_pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  if (!g_encode && resolve_encoder() != W8A8_OK) return W8A8_ERR_CUDA;
  if (!aligned16(base) || (row_pitch_bytes & 15u) || (plane_pitch_bytes & 15u) || rows == 0 ||
      cols == 0 || planes == 0)
    return W8A8_ERR_INVALID;
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {row_pitch_bytes, plane_pitch_bytes};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? W8A8_OK : W8A8_ERR_INVALID;
}

}  // namespace w8a8

using namespace w8a8;

extern "C" int w8a8_init(int device) {
  if (cudaSetDevice(device) != cudaSuccess) return W8A8_ERR_CUDA;
  int st;
  DeviceCtx *c = device_ctx(&st);
  return c ? W8A8_OK : st;
}

extern "C" const char *w8a8_last_cuda_error(void) {
  return g_last_cuda_error == cudaSuccess ? "no error" : cudaGetErrorString(g_last_cuda_error);
}

extern "C" const char *w8a8_status_string(int status) {
  switch (status) {
    case W8A8_OK: return "ok";
    case W8A8_ERR_INVALID: return "invalid argument (shape, null pointer or alignment)";
    case W8A8_ERR_UNSUPPORTED: return "shape not supported by this build";
    case W8A8_ERR_CUDA: return "CUDA runtime call or kernel launch failed";
    case W8A8_ERR_DEVICE: return "a kernel recorded an error in the device error word";
    case W8A8_ERR_NOMEM: return "out of memory";
    case W8A8_ERR_IO: return "I/O error";
    default: return "unknown status";
  }
}

extern "C" int w8a8_device_error(int reset) {
  int st;
  DeviceCtx *c = device_ctx(&st);
  if (!c) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return W8A8_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, c->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return W8A8_ERR_CUDA;
  if (reset && v) {
    int z = 0;
    if (cudaMemcpy(c->err, &z, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
      return W8A8_ERR_CUDA;
  }
  return v;
}
