// Per-device runtime state shared by the kernel launchers: SM count, device
// error word, TMA descriptor encoder (resolved through the runtime's driver
// entry-point query, so the library links against libcudart only).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gpt2_w8a8.h"

namespace w8a8 {

struct DeviceCtx {
  int ready;
  int sm_count;
  int *err;  // device error word (in device memory of this device)
};

// Returns the context of the current device, initialising it on first use
// (first use must not happen inside stream capture; w8a8_init does it early).
DeviceCtx *device_ctx(int *status);

// 2-D row-major tensor map: `rows` x `cols` elements, row pitch in bytes,
// box of box_cols x box_rows, 128-byte swizzle, out-of-bounds reads as zero.
// 2-D tensor map over a row-major matrix; boxes of box_rows x box_cols,
// written to shared memory with the 128-byte swizzle (the MMA operands), the
// 32-byte swizzle (swizzle_bytes = 32: 16-byte halves of 32-byte rows swapped
// on rows 4..7 of every 8) or none (0: maps used only for L2 prefetches).
int make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, uint64_t rows,
                 uint64_t cols, uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 int swizzle_bytes = 128);
// [planes][rows][cols] view (cols contiguous), box {box_cols, box_rows, 1},
// 128-byte swizzle; elements outside the extents read as zero.
int make_tmap_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, uint64_t planes,
                 uint64_t rows, uint64_t cols, uint64_t row_pitch_bytes,
                 uint64_t plane_pitch_bytes, uint32_t box_cols, uint32_t box_rows);

// Launch `kernel` with programmatic dependent launch allowed: it may begin
// while the preceding kernel of the stream finishes (see pdl_wait()).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Remember the CUDA error behind a W8A8_ERR_CUDA (w8a8_last_cuda_error).
void note_cuda_error(cudaError_t e);

inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  (void)what;
  if (e == cudaSuccess) return W8A8_OK;
  note_cuda_error(e);
  return W8A8_ERR_CUDA;
}

__host__ __device__ inline bool aligned16(const void *p) { return (((uintptr_t)p) & 15u) == 0; }

}  // namespace w8a8
