// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
// D[n, m] = sum_k W[n, k] * X[m, k] — the weight tile is the MMA's A operand
// (128 rows of output channels) and the token tile its B operand (BN tokens),
// so a decode batch of 16..256 tokens fills one MMA N dimension and prefill
// tiles the token dimension. Both operands are K-major exactly as the
// reference stores them (W [OUT, IN], activations [tokens, IN]).
//
//   warp 0      TMA producer: 128 x 128 B weight box + BN x 128 B token box
//               per stage (SWIZZLE_128B, no multicast).
//   warp 1      TMEM allocator + single-thread MMA issuer
//               (kind::i8 -> s32, or kind::f16 with bf16 -> f32 for the LM head).
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused dequant / bias /
//               residual / GELU / QKV scatter, bf16 stores.
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Replaces the reference's cublasGemmEx INT8 call (gpt2.c:404-415), its
// dequant kernel (cuda/activation_quant.cu:117-131) and the add_bias /
// add_2d / gelu kernels that follow each GEMM (gpt2.c:1145-1325), and the
// bf16 LM-head GEMM (gpt2.c:2160).
#include <stdio.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

struct GemmArgs : LinearArgs {
  int BN;       // token tile (multiple of 32, <= 256)
  int stages;
  int num_n_tiles, num_m_tiles;
  int kblocks;  // ceil(K bytes / 128)
  // split-K: each (tile, split) unit reduces k-blocks [ks*kb_per, ..); the
  // partial int32 sums meet in `ws` ([M][N], zero between calls) through
  // integer atomics (exact in any order), and the last unit of a tile, found
  // by a ticket counter, applies the epilogue and re-zeroes its tile.
  int ksplit, kb_per;
  int32_t *ws;
  int *tickets;
  int *err;
};

constexpr int kBM = 128;            // weight rows per tile (MMA M)
constexpr int kBoxBytes = 128;      // K bytes per stage (one 128 B swizzle atom)
constexpr int kThreads = 192;       // 6 warps
constexpr int kEpiWarp0 = 2;

struct __align__(8) SmemCtl {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;  // k-iterations consumed by the MMA thread (for abort drain)
  int last_flag; // split-K: this CTA holds the last partial of the tile
  int vote[2][4]; // epilogue warps' wait verdicts, double-buffered by unit
};

__device__ __forceinline__ void store_out(const GemmArgs &a, int epi, int m, int n, int32_t acc,
                                          float sw, float sx, float bias, int qseg, int qcol) {
  (void)qseg;
  (void)qcol;
  switch (epi) {
    case EPI_S32:
      reinterpret_cast<int32_t *>(a.Y)[(int64_t)m * a.ldy + n] = acc;
      break;
    case EPI_DEQUANT:
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(dequant_bf(acc, sw, sx));
      break;
    case EPI_BIAS:
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] =
          f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bias));
      break;
    case EPI_RESID: {
      float y = add_bf(dequant_bf(acc, sw, sx), bias);
      float r = bf2f(a.R[(int64_t)m * a.ldr + n]);
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(__fadd_rn(r, y));
      break;
    }
    case EPI_GELU: {
      float y = add_bf(dequant_bf(acc, sw, sx), bias);
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(gelu_tanh(y));
      break;
    }
    case EPI_QKV: {
      uint16_t v = f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bias));
      if (qseg == 0) {
        reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + qcol] = v;
      } else {
        int b = m / a.T;
        int t = m - b * a.T;
        int p = (a.pos0 ? a.pos0[b] : 0) + t;
        uint16_t *base = qseg == 1 ? a.Kc : a.Vc;
        base[(int64_t)b * a.seq_stride + (int64_t)p * a.dseg + qcol] = v;
      }
      break;
    }
    default: {  // EPI_F32_BF16
      reinterpret_cast<uint16_t *>(a.Y)[(int64_t)m * a.ldy + n] = f2bf(__int_as_float(acc));
      break;
    }
  }
}

template <int KIND, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int BN = a.BN;
  const int stages = a.stages;
  const uint32_t a_bytes = kBM * kBoxBytes;
  const uint32_t b_bytes = (uint32_t)BN * kBoxBytes;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  SmemCtl *ctl = reinterpret_cast<SmemCtl *>(smem + (size_t)stages * stage_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = a.num_n_tiles * a.num_m_tiles * a.ksplit;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * BN)) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->tmem_full[i], 1);
      mbar_init(&ctl->tmem_empty[i], 128);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    ctl->consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int *abort_flag = &ctl->abort_flag;
  int issued = 0;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    const int kbox = kBoxBytes / (KIND == 0 ? 1 : 2);
    int stage = 0;
    uint32_t phase = 0;
    for (int u = blockIdx.x; u < total_units && !*abort_flag; u += gridDim.x) {
      const int t = u / a.ksplit, ks = u - (u / a.ksplit) * a.ksplit;
      const int n0 = (t % a.num_n_tiles) * kBM;
      const int m0 = (t / a.num_n_tiles) * BN;
      const int kb0 = ks * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort_flag, a.err, 0x1101)) break;
        uint8_t *sa = smem + (size_t)stage * stage_bytes;
        mbar_arrive_expect_tx(&ctl->full[stage], stage_bytes);
        tma_load_2d(sa, &tmW, &ctl->full[stage], kb * kbox, n0);
        tma_load_2d(sa + a_bytes, &tmX, &ctl->full[stage], kb * kbox, m0);
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc =
        KIND == 0 ? make_idesc(2, 1, kBM, BN) : make_idesc(1, 1, kBM, BN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int consumed = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const int ks = u - (u / a.ksplit) * a.ksplit;
      const int kb0 = ks * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
      if (!mbar_wait(&ctl->tmem_empty[acc], acc_phase ^ 1, abort_flag, a.err, 0x1102)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&ctl->full[stage], phase, abort_flag, a.err, 0x1103)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)stage * stage_bytes);
        const uint32_t sb = sa + a_bytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // 4 x 32-byte K steps inside the 128-byte atom
          const uint64_t da = make_sw128_desc(sa + 32 * k);
          const uint64_t db = make_sw128_desc(sb + 32 * k);
          const uint32_t accum = (kb != kb0) || (k != 0);
          if (KIND == 0)
            tc_mma_i8(d_tmem, da, db, idesc, accum);
          else
            tc_mma_bf16(d_tmem, da, db, idesc, accum);
        }
        tc_commit(&ctl->empty[stage]);
        ++consumed;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      tc_commit(&ctl->tmem_full[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    ctl->consumed = consumed;
    if (!ok) {
      // Make sure no MMA is still writing TMEM before the CTA releases it.
      tc_commit(&ctl->drain);
      mbar_wait(&ctl->drain, 0, nullptr, a.err, 0x1104);
    }
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
      const int t = u / a.ksplit;
      // Warp-uniform wait: lane 0 polls with the bound, the verdict is
      // broadcast, so the warp-collective tcgen05.ld below never runs with
      // part of the warp gone.
      // All four epilogue warps then agree through a vote before any of them
      // proceeds, so the named barriers below always see all 128 threads.
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&ctl->tmem_full[acc], acc_phase, abort_flag, a.err, 0x1105);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane == 0) ctl->vote[iter & 1][quarter] = ok;
      named_barrier_sync(1, 128);
      ok = ctl->vote[iter & 1][0] & ctl->vote[iter & 1][1] & ctl->vote[iter & 1][2] &
           ctl->vote[iter & 1][3];
      ++iter;
      if (!ok) break;
      mbar_wait(&ctl->tmem_full[acc], acc_phase, nullptr, a.err, 0x1107);  // completed: returns at once
      tc_fence_after();
      const int n0 = (t % a.num_n_tiles) * kBM;
      const int m0 = (t / a.num_n_tiles) * BN;
      const int n = n0 + quarter * 32 + lane;
      const bool n_ok = n < a.N;
      float sw = 0.f, bias = 0.f;
      int qseg = 0, qcol = n;
      if (n_ok) {
        if (EPI != EPI_S32 && EPI != EPI_F32_BF16) sw = a.sW[n];
        if (EPI >= EPI_BIAS && EPI <= EPI_QKV) bias = bf2f(a.bias[n]);
        if (EPI == EPI_QKV) {
          qseg = n / a.dseg;
          qcol = n - qseg * a.dseg;
        }
      }
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      if (a.ksplit == 1) {
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)c, r);
          tmem_ld_wait();
          const int mbase = m0 + c;
          float sx_lane = 0.f;
          if (EPI != EPI_S32 && EPI != EPI_F32_BF16 && mbase + lane < a.M)
            sx_lane = a.sX[mbase + lane];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float sx = __shfl_sync(0xffffffffu, sx_lane, i);
            const int m = mbase + i;
            if (n_ok && m < a.M) store_out(a, EPI, m, n, (int32_t)r[i], sw, sx, bias, qseg, qcol);
          }
        }
        tc_fence_before();
        mbar_arrive(&ctl->tmem_empty[acc]);
      } else {
        // add this split's partial sums into the workspace tile
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + c + i;
            if (n_ok && m < a.M) atomicAdd(a.ws + (int64_t)m * a.N + n, (int)r[i]);
          }
        }
        tc_fence_before();
        mbar_arrive(&ctl->tmem_empty[acc]);  // TMEM is free for the next unit
        __threadfence();
        named_barrier_sync(1, 128);
        if (warp == kEpiWarp0 && lane == 0) {
          const int ticket = atomicAdd(a.tickets + t, 1);
          ctl->last_flag = (ticket == a.ksplit - 1);
        }
        named_barrier_sync(1, 128);
        if (ctl->last_flag) {
          __threadfence();
          for (int c = 0; c < BN; c += 32) {
            const int mbase = m0 + c;
            float sx_lane = 0.f;
            if (EPI != EPI_S32 && EPI != EPI_F32_BF16 && mbase + lane < a.M)
              sx_lane = a.sX[mbase + lane];
#pragma unroll 4
            for (int i = 0; i < 32; ++i) {
              const float sx = __shfl_sync(0xffffffffu, sx_lane, i);
              const int m = mbase + i;
              if (n_ok && m < a.M) {
                int32_t *w = a.ws + (int64_t)m * a.N + n;
                const int32_t tot = __ldcg(w);
                *w = 0;
                store_out(a, EPI, m, n, tot, sw, sx, bias, qseg, qcol);
              }
            }
          }
          if (warp == kEpiWarp0 && lane == 0) a.tickets[t] = 0;
        }
        named_barrier_sync(1, 128);  // last_flag is reused by the next unit
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // Drain TMA loads that were issued but never consumed so no bulk copy is
    // still writing this CTA's shared memory when it exits.
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < issued; ++i) {
      if (i >= ctl->consumed) mbar_wait(&ctl->full[stage], phase, nullptr, a.err, 0x1106);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// host-side launcher
// ---------------------------------------------------------------------------
static int pick_bn(int M) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 96) return 96;
  if (M <= 128) return 128;
  if (M <= 192) return 192;
  return 256;
}

template <int KIND, int EPI>
static int launch_tc(const void *W, const void *X, int64_t ldx_elems, const LinearArgs &la,
                     cudaStream_t stream) {
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  GemmArgs a;
  static_cast<LinearArgs &>(a) = la;
  const int M = la.M, N = la.N, K = la.K;
  const int esz = KIND == 0 ? 1 : 2;
  const CUtensorMapDataType dt =
      KIND == 0 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  a.BN = pick_bn(M);
  CUtensorMap tmW, tmX;
  st = make_tmap_2d(&tmW, W, dt, (uint64_t)N, (uint64_t)K, (uint64_t)K * esz, kBoxBytes / esz, kBM);
  if (st) return st;
  st = make_tmap_2d(&tmX, X, dt, (uint64_t)M, (uint64_t)K, (uint64_t)ldx_elems * esz,
                    kBoxBytes / esz, (uint32_t)a.BN);
  if (st) return st;
  const int stage_bytes = (kBM + a.BN) * kBoxBytes;
  const int budget = 227 * 1024 - 1024 - (int)sizeof(SmemCtl) - 64;
  a.stages = budget / stage_bytes;
  if (a.stages > 8) a.stages = 8;
  if (a.stages < 2) return W8A8_ERR_UNSUPPORTED;
  const size_t smem = 1024 + (size_t)a.stages * stage_bytes + sizeof(SmemCtl);
  a.num_n_tiles = (N + kBM - 1) / kBM;
  a.num_m_tiles = (M + a.BN - 1) / a.BN;
  a.kblocks = (K * esz + kBoxBytes - 1) / kBoxBytes;
  a.err = ctx->err;
  a.ksplit = 1;
  a.kb_per = a.kblocks;
  a.ws = nullptr;
  a.tickets = nullptr;
  const int tiles0 = a.num_n_tiles * a.num_m_tiles;
  if (KIND == 0 && la.workspace && 2 * tiles0 <= ctx->sm_count && a.kblocks > 1 &&
      la.workspace_bytes >= linear_workspace_bytes(M, N)) {
    // Too few output tiles to occupy the GPU (decode): split K so that about
    // one unit lands on every SM.
    int ks = ctx->sm_count / tiles0;
    if (ks > a.kblocks) ks = a.kblocks;
    a.kb_per = (a.kblocks + ks - 1) / ks;
    a.ksplit = (a.kblocks + a.kb_per - 1) / a.kb_per;
    if (a.ksplit > 1) {
      uint8_t *w = (uint8_t *)la.workspace;
      a.ws = (int32_t *)w;
      a.tickets = (int *)(w + (((size_t)M * N * 4 + 255) & ~(size_t)255));
    } else {
      a.kb_per = a.kblocks;
    }
  }
  static bool attr_set[64] = {};  // per template instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<KIND, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return W8A8_ERR_CUDA;
    attr_set[dev] = true;
  }
  int units = a.num_n_tiles * a.num_m_tiles * a.ksplit;
  int grid = units < ctx->sm_count ? units : ctx->sm_count;
  gemm_tc_kernel<KIND, EPI><<<grid, kThreads, smem, stream>>>(tmW, tmX, a);
  return check_launch("gemm_tc");
}

size_t linear_workspace_bytes(int M, int N) {
  const size_t tiles = (size_t)((N + kBM - 1) / kBM) * (size_t)((M + 31) / 32);
  return (((size_t)M * N * 4 + 255) & ~(size_t)255) + tiles * 4;
}

int gemm_tc_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
               cudaStream_t stream) {
  switch (a.epi) {
    case EPI_S32: return launch_tc<0, EPI_S32>(W, X, ldx, a, stream);
    case EPI_DEQUANT: return launch_tc<0, EPI_DEQUANT>(W, X, ldx, a, stream);
    case EPI_BIAS: return launch_tc<0, EPI_BIAS>(W, X, ldx, a, stream);
    case EPI_RESID: return launch_tc<0, EPI_RESID>(W, X, ldx, a, stream);
    case EPI_GELU: return launch_tc<0, EPI_GELU>(W, X, ldx, a, stream);
    case EPI_QKV: return launch_tc<0, EPI_QKV>(W, X, ldx, a, stream);
    default: return W8A8_ERR_INVALID;
  }
}

int gemm_tc_bf16(const uint16_t *W, const uint16_t *X, int64_t ldx, const LinearArgs &a,
                 cudaStream_t stream) {
  if (a.epi != EPI_F32_BF16) return W8A8_ERR_INVALID;
  return launch_tc<1, EPI_F32_BF16>(W, X, ldx, a, stream);
}

}  // namespace w8a8
