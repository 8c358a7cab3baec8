// Decode-sized INT8 GEMM (M <= 128 tokens) with split-K partial sums reduced
// in distributed shared memory.
//
// Y[m, n] = epilogue(sum_k X[m, k] * W[n, k]) for the few tokens of a decode
// step. The weights are the MMA's M = 128 operand (channel-major: TMEM lane =
// output channel) and the BN <= 128 tokens its N operand. A decode GEMM has
// too few 128-channel tiles to occupy the GPU, so each tile's K range is split
// over the `ks` CTAs of one thread-block cluster:
//
//   1. every CTA streams its K slice of the weight tile with TMA (the weight
//      boxes are requested before waiting for the previous kernel), issues
//      tcgen05.mma kind::i8 into TMEM, and copies its int32 partial tile from
//      TMEM into its own shared memory, transposed to [token][channel];
//   2. one cluster barrier, then CTA r reduces slice r of the tile: it reads
//      the ks partials of its slice from the cluster's shared memory with
//      16-byte DSMEM loads, adds them in rank order (integer sums: exact in
//      any order) and applies the fused epilogue to 4 channels at a time;
//   3. a second cluster barrier keeps every CTA's shared memory alive until
//      all slices have been read.
//
// No global workspace, no atomics, no ticket counter and no second pass over
// L2. Roles: warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps
// 4..7 read the accumulator (warp w owns TMEM lanes 32*(w%4)...), all eight
// warps reduce. Every wait is bounded; a stalled pipeline records an error
// code, skips the copy-out and still reaches both cluster barriers.
//
// Replaces, for batched decode, the reference's cublasGemmEx INT8 call
// (gpt2.c:404-415), its dequant kernel (cuda/activation_quant.cu:117-131)
// and the add_bias / add_2d / gelu kernels after it (gpt2.c:1145-1325).
#include <stddef.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

constexpr int kCBM = 128;       // weight rows (channels) per tile
constexpr int kCBox = 128;      // K bytes per stage
constexpr int kCThreads = 256;  // 8 warps
constexpr int kCMaxStages = 8;
constexpr int kCMaxCluster = 8;  // portable cluster size
constexpr int kCPre = 2;         // reduction groups per thread with preloaded epilogue inputs

struct ClusterGemmArgs : LinearArgs {
  int BN;       // tokens per tile (multiple of 32, <= 128)
  int stages;
  int kblocks;  // ceil(K / 128)
  int kb_per;   // K blocks per split
  int ksplit;   // CTAs per cluster
  int *err;
  int early_dependents;  // let the next kernel launch once the partials are reduced
};

struct __align__(16) ClusterCtl {
  uint64_t full[kCMaxStages];
  uint64_t empty[kCMaxStages];
  uint64_t tmem_full;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
};

// Epilogue inputs of 4 consecutive channels n..n+3 of token m (loaded before
// the partial sums so that both latencies overlap).
struct Epi4In {
  float sx;
  float sw[4];
  uint2 b;  // 4 bf16 biases
  uint2 r;  // 4 bf16 residual values
};

template <int EPI>
__device__ __forceinline__ Epi4In load4(const ClusterGemmArgs &a, int m, int n) {
  Epi4In in = {};
  if (EPI == EPI_S32) return in;
  in.sx = a.sX[m];
  const float4 sw = __ldg(reinterpret_cast<const float4 *>(a.sW + n));
  in.sw[0] = sw.x;
  in.sw[1] = sw.y;
  in.sw[2] = sw.z;
  in.sw[3] = sw.w;
  if (EPI >= EPI_BIAS && EPI <= EPI_QKV) in.b = __ldg(reinterpret_cast<const uint2 *>(a.bias + n));
  if (EPI == EPI_RESID) in.r = *reinterpret_cast<const uint2 *>(a.R + (int64_t)m * a.ldr + n);
  return in;
}

// Epilogue of 4 consecutive channels n..n+3 (same QKV segment) of token m.
template <int EPI>
__device__ __forceinline__ void store4(const ClusterGemmArgs &a, int m, int n, const int4 &acc,
                                       const Epi4In &in) {
  const int32_t v[4] = {acc.x, acc.y, acc.z, acc.w};
  if (EPI == EPI_S32) {
    *reinterpret_cast<int4 *>(s32_row(a, m) + n) = acc;
    return;
  }
  // dequant_bf of the 4 channels as two paired bf16 conversions, then the
  // bias / residual additions of bf16 values as bf16x2 additions (bit-identical
  // to the fp32 additions rounded to bf16; see add_bf2)
  uint32_t t2[2], o2[2];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    t2[h] = pack_bf2(__fmul_rn(__fmul_rn((float)v[2 * h], in.sw[2 * h]), in.sx),
                     __fmul_rn(__fmul_rn((float)v[2 * h + 1], in.sw[2 * h + 1]), in.sx));
  const uint32_t b2[2] = {in.b.x, in.b.y}, r2[2] = {in.r.x, in.r.y};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (EPI == EPI_DEQUANT) {
      o2[h] = t2[h];
    } else if (EPI == EPI_BIAS || EPI == EPI_QKV) {
      o2[h] = add_bf2(t2[h], b2[h]);
    } else if (EPI == EPI_RESID) {
      o2[h] = add_bf2(r2[h], add_bf2(t2[h], b2[h]));
    } else {  // EPI_GELU
      const uint32_t u = add_bf2(t2[h], b2[h]);
      o2[h] = pack_bf2(gelu_tanh(__uint_as_float(u << 16)),
                       gelu_tanh(__uint_as_float(u & 0xffff0000u)));
    }
  }
  const uint2 packed = make_uint2(o2[0], o2[1]);
  uint16_t *dst;
  if (EPI == EPI_QKV) {
    const int seg = n / a.dseg, col = n - seg * a.dseg;
    if (seg == 0) {
      dst = reinterpret_cast<uint16_t *>(a.Y) + (int64_t)m * a.ldy + col;
    } else {
      const int b = m / a.T, tt = m - (m / a.T) * a.T;
      const int p = (a.pos0 ? a.pos0[b] : 0) + tt;
      dst = (seg == 1 ? a.Kc : a.Vc) + (int64_t)b * a.seq_stride + (int64_t)p * a.dseg + col;
    }
  } else {
    dst = reinterpret_cast<uint16_t *>(a.Y) + (int64_t)m * a.ldy + n;
  }
  *reinterpret_cast<uint2 *>(dst) = packed;
}

// At most 128 registers a thread: the CTA must fit on an SM beside the CTAs
// of the kernel before it, so that the weight boxes stream during its tail.
template <int EPI>
__global__ void __launch_bounds__(kCThreads, 2)
    gemm_cm_cluster_kernel(const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmX, ClusterGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int BN = a.BN, stages = a.stages;
  const uint32_t w_bytes = kCBM * kCBox, stage_bytes = w_bytes + (uint32_t)BN * kCBox;
  const uint32_t region = max((uint32_t)stages * stage_bytes, (uint32_t)BN * kCBM * 4u);
  ClusterCtl *ctl = reinterpret_cast<ClusterCtl *>(smem + region);
  // the [BN][128] int32 partial tile reuses the operand stages once the MMAs are done
  int32_t *partial = reinterpret_cast<int32_t *>(smem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tile = blockIdx.x / a.ksplit;
  const int n0 = tile * kCBM;
  const int kb0 = (int)rank * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
  const int nkb = kb1 - kb0;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)BN) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    mbar_init(&ctl->tmem_full, 1);
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
  // griddepcontrol.launch_dependents: at 64 tokens, none (the next kernel
  // launches when this grid exits): letting its CTAs become resident during
  // the GEMM made a graphed GPT-2 large decode step 15% slower, even when
  // triggered after the MMAs. At <= 32 tokens, right after the cluster
  // barrier that completes the partial tiles (a.early_dependents): steps of 8
  // and 16 sequences 1616 -> 1585 and 1742 -> 1734 us, same box, two repeats
  // (at the start of the kernel instead: slower than none).

  int issued = 0;
  const int pre = min(nkb, stages);
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < pre; ++i) {  // weights: independent of the previous kernel
      mbar_arrive_expect_tx(&ctl->full[i], stage_bytes);
      tma_load_2d(smem + (size_t)i * stage_bytes, &tmW, &ctl->full[i], (kb0 + i) * kCBox, n0);
    }
  }
  pdl_wait();  // everything below may read what the previous kernel wrote

  // This thread's share of the reduction: groups (token, 4 channels)
  // g = g0 + threadIdx.x + i * kCThreads of slice `rank`. Their epilogue
  // inputs (per-token scale, channel scales, bias, residual) are loaded now,
  // so they arrive while the MMAs run.
  const int groups = BN * (kCBM / 4);
  const int g0 = (int)((long long)groups * rank / a.ksplit);
  const int g1 = (int)((long long)groups * (rank + 1) / a.ksplit);
  const bool preloaded = g1 - g0 <= kCPre * kCThreads;  // else the plain loop below
  Epi4In pin[kCPre];
#pragma unroll
  for (int i = 0; i < kCPre; ++i) {
    pin[i] = Epi4In{};
    const int g = g0 + (int)threadIdx.x + i * kCThreads;
    if (preloaded && g < g1) {
      const int m = g >> 5, n = n0 + (g & 31) * 4;
      if (m < a.M && n < a.N) pin[i] = load4<EPI>(a, m, n);
    }
  }

  bool have_partial = false;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      uint8_t *sa = smem + (size_t)stage * stage_bytes;
      if (i >= pre) {
        if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort_flag, a.err, 0x1201)) break;
        mbar_arrive_expect_tx(&ctl->full[stage], stage_bytes);
        tma_load_2d(sa, &tmW, &ctl->full[stage], (kb0 + i) * kCBox, n0);
      }
      tma_load_2d(sa + w_bytes, &tmX, &ctl->full[stage], (kb0 + i) * kCBox, 0);
      ++issued;
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
    // On abort, give every prefetched weight box its activation box so that
    // each issued copy completes a barrier the drain below can wait on.
    for (int i = issued; i < pre; ++i, ++issued)
      tma_load_2d(smem + (size_t)i * stage_bytes + w_bytes, &tmX, &ctl->full[i],
                  (kb0 + i) * kCBox, 0);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = make_idesc(2, 1, kCBM, BN);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int consumed = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&ctl->full[stage], phase, abort_flag, a.err, 0x1202)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + (size_t)stage * stage_bytes);
      const uint32_t sb = sa + w_bytes;
#pragma unroll
      for (int k = 0; k < 4; ++k)  // 4 x 32-byte K steps inside the 128-byte swizzle atom
        tc_mma_i8(tmem_base, make_sw128_desc(sa + 32 * k), make_sw128_desc(sb + 32 * k), idesc,
                  (i != 0 || k != 0) ? 1u : 0u);
      tc_commit(&ctl->empty[stage]);
      ++consumed;
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
    ctl->consumed = consumed;
    tc_commit(&ctl->tmem_full);  // also completes after an abort: no MMA left running
  } else if (warp >= 4) {
    // ---------------- accumulator -> shared memory ----------------
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&ctl->tmem_full, 0, abort_flag, a.err, 0x1203);
    ok = __shfl_sync(0xffffffffu, ok, 0) && !*abort_flag;
    if (ok) {
      tc_fence_after();
      const int q = warp & 3;
      const int ch = q * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16);
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_row + (uint32_t)c, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) partial[(c + i) * kCBM + ch] = (int32_t)r[i];
      }
      have_partial = true;
    }
  }
  (void)have_partial;
  tc_fence_before();
  cluster_sync_all();  // every partial tile of the cluster is in shared memory
  if (a.early_dependents) pdl_launch_dependents();

  // ---------------- distributed reduction + epilogue ----------------
  // All DSMEM reads first; then the CTA tells the cluster it is done reading
  // (a peer may exit once every CTA has), and the epilogue arithmetic and
  // stores overlap that barrier. One arrive and one wait for every thread,
  // outside the branches.
  const bool run = !*abort_flag;
  int4 sum[kCPre];
#pragma unroll
  for (int i = 0; i < kCPre; ++i) sum[i] = make_int4(0, 0, 0, 0);
  if (run && preloaded) {
#pragma unroll
    for (int i = 0; i < kCPre; ++i) {
      const int g = g0 + (int)threadIdx.x + i * kCThreads;
      if (g < g1) {
        const int32_t *src = partial + (g >> 5) * kCBM + (g & 31) * 4;
        int4 p[kCMaxCluster];  // all ks loads in flight before the first addition
#pragma unroll
        for (int r = 0; r < kCMaxCluster; ++r)
          if (r < a.ksplit) p[r] = ld_dsmem_v4(dsmem_addr(src, (uint32_t)r));
#pragma unroll
        for (int r = 0; r < kCMaxCluster; ++r) {
          if (r < a.ksplit) {
            sum[i].x += p[r].x;
            sum[i].y += p[r].y;
            sum[i].z += p[r].z;
            sum[i].w += p[r].w;
          }
        }
      }
    }
  } else if (run) {
    for (int g = g0 + (int)threadIdx.x; g < g1; g += kCThreads) {
      const int tok = g >> 5, ch = (g & 31) * 4;
      const int m = tok, n = n0 + ch;
      const bool live = m < a.M && n < a.N;
      Epi4In in = {};
      if (live) in = load4<EPI>(a, m, n);
      const int32_t *src = partial + tok * kCBM + ch;
      // all ks loads in flight before the first addition
      int4 p[kCMaxCluster];
#pragma unroll
      for (int r = 0; r < kCMaxCluster; ++r)
        if (r < a.ksplit) p[r] = ld_dsmem_v4(dsmem_addr(src, (uint32_t)r));
      int4 sum = make_int4(0, 0, 0, 0);
#pragma unroll
      for (int r = 0; r < kCMaxCluster; ++r) {
        if (r < a.ksplit) {
          sum.x += p[r].x;
          sum.y += p[r].y;
          sum.z += p[r].z;
          sum.w += p[r].w;
        }
      }
      if (live) store4<EPI>(a, m, n, sum, in);
    }
  }
  cluster_arrive();  // this CTA has read every partial it needs
  if (run && preloaded) {
#pragma unroll
    for (int i = 0; i < kCPre; ++i) {
      const int g = g0 + (int)threadIdx.x + i * kCThreads;
      const int m = g >> 5, n = n0 + (g & 31) * 4;
      if (g < g1 && m < a.M && n < a.N) store4<EPI>(a, m, n, sum[i], pin[i]);
    }
  }
  cluster_wait();  // no CTA leaves while another still reads its partial tile

  if (warp == 0 && lane == 0 && *abort_flag) {
    // drain loads that were issued but never consumed by an MMA
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < issued; ++i) {
      if (i >= ctl->consumed) mbar_wait(&ctl->full[stage], phase, nullptr, a.err, 0x1204);
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

static int round_up32c(int x) { return (x + 31) & ~31; }

// Whether a decode GEMM takes the cluster path: int8, at most 128 tokens,
// 4-channel vector epilogue (N % 4, aligned rows).
bool cluster_gemm_ok(const LinearArgs &a, const void *X, int64_t ldx) {
  if (a.M < 1 || a.M > 128 || (a.N & 3) || (a.K & 15) || (ldx & 15) || !aligned16(X)) return false;
  const int esz = a.epi == EPI_S32 ? 4 : 2;
  if (((uintptr_t)a.Y & 15) || (a.ldy * esz) % 16) return false;
  if (a.epi == EPI_RESID && (((uintptr_t)a.R & 7) || (a.ldr & 3))) return false;
  if (a.epi != EPI_S32 && ((uintptr_t)a.sW & 15)) return false;
  if (a.epi >= EPI_BIAS && a.epi <= EPI_QKV && ((uintptr_t)a.bias & 7)) return false;
  if (a.epi == EPI_QKV && (((uintptr_t)a.Kc & 7) || ((uintptr_t)a.Vc & 7) || (a.dseg & 31) ||
                           (a.seq_stride & 3)))
    return false;
  return true;
}

template <int EPI>
static int launch_cluster(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &la,
                          cudaStream_t stream) {
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  ClusterGemmArgs a;
  static_cast<LinearArgs &>(a) = la;
  a.BN = round_up32c(la.M);
  a.kblocks = (la.K + kCBox - 1) / kCBox;
  const int tiles = (la.N + kCBM - 1) / kCBM;
  int ks = ctx->sm_count / tiles;
  if (ks > kCMaxCluster) ks = kCMaxCluster;
  if (ks > a.kblocks) ks = a.kblocks;
  if (ks < 1) ks = 1;
  a.kb_per = (a.kblocks + ks - 1) / ks;
  a.ksplit = (a.kblocks + a.kb_per - 1) / a.kb_per;
  a.err = ctx->err;
  a.early_dependents = la.M <= 32;
  const int stage_bytes = (kCBM + a.BN) * kCBox;
  const int budget = 227 * 1024 - 1024 - (int)sizeof(ClusterCtl) - 64;
  a.stages = a.kb_per < kCMaxStages ? a.kb_per : kCMaxStages;
  if (a.stages * stage_bytes > budget) a.stages = budget / stage_bytes;
  if (a.stages < 1) return W8A8_ERR_UNSUPPORTED;
  size_t region = (size_t)a.stages * stage_bytes;
  if (region < (size_t)a.BN * kCBM * 4) region = (size_t)a.BN * kCBM * 4;
  const size_t smem = 1024 + region + sizeof(ClusterCtl);
  if (smem > 227 * 1024) return W8A8_ERR_UNSUPPORTED;

  CUtensorMap tmW, tmX;
  st = make_tmap_2d(&tmW, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)la.N, (uint64_t)la.K,
                    (uint64_t)la.K, kCBox, kCBM);
  if (st) return st;
  st = make_tmap_2d(&tmX, X, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)la.M, (uint64_t)la.K,
                    (uint64_t)ldx, kCBox, (uint32_t)a.BN);
  if (st) return st;

  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_cm_cluster_kernel<EPI>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return W8A8_ERR_CUDA;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * a.ksplit);
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.ksplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, gemm_cm_cluster_kernel<EPI>, tmW, tmX, a) != cudaSuccess) {
    cudaGetLastError();
    return W8A8_ERR_CUDA;
  }
  return check_launch("gemm_cm_cluster");
}

int gemm_cluster_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
                    cudaStream_t stream) {
  switch (a.epi) {
    case EPI_S32: return launch_cluster<EPI_S32>(W, X, ldx, a, stream);
    case EPI_DEQUANT: return launch_cluster<EPI_DEQUANT>(W, X, ldx, a, stream);
    case EPI_BIAS: return launch_cluster<EPI_BIAS>(W, X, ldx, a, stream);
    case EPI_RESID: return launch_cluster<EPI_RESID>(W, X, ldx, a, stream);
    case EPI_GELU: return launch_cluster<EPI_GELU>(W, X, ldx, a, stream);
    case EPI_QKV: return launch_cluster<EPI_QKV>(W, X, ldx, a, stream);
    default: return W8A8_ERR_INVALID;
  }
}

}  // namespace w8a8
