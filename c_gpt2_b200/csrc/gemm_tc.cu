// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
// Y[m, n] = epilogue(sum_k X[m, k] * W[n, k]) with both operands K-major,
// exactly as the reference stores them (W [OUT, IN], activations
// [tokens, IN]). Two orientations of the same pipeline:
//
//   token-major (prefill, M > 128): A = 128 token rows, B = BN weight rows.
//     TMEM lane = token, columns = output channels. Each epilogue warp turns
//     its 32 x 16 blocks into whole-sector coalesced stores (and residual
//     loads) through a 1 KiB shared buffer; see epilogue_tm.
//   channel-major (decode, M <= 128): A = 128 weight rows, B = the BN tokens
//     of the batch (16..128). When the output tiles alone cannot occupy the
//     GPU the reduction is split over K; partial int32 sums meet in a
//     workspace through integer atomics (exact in any order) and the last
//     split of a tile, found by a ticket counter, runs the epilogue.
//
// Roles: warp 0 TMA producer (128-byte swizzled boxes, no multicast),
// warp 1 TMEM allocator + single-thread MMA issuer (kind::i8 -> s32, or
// kind::f16 with bf16 operands -> f32 for the LM head), warps 2..17 the
// epilogue (4 warps per TMEM lane quarter, splitting the 32-column chunks).
// In token-major residual GEMMs the TMA warp also pulls the next tile's
// residual block into L2 (one tensor-map prefetch per tile).
// The accumulator is double-buffered in TMEM so the epilogue of one tile
// overlaps the main loop of the next. Every wait is bounded: a stalled
// pipeline records an error code and the kernel returns.
//
// Token-major INT8 GEMMs with at least 256 output channels and K > 4608 run
// on CTA pairs instead (gemm_tc_pair_kernel): one tcgen05.mma.cta_group::2
// per K step covers 256 tokens x 256 channels, each CTA loading half of both
// operands, with the same epilogue per CTA.
//
// Replaces the reference's cublasGemmEx INT8 call (gpt2.c:404-415), its
// dequant kernel (cuda/activation_quant.cu:117-131) and the add_bias /
// add_2d / gelu kernels that follow each GEMM (gpt2.c:1145-1325), and the
// bf16 LM-head GEMM (gpt2.c:2160).
#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

constexpr int kBM = 128;        // rows of the A tile (MMA M)
constexpr int kBoxBytes = 128;  // K bytes per stage (one 128-byte swizzle atom)
constexpr int kEpiWarps = 16;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;
constexpr int kEpiWarp0 = 2;
constexpr int kEpiBarrier = 1;  // named barrier id of the epilogue warps

struct GemmArgs : LinearArgs {
  int BN;                // rows of the B tile (multiple of 32, <= 256)
  int stages;
  int a_tiles, b_tiles;  // 128-row A tiles x BN-row B tiles
  int kblocks;           // ceil(K bytes / 128)
  int ksplit, kb_per;    // split-K (channel-major only)
  int32_t *ws;           // [M][N] int32 partial sums, zero between calls
  int *tickets;          // one per tile
  int *err;
  int vec_params;        // sW and bias 16-byte aligned (token-major epilogue)
};

struct __align__(16) SmemCtl {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;    // k-iterations consumed by the MMA thread (for abort drain)
  int last_flag;   // split-K: this CTA holds the last partial of the tile
  int vote[2][kEpiWarps];
  uint64_t rbar[kEpiWarps][3];  // residual slots of each epilogue warp (RT mode)
};

// ---------------------------------------------------------------------------
// channel-major epilogue: one output channel n per thread, r[i] = token mbase+i
// (W = 16 consecutive tokens of the TMEM accumulator)
// ---------------------------------------------------------------------------
template <int EPI>
__device__ __forceinline__ void store_one_cm(const GemmArgs &a, int m, int n, int32_t acc,
                                             float sw, float sx, float bias, uint16_t rv,
                                             int qseg, int qcol, int64_t kv) {
  uint16_t *Yb = reinterpret_cast<uint16_t *>(a.Y);
  if (EPI == EPI_S32) {
    s32_row(a, m)[n] = acc;
  } else if (EPI == EPI_DEQUANT) {
    Yb[(int64_t)m * a.ldy + n] = f2bf(dequant_bf(acc, sw, sx));
  } else if (EPI == EPI_BIAS) {
    Yb[(int64_t)m * a.ldy + n] = f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bias));
  } else if (EPI == EPI_RESID) {
    const float y = add_bf(dequant_bf(acc, sw, sx), bias);
    Yb[(int64_t)m * a.ldy + n] = f2bf(__fadd_rn(bf2f(rv), y));
  } else if (EPI == EPI_GELU) {
    const float y = add_bf(dequant_bf(acc, sw, sx), bias);
    Yb[(int64_t)m * a.ldy + n] = f2bf(gelu_tanh(y));
  } else if (EPI == EPI_QKV) {
    const uint16_t v = f2bf(__fadd_rn(dequant_bf(acc, sw, sx), bias));
    if (qseg == 0)
      Yb[(int64_t)m * a.ldy + qcol] = v;
    else
      (qseg == 1 ? a.Kc : a.Vc)[kv + qcol] = v;
  } else {  // EPI_F32_BF16
    Yb[(int64_t)m * a.ldy + n] = f2bf(__int_as_float(acc));
  }
}

template <int EPI>
__device__ __forceinline__ int64_t qkv_row_offset(const GemmArgs &a, int m) {
  const int b = m / a.T, t = m - (m / a.T) * a.T;
  const int p = (a.pos0 ? a.pos0[b] : 0) + t;
  return (int64_t)b * a.seq_stride + (int64_t)p * a.dseg;
}

template <int EPI>
__device__ __forceinline__ void finish_chunk_cm(const GemmArgs &a, int n, bool n_ok, float sw,
                                                float bias, int qseg, int qcol, int mbase,
                                                const uint32_t (&r)[16], int lane) {
  // per-token values fetched lane-parallel (lanes 0..15) and broadcast
  const int m_lane = mbase + (lane & 15);
  const bool m_lane_ok = m_lane < a.M;
  float sx_lane = 0.f;
  if (EPI != EPI_S32 && EPI != EPI_F32_BF16 && m_lane_ok) sx_lane = a.sX[m_lane];
  int64_t kv_lane = 0;
  if (EPI == EPI_QKV && m_lane_ok) kv_lane = qkv_row_offset<EPI>(a, m_lane);
  uint16_t rv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) rv[i] = 0;
  if (EPI == EPI_RESID) {
    // every residual value of the chunk in flight before the first store
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n_ok && mbase + i < a.M) rv[i] = a.R[(int64_t)(mbase + i) * a.ldr + n];
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float sx = __shfl_sync(0xffffffffu, sx_lane, i);
    const int64_t kv = EPI == EPI_QKV ? __shfl_sync(0xffffffffu, kv_lane, i) : 0;
    const int m = mbase + i;
    if (n_ok && m < a.M)
      store_one_cm<EPI>(a, m, n, (int32_t)r[i], sw, sx, bias, rv[i], qseg, qcol, kv);
  }
}

// Split-K: the last unit of a tile reads the summed int32 tile back from the
// workspace, re-zeroes it, and applies the epilogue. The tile is spread over
// all epilogue threads (thread -> channel tid % 128, tokens (tid / 128) + 4j)
// with every load of a batch in flight together.
template <int EPI>
__device__ __forceinline__ void final_from_ws(const GemmArgs &a, int n0, int m0, int etid) {
  const int n = n0 + (etid & 127);
  if (n >= a.N) return;
  float sw = 0.f, bias = 0.f;
  int qseg = 0, qcol = n;
  if (EPI != EPI_S32 && EPI != EPI_F32_BF16) sw = a.sW[n];
  if (EPI >= EPI_BIAS && EPI <= EPI_QKV) bias = bf2f(a.bias[n]);
  if (EPI == EPI_QKV) {
    qseg = n / a.dseg;
    qcol = n - qseg * a.dseg;
  }
  const int mq = etid >> 7;  // 0..3
  const int per = a.BN >> 2;
  for (int j0 = 0; j0 < per; j0 += 16) {
    int32_t v[16];
    float sxv[16];
    uint16_t rv[16];
    int64_t kvv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int m = m0 + mq + 4 * (j0 + j);
      const bool ok = (j0 + j < per) && m < a.M;
      v[j] = ok ? __ldcg(a.ws + (int64_t)m * a.N + n) : 0;
      sxv[j] = (ok && EPI != EPI_S32 && EPI != EPI_F32_BF16) ? a.sX[m] : 0.f;
      rv[j] = (ok && EPI == EPI_RESID) ? a.R[(int64_t)m * a.ldr + n] : (uint16_t)0;
      kvv[j] = (ok && EPI == EPI_QKV) ? qkv_row_offset<EPI>(a, m) : 0;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int m = m0 + mq + 4 * (j0 + j);
      if ((j0 + j < per) && m < a.M) {
        a.ws[(int64_t)m * a.N + n] = 0;
        store_one_cm<EPI>(a, m, n, v[j], sw, sxv[j], bias, rv[j], qseg, qcol, kvv[j]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// token-major epilogue, int32 output (tensor-parallel partial sums): one token
// row m per thread, r[j] = channel nbase+j, written to the (possibly remote)
// row of s32_row().
// ---------------------------------------------------------------------------
__device__ __forceinline__ void finish_chunk_tm_s32(const GemmArgs &a, int m, int nbase,
                                                    const uint32_t (&r)[32]) {
  if (m >= a.M || nbase >= a.N) return;
  int4 *dst = reinterpret_cast<int4 *>(s32_row(a, m) + nbase);
#pragma unroll
  for (int v = 0; v < 8; ++v)
    dst[v] = make_int4((int)r[4 * v], (int)r[4 * v + 1], (int)r[4 * v + 2], (int)r[4 * v + 3]);
}

// ---------------------------------------------------------------------------
// token-major epilogue, bf16 outputs (DEQUANT, BIAS, RESID, GELU, QKV).
//
// Each epilogue warp owns TMEM lanes [32*quarter, +32) (32 token rows) and,
// of every 128 x BN tile, the 16-column halves of chunks `group` and
// `group + 4`: four items per tile. Per item the warp
//   - reads its 32 x 16 accumulators (a lane per token row),
//   - reads the residual block with two coalesced 16-byte loads per lane
//     (two lanes per row, sixteen rows per instruction), issued one item
//     ahead, and turns it into a lane-per-row layout through its 1 KiB
//     shared-memory buffer,
//   - computes 16 bf16 outputs per row into the same buffer, and
//   - stores the 32 x 32-byte block with two coalesced 16-byte stores per
//     lane, whole 32-byte sectors.
// Channel scales and biases are warp-uniform vector loads; the per-token
// scale (and the QKV cache row) of the next tile is loaded a tile ahead.
// There is no barrier between the epilogue warps.
// ---------------------------------------------------------------------------
constexpr int kStageRowBytes = 32;                    // 16 bf16 of one token row
constexpr int kWarpStageBytes = 32 * kStageRowBytes;  // 1 KiB output / residual block
// channel scales (fp32) and biases (bf16) of the warp's 64 columns of a tile,
// double-buffered so the next tile's are copied while this tile's are used
constexpr int kParamBytes = 64 * 4 + 64 * 2;
constexpr int kWarpEpiBytes = kWarpStageBytes + 2 * kParamBytes;
constexpr int kEpiStageBytes = kEpiWarps * kWarpEpiBytes;  // 28 KiB
// Residual by TMA (RT mode, residual GEMMs with short K): per warp three 1 KiB
// residual slots, then the output buffer and the parameter buffers.
constexpr int kRSlots = 3;
constexpr int kWarpEpiBytesRT = 5 * 1024;
constexpr int kEpiStageBytesRT = kEpiWarps * kWarpEpiBytesRT;  // 80 KiB

// Byte offset of 16-byte half h of row r in a warp's buffer. The half is
// flipped on rows 4..7 of every 8, which makes both access patterns below
// (a lane per row; two lanes per row over sixteen rows) free of bank conflicts.
__device__ __forceinline__ uint32_t stage_off(int r, int h) {
  return (uint32_t)(r * kStageRowBytes + ((h ^ ((r >> 2) & 1)) << 4));
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Copy the channel scales and biases of the warp's two 32-column chunks of
// tile t into its parameter buffer: [64] fp32 scales, then [64] bf16 biases.
template <int EPI>
__device__ __forceinline__ void tm_load_params(const GemmArgs &a, int t, int group, int lane,
                                               uint32_t buf, bool vec) {
  const int b0 = (t % a.b_tiles) * a.BN;
#pragma unroll
  for (int cs = 0; cs < 2; ++cs) {
    const int col0 = 32 * (group + 4 * cs), n0 = b0 + col0;
    if (col0 >= a.BN || n0 >= a.N) continue;  // N % 32 == 0: a live chunk is whole
    if (vec) {
      if (lane < 8)
        cp_async16(buf + (uint32_t)((32 * cs + 4 * lane) * 4), a.sW + n0 + 4 * lane);
      else if (lane < 12 && EPI != EPI_DEQUANT)
        cp_async16(buf + 256u + (uint32_t)((32 * cs + 8 * (lane - 8)) * 2),
                   a.bias + n0 + 8 * (lane - 8));
    } else {
      const float w = a.sW[n0 + lane];
      const uint16_t bb = EPI != EPI_DEQUANT ? a.bias[n0 + lane] : (uint16_t)0;
      asm volatile("st.shared.f32 [%0], %1;" ::"r"(buf + (uint32_t)((32 * cs + lane) * 4)),
                   "f"(w) : "memory");
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(buf + 256u + (uint32_t)((32 * cs + lane) * 2)),
                   "h"(bb) : "memory");
    }
  }
  cp_async_commit();
}

// Column offset (within the tile) of item j of an epilogue warp of `group`.
__device__ __forceinline__ int tm_item_col(int group, int j) {
  return 32 * (group + 4 * (j >> 1)) + 16 * (j & 1);
}

// Geometry of one tile for one epilogue lane, computed once per tile. The
// lane moves two 16-byte pieces per item: rows (lane >> 1) and 16 + (lane >> 1)
// of the warp's 32, half (lane & 1) of the item's 16 columns.
struct TmTile {
  int a0, b0;
  int64_t rpiece;          // element offset of piece 0 in R (without the column)
  bool ok0, ok1;           // the pieces' rows are inside M
  bool live0, live1;       // chunk slots group and group + 4 exist in this tile
};

__device__ __forceinline__ TmTile tm_tile(const GemmArgs &a, int t, int quarter, int group,
                                          int lane) {
  TmTile g;
  const int ta = t / a.b_tiles;
  g.a0 = ta * kBM;
  g.b0 = (t - ta * a.b_tiles) * a.BN;
  const int r0 = g.a0 + 32 * quarter + (lane >> 1);
  g.ok0 = r0 < a.M;
  g.ok1 = r0 + 16 < a.M;
  g.rpiece = (int64_t)r0 * a.ldr + 8 * (lane & 1);
  const int c0 = 32 * group, c1 = 32 * (group + 4);
  g.live0 = c0 < a.BN && g.b0 + c0 < a.N;  // N % 32 == 0: a live chunk is whole
  g.live1 = c1 < a.BN && g.b0 + c1 < a.N;
  return g;
}

// Residual pieces of item j of tile g (zeros where there is nothing to read).
template <int EPI>
__device__ __forceinline__ void tm_load_resid(const GemmArgs &a, const TmTile &g, int group, int j,
                                              uint4 (&rp)[2]) {
  rp[0] = rp[1] = make_uint4(0, 0, 0, 0);
  if (EPI != EPI_RESID || !((j >> 1) ? g.live1 : g.live0)) return;
  const uint16_t *p = a.R + g.rpiece + g.b0 + tm_item_col(group, j);
  if (g.ok0) rp[0] = __ldcs(reinterpret_cast<const uint4 *>(p));
  if (g.ok1) rp[1] = __ldcs(reinterpret_cast<const uint4 *>(p + 16 * a.ldr));
}

// Copy the channel scales and biases of the warp's two 32-column chunks of
// tile g into its parameter buffer: [64] fp32 scales, then [64] bf16 biases.
template <int EPI>
__device__ __forceinline__ void tm_load_params(const GemmArgs &a, const TmTile &g, int group,
                                               int lane, uint32_t buf, bool vec) {
#pragma unroll
  for (int cs = 0; cs < 2; ++cs) {
    if (!(cs ? g.live1 : g.live0)) continue;
    const int n0 = g.b0 + 32 * (group + 4 * cs);
    if (vec) {
      if (lane < 8)
        cp_async16(buf + (uint32_t)((32 * cs + 4 * lane) * 4), a.sW + n0 + 4 * lane);
      else if (lane < 12 && EPI != EPI_DEQUANT)
        cp_async16(buf + 256u + (uint32_t)((32 * cs + 8 * (lane - 8)) * 2),
                   a.bias + n0 + 8 * (lane - 8));
    } else {
      const float w = a.sW[n0 + lane];
      const uint16_t bb = EPI != EPI_DEQUANT ? a.bias[n0 + lane] : (uint16_t)0;
      asm volatile("st.shared.f32 [%0], %1;" ::"r"(buf + (uint32_t)((32 * cs + lane) * 4)),
                   "f"(w) : "memory");
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(buf + 256u + (uint32_t)((32 * cs + lane) * 2)),
                   "h"(bb) : "memory");
    }
  }
  cp_async_commit();
}

// Per-token scale (and QKV cache-row offset) of this lane's own row of tile g.
template <int EPI>
__device__ __forceinline__ void tm_row_info(const GemmArgs &a, const TmTile &g, int quarter,
                                            int lane, float &sx, int64_t &kv) {
  sx = 0.f;
  kv = 0;
  const int m = g.a0 + 32 * quarter + lane;
  if (m >= a.M) return;
  sx = a.sX[m];
  if (EPI == EPI_QKV) kv = qkv_row_offset<EPI>(a, m);
}

// RT mode: lane 0 requests item j's 32 x 16 residual block into a slot by TMA
// (the 32-byte swizzle lays it out as stage_off does); an item without
// columns (a partial tile) completes the slot's phase without data.
__device__ __forceinline__ void tm_issue_resid(const CUtensorMap *tmRb, uint64_t *bar,
                                               uint32_t slot, const TmTile &g, int quarter,
                                               int group, int j) {
  if (!((j >> 1) ? g.live1 : g.live0)) {
    mbar_arrive(bar);
    return;
  }
  mbar_arrive_expect_tx(bar, (uint32_t)kWarpStageBytes);
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(slot),
      "l"(tmRb), "r"(smem_u32(bar)), "r"(g.b0 + tm_item_col(group, j)), "r"(g.a0 + 32 * quarter)
      : "memory");
}

// Units of the epilogue loop. One CTA: unit = 128 x BN tile, CTAs stride the
// grid. CTA pair: unit = 256-row x BN tile pair, clusters stride the grid, and
// CTA `rank` of the pair finishes the 128-row tile 2 * (unit / b_tiles) + rank.
template <bool PAIR>
struct TmUnits {
  int first, stride, total, rank;
  __device__ __forceinline__ TmUnits(const GemmArgs &a) {
    if (PAIR) {
      rank = (int)cluster_ctarank();
      first = (int)(blockIdx.x >> 1);
      stride = (int)(gridDim.x >> 1);
      total = ((a.a_tiles + 1) >> 1) * a.b_tiles;
    } else {
      rank = 0;
      first = (int)blockIdx.x;
      stride = (int)gridDim.x;
      total = a.a_tiles * a.b_tiles;
    }
  }
  __device__ __forceinline__ int tile(const GemmArgs &a, int u) const {
    if (!PAIR) return u;
    const int pm = u / a.b_tiles;
    return (2 * pm + rank) * a.b_tiles + (u - pm * a.b_tiles);
  }
};

template <int EPI, bool RT, bool PAIR = false>
__device__ __forceinline__ void epilogue_tm(const GemmArgs &a, SmemCtl *ctl, uint32_t tmem_base,
                                            uint32_t wbase, int e, int lane,
                                            volatile int *abort_flag, bool vec_params,
                                            const CUtensorMap *tmRb) {
  const int quarter = (e + kEpiWarp0) & 3, group = e >> 2;
  const TmUnits<PAIR> units(a);
  const int total_units = units.total;
  // a pair's accumulators are handed back to the MMA issuer of the even CTA
  const uint32_t empty_at[2] = {PAIR ? dsmem_addr(&ctl->tmem_empty[0], 0) : 0u,
                                PAIR ? dsmem_addr(&ctl->tmem_empty[1], 0) : 0u};
  // output (and, without RT, residual) buffer; RT: the residual slots first
  const uint32_t stage = RT ? wbase + (uint32_t)(kRSlots * kWarpStageBytes) : wbase;
  const uint32_t params = stage + kWarpStageBytes;  // two buffers of kParamBytes
  int acc = 0;
  uint32_t acc_phase = 0;
  // residual pieces of the next two items (items run 0..3 within a tile,
  // then on to the CTA's next tile); RT: items issued / consumed
  uint4 rp[2], rq[2];
  int r_issued = 0, r_used = 0;
  float sx_next = 0.f;
  int64_t kv_next = 0;
  TmTile gn = {};
  if (units.first < total_units) {
    gn = tm_tile(a, units.tile(a, units.first), quarter, group, lane);
    tm_load_params<EPI>(a, gn, group, lane, params, vec_params);
    if (RT) {
      if (lane == 0)
        for (int j = 0; j < 2; ++j)
          tm_issue_resid(tmRb, &ctl->rbar[e][j], wbase + (uint32_t)(j * kWarpStageBytes), gn,
                         quarter, group, j);
      r_issued = 2;
    } else {
      tm_load_resid<EPI>(a, gn, group, 0, rp);
      tm_load_resid<EPI>(a, gn, group, 1, rq);
    }
    tm_row_info<EPI>(a, gn, quarter, lane, sx_next, kv_next);
  }
  int iter = 0;
  for (int u = units.first; u < total_units; u += units.stride, ++iter) {
    const TmTile g = gn;
    const bool has_next = u + units.stride < total_units;
    if (has_next) gn = tm_tile(a, units.tile(a, u + units.stride), quarter, group, lane);
    const uint32_t pbuf = params + (uint32_t)((iter & 1) * kParamBytes);
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&ctl->tmem_full[acc], acc_phase, abort_flag, a.err, 0x1105);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) break;
    mbar_wait(&ctl->tmem_full[acc], acc_phase, nullptr, a.err, 0x1107);  // completed: returns at once
    tc_fence_after();
    const float sx = sx_next;
    const int64_t kv_own = kv_next;
    cp_async_wait_all();  // this tile's parameters
    __syncwarp();
    if (has_next) {
      tm_row_info<EPI>(a, gn, quarter, lane, sx_next, kv_next);
      tm_load_params<EPI>(a, gn, group, lane,
                          params + (uint32_t)(((iter + 1) & 1) * kParamBytes), vec_params);
    }
    // cache-row offsets of the two rows this lane stores (QKV)
    int64_t kvp[2] = {0, 0};
    if (EPI == EPI_QKV) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        kvp[i] = __shfl_sync(0xffffffffu, kv_own, (lane >> 1) + 16 * i) + 8 * (lane & 1);
    }
    const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * a.BN);
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      const int jcol = tm_item_col(group, j);
      const int n = g.b0 + jcol;
      const bool live = (j >> 1) ? g.live1 : g.live0;  // warp-uniform
      uint32_t r[16];
      float sw[16];
      uint32_t bias2[8];
      if (live) {
        tmem_ld_32x32b_x16(t_row + (uint32_t)jcol, r);
        if (EPI == EPI_RESID && !RT) {  // this item's residual pieces into the row buffer
#pragma unroll
          for (int i = 0; i < 2; ++i)
            st_shared_v4(stage + stage_off((lane >> 1) + 16 * i, lane & 1), rp[i]);
        }
      }
      if (RT) {
        // refill the slot read by the previous item with the item two ahead:
        // every lane's reads of it before the asynchronous write
        if (j < 2 || has_next) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int q = r_issued % kRSlots;
            tm_issue_resid(tmRb, &ctl->rbar[e][q], wbase + (uint32_t)(q * kWarpStageBytes),
                           j < 2 ? g : gn, quarter, group, j < 2 ? j + 2 : j - 2);
          }
          ++r_issued;
        }
      } else {
        rp[0] = rq[0];
        rp[1] = rq[1];
        if (j < 2)
          tm_load_resid<EPI>(a, g, group, j + 2, rq);
        else if (has_next)
          tm_load_resid<EPI>(a, gn, group, j - 2, rq);
      }
      if (live) {
        const uint32_t pi = (uint32_t)(32 * (j >> 1) + 16 * (j & 1));  // column in the buffer
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint4 x = ld_shared_v4(pbuf + (pi + 4 * v) * 4);
          sw[4 * v] = __uint_as_float(x.x);
          sw[4 * v + 1] = __uint_as_float(x.y);
          sw[4 * v + 2] = __uint_as_float(x.z);
          sw[4 * v + 3] = __uint_as_float(x.w);
        }
        if (EPI != EPI_DEQUANT) {
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const uint4 x = ld_shared_v4(pbuf + 256u + (pi + 8 * v) * 2);
            bias2[4 * v] = x.x;
            bias2[4 * v + 1] = x.y;
            bias2[4 * v + 2] = x.z;
            bias2[4 * v + 3] = x.w;
          }
        }
        tmem_ld_wait();
      }
      if (j == 3) {  // the tile's accumulator is read: hand it back to the MMA warp
        tc_fence_before();
        if (PAIR) {  // one arrival per warp, on the even CTA's barrier
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(empty_at[acc]);
        } else {
          mbar_arrive(&ctl->tmem_empty[acc]);
        }
      }
      uint4 rown[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (RT) {  // this item's slot (its phase completes even for an item without columns)
        const int q = r_used % kRSlots;
        mbar_wait(&ctl->rbar[e][q], (uint32_t)((r_used / kRSlots) & 1), nullptr, a.err, 0x1108);
        ++r_used;
        if (live) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            rown[h] = ld_shared_v4(wbase + (uint32_t)(q * kWarpStageBytes) + stage_off(lane, h));
        }
      }
      if (!live) continue;
      if (EPI == EPI_RESID && !RT) {  // the residual of this lane's own row
        __syncwarp();
#pragma unroll
        for (int h = 0; h < 2; ++h) rown[h] = ld_shared_v4(stage + stage_off(lane, h));
      }
      // Same operations and rounding points as dequant_bf / add_bf / f2bf,
      // on pairs of channels: t = bf16(y) by one paired conversion, then the
      // bias and residual additions of bf16 values as bf16x2 additions.
      uint32_t packed[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float y0 = __fmul_rn(__fmul_rn((float)(int32_t)r[i], sw[i]), sx);
        const float y1 = __fmul_rn(__fmul_rn((float)(int32_t)r[i + 1], sw[i + 1]), sx);
        const uint32_t t2 = pack_bf2(y0, y1);  // dequant_bf of both
        if (EPI == EPI_DEQUANT) {
          packed[i >> 1] = t2;
        } else if (EPI == EPI_BIAS || EPI == EPI_QKV) {
          packed[i >> 1] = add_bf2(t2, bias2[i >> 1]);
        } else if (EPI == EPI_RESID) {
          packed[i >> 1] = add_bf2((&rown[0].x)[i >> 1], add_bf2(t2, bias2[i >> 1]));
        } else {  // EPI_GELU
          const uint32_t u2 = add_bf2(t2, bias2[i >> 1]);
          packed[i >> 1] = pack_bf2(gelu_tanh(__uint_as_float(u2 << 16)),
                                    gelu_tanh(__uint_as_float(u2 & 0xffff0000u)));
        }
      }
      st_shared_v4(stage + stage_off(lane, 0), make_uint4(packed[0], packed[1], packed[2], packed[3]));
      st_shared_v4(stage + stage_off(lane, 1), make_uint4(packed[4], packed[5], packed[6], packed[7]));
      __syncwarp();
      uint16_t *dst0, *dst1;  // this lane's two 16-byte pieces of the item
      const int64_t ypiece = (int64_t)(g.a0 + 32 * quarter + (lane >> 1)) * a.ldy + 8 * (lane & 1);
      if (EPI == EPI_QKV) {
        const int seg = n / a.dseg;
        const int64_t col = n - (int64_t)seg * a.dseg;
        if (seg == 0) {
          uint16_t *y = reinterpret_cast<uint16_t *>(a.Y) + ypiece + col;
          dst0 = y;
          dst1 = y + 16 * a.ldy;
        } else {
          uint16_t *c = (seg == 1 ? a.Kc : a.Vc) + col;
          dst0 = c + kvp[0];
          dst1 = c + kvp[1];
        }
      } else {
        dst0 = reinterpret_cast<uint16_t *>(a.Y) + ypiece + n;
        dst1 = dst0 + 16 * a.ldy;
      }
      const uint4 v0 = ld_shared_v4(stage + stage_off(lane >> 1, lane & 1));
      const uint4 v1 = ld_shared_v4(stage + stage_off(16 + (lane >> 1), lane & 1));
      if (g.ok0) *reinterpret_cast<uint4 *>(dst0) = v0;
      if (g.ok1) *reinterpret_cast<uint4 *>(dst1) = v1;
      __syncwarp();  // the buffer is rewritten by the next item
    }
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1;
    }
  }
  cp_async_wait_all();  // no copy into shared memory outlives the loop
  if (RT) {             // nor a residual load (only after an abort are any left)
    for (; r_used < r_issued; ++r_used)
      mbar_wait(&ctl->rbar[e][r_used % kRSlots], (uint32_t)((r_used / kRSlots) & 1), nullptr,
                a.err, 0x1109);
    __syncwarp();
  }
}

template <int KIND, int EPI, bool CM, bool RT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmRb,
                   GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int BN = a.BN;
  const int stages = a.stages;
  const uint32_t a_bytes = kBM * kBoxBytes;
  const uint32_t b_bytes = (uint32_t)BN * kBoxBytes;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  // [stages][A box | B box] | token-major bf16: epilogue buffers | SmemCtl
  constexpr bool kStaged = !CM && EPI != EPI_S32;
  uint8_t *epi_stage = smem + (size_t)stages * stage_bytes;
  SmemCtl *ctl = reinterpret_cast<SmemCtl *>(
      epi_stage + (kStaged ? (RT ? kEpiStageBytesRT : kEpiStageBytes) : 0));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_units = a.a_tiles * a.b_tiles * a.ksplit;
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * BN)) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->tmem_full[i], 1);
      mbar_init(&ctl->tmem_empty[i], kEpiThreads);
    }
    mbar_init(&ctl->drain, 1);
    if (RT)
      for (int w = 0; w < kEpiWarps; ++w)
        for (int q = 0; q < kRSlots; ++q) mbar_init(&ctl->rbar[w][q], 1);
    ctl->abort_flag = 0;
    ctl->consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (!CM && EPI == EPI_RESID) prefetch_tmap(&tmR);
    if (RT) prefetch_tmap(&tmRb);
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

  // No early griddepcontrol.launch_dependents: the next kernel launches when
  // this grid exits. Measured on a graphed decode step of GPT-2 large (64
  // sequences), letting the next kernel's CTAs become resident during the GEMM
  // made the step 15% slower, even when triggered after the MMAs.
  int issued = 0;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    // The weight operand does not depend on the previous kernel: the boxes of
    // the first unit's first stages are issued before waiting for it
    // (programmatic dependent launch), so they stream while it finishes.
    const int kbox = kBoxBytes / (KIND == 0 ? 1 : 2);
    const CUtensorMap *tmW = CM ? &tmA : &tmB;
    const CUtensorMap *tmX = CM ? &tmB : &tmA;
    const uint32_t w_off = CM ? 0u : a_bytes, x_off = CM ? a_bytes : 0u;
    int pre = 0, pre_kb0 = 0, pre_x = 0, pre_w = 0;
    if ((int)blockIdx.x < total_units) {
      const int u = blockIdx.x;
      const int t = u / a.ksplit, ks = u - (u / a.ksplit) * a.ksplit;
      const int a0 = (t / a.b_tiles) * kBM, b0 = (t % a.b_tiles) * BN;
      pre_kb0 = ks * a.kb_per;
      const int kb1 = min(a.kblocks, pre_kb0 + a.kb_per);
      pre_w = CM ? a0 : b0;
      pre_x = CM ? b0 : a0;
      for (int kb = pre_kb0; kb < kb1 && pre < stages; ++kb, ++pre) {
        uint8_t *sa = smem + (size_t)pre * stage_bytes;
        mbar_arrive_expect_tx(&ctl->full[pre], stage_bytes);
        tma_load_2d(sa + w_off, tmW, &ctl->full[pre], kb * kbox, pre_w);
      }
    }
    pdl_wait();
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    for (int u = blockIdx.x; u < total_units && !*abort_flag; u += gridDim.x) {
      const int t = u / a.ksplit, ks = u - (u / a.ksplit) * a.ksplit;
      const int a0 = (t / a.b_tiles) * kBM;
      const int b0 = (t % a.b_tiles) * BN;
      const int kb0 = ks * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
      if (!CM && EPI == EPI_RESID && u + (int)gridDim.x < total_units) {
        // the residual block of this CTA's next tile: into L2 now, so the
        // epilogue's loads of it hit L2 instead of waiting on DRAM
        const int un = u + gridDim.x;
        tma_prefetch_l2_2d(&tmR, (un % a.b_tiles) * BN, (un / a.b_tiles) * kBM);
      }
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort_flag, a.err, 0x1101)) break;
        uint8_t *sa = smem + (size_t)stage * stage_bytes;
        if (it >= pre) {
          mbar_arrive_expect_tx(&ctl->full[stage], stage_bytes);
          tma_load_2d(sa + w_off, tmW, &ctl->full[stage], kb * kbox, CM ? a0 : b0);
        }
        tma_load_2d(sa + x_off, tmX, &ctl->full[stage], kb * kbox, CM ? b0 : a0);
        ++it;
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // On abort, complete any prefetched stage whose activation box was never
    // issued, so every issued copy has a barrier to drain on below.
    for (; it < pre; ++it, ++issued)
      tma_load_2d(smem + (size_t)it * stage_bytes + x_off, tmX, &ctl->full[it],
                  (pre_kb0 + it) * kbox, pre_x);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    pdl_wait();
    const uint32_t idesc = KIND == 0 ? make_idesc(2, 1, kBM, BN) : make_idesc(1, 1, kBM, BN);
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
  } else if (kStaged && warp >= kEpiWarp0) {
    // ---------------- epilogue (token-major, bf16) ----------------
    pdl_wait();
    const int e = warp - kEpiWarp0;
    epilogue_tm<EPI, RT>(a, ctl, tmem_base,
                         smem_u32(epi_stage) + (uint32_t)(e * (RT ? kWarpEpiBytesRT : kWarpEpiBytes)),
                         e, lane, abort_flag, a.vec_params != 0, &tmRb);
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue ----------------
    pdl_wait();
    const int e = warp - kEpiWarp0;     // 0..15
    const int quarter = warp & 3;       // TMEM lanes [32*quarter, 32*quarter+32)
    const int group = e >> 2;           // chunks c == group (mod 4)
    const int nchunks = BN >> 5;
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
      const int t = u / a.ksplit;
      // Warp-uniform bounded wait, then a vote of all epilogue warps, so the
      // named barriers below always see every epilogue thread.
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&ctl->tmem_full[acc], acc_phase, abort_flag, a.err, 0x1105);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane == 0) ctl->vote[iter & 1][e] = ok;
      named_barrier_sync(kEpiBarrier, kEpiThreads);
#pragma unroll
      for (int w = 0; w < kEpiWarps; ++w) ok &= ctl->vote[iter & 1][w];
      ++iter;
      if (!ok) break;
      mbar_wait(&ctl->tmem_full[acc], acc_phase, nullptr, a.err, 0x1107);  // completed: returns at once
      tc_fence_after();
      const int a0 = (t / a.b_tiles) * kBM;
      const int b0 = (t % a.b_tiles) * BN;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      if (!CM) {
        // token-major int32 (only EPI_S32 reaches this branch)
        const int m = a0 + quarter * 32 + lane;
        for (int c = group; c < nchunks; c += 4) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(32 * c), r);
          tmem_ld_wait();
          finish_chunk_tm_s32(a, m, b0 + 32 * c, r);
        }
        tc_fence_before();
        mbar_arrive(&ctl->tmem_empty[acc]);
      } else {
        const int n = a0 + quarter * 32 + lane;
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
        if (a.ksplit == 1) {
          for (int c = group; c < 2 * nchunks; c += 4) {  // 16-token chunks
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_row + (uint32_t)(16 * c), r);
            tmem_ld_wait();
            finish_chunk_cm<EPI>(a, n, n_ok, sw, bias, qseg, qcol, b0 + 16 * c, r, lane);
          }
          tc_fence_before();
          mbar_arrive(&ctl->tmem_empty[acc]);
        } else {
          // add this split's partial sums into the workspace tile
          for (int c = group; c < 2 * nchunks; c += 4) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_row + (uint32_t)(16 * c), r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int m = b0 + 16 * c + i;
              if (n_ok && m < a.M) atomicAdd(a.ws + (int64_t)m * a.N + n, (int)r[i]);
            }
          }
          tc_fence_before();
          mbar_arrive(&ctl->tmem_empty[acc]);  // TMEM is free for the next unit
          __threadfence();
          named_barrier_sync(kEpiBarrier, kEpiThreads);
          if (e == 0 && lane == 0) {
            const int ticket = atomicAdd(a.tickets + t, 1);
            ctl->last_flag = (ticket == a.ksplit - 1);
          }
          named_barrier_sync(kEpiBarrier, kEpiThreads);
          if (ctl->last_flag) {
            __threadfence();
            final_from_ws<EPI>(a, a0, b0, e * 32 + lane);
            if (e == 0 && lane == 0) a.tickets[t] = 0;
          }
          named_barrier_sync(kEpiBarrier, kEpiThreads);  // last_flag is reused by the next unit
        }
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
// Token-major INT8 GEMM on CTA pairs (tcgen05.mma.cta_group::2, M = 256).
//
// A cluster of two CTAs (one TPC) computes 256-token x 256-channel units:
// CTA r loads tokens [m0 + 128 r, +128) and weight rows [n0 + 128 r, +128) of
// every 128-byte K block, and the even CTA's MMA thread multiplies the pair's
// 256 x 128 A and 256 x 128 B halves in one instruction per 32-byte K step.
// Each CTA's TMEM receives its own 128 tokens x 256 channels, finished by the
// same epilogue as the one-CTA kernel. Per SM and K block that is 32 KB of
// operands for 128 x 256 outputs, against 48 KB with one CTA per tile: the
// operand stream from L2, which sets the pace of the one-CTA kernel, shrinks
// by a third.
//
// Barriers: the even CTA's full[s] counts both CTAs' bytes (its producer arms
// it with both halves; the odd CTA's loads complete on it across the pair);
// the MMA commits signal empty[s] and tmem_full[acc] in both CTAs; each
// epilogue warp of either CTA releases tmem_empty[acc] of the even CTA. Every
// wait is bounded; a CTA whose wait ran out stops issuing, lets its copies in
// flight land, and both CTAs meet at a cluster barrier before TMEM is freed.
// ---------------------------------------------------------------------------
constexpr int kPairBN = 256;         // channels per unit (each CTA loads half)
constexpr int kPairMinKBlocks = 36;  // pairs for reductions longer than 36 x 128 bytes

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmR, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int stages = a.stages;
  const uint32_t a_bytes = kBM * kBoxBytes;                // this CTA's 128 token rows
  const uint32_t b_bytes = (kPairBN / 2) * kBoxBytes;      // this CTA's 128 weight rows
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint8_t *epi_stage = smem + (size_t)stages * stage_bytes;
  SmemCtl *ctl = reinterpret_cast<SmemCtl *>(epi_stage + kEpiStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const TmUnits<true> units(a);
  constexpr uint32_t kCols = 2 * kPairBN;  // double-buffered 256-column accumulator

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->tmem_full[i], 1);
      mbar_init(&ctl->tmem_empty[i], 2 * kEpiWarps);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    ctl->consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (EPI == EPI_RESID) prefetch_tmap(&tmR);
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, kCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int *abort_flag = &ctl->abort_flag;

  int issued = 0;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    // Weight boxes of the first unit go out before waiting for the previous
    // kernel (they do not depend on it).
    const uint32_t full0 = dsmem_addr(&ctl->full[0], 0);  // the even CTA's full[0]
    const uint32_t full_stride = (uint32_t)sizeof(uint64_t);
    const uint32_t both = 2 * stage_bytes;
    const int half = (int)rank * (kPairBN / 2);
    int pre = 0;
    if (units.first < units.total) {
      const int b0 = (units.first % a.b_tiles) * kPairBN + half;
      for (; pre < a.kblocks && pre < stages; ++pre) {
        if (leader) mbar_arrive_expect_tx(&ctl->full[pre], both);
        tma_load_2d_pair(smem + (size_t)pre * stage_bytes + a_bytes, &tmB,
                         full0 + (uint32_t)pre * full_stride, pre * kBoxBytes, b0);
      }
    }
    pdl_wait();
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    for (int u = units.first; u < units.total && !*abort_flag; u += units.stride) {
      const int pm = u / a.b_tiles, pn = u - (u / a.b_tiles) * a.b_tiles;
      const int a0 = pm * (2 * kBM) + (int)rank * kBM;
      const int b0 = pn * kPairBN + half;
      if (EPI == EPI_RESID && u + units.stride < units.total) {
        // this CTA's residual rows of its next unit: into L2 now
        const int un = u + units.stride;
        const int pmn = un / a.b_tiles;
        tma_prefetch_l2_2d(&tmR, (un - pmn * a.b_tiles) * kPairBN, pmn * (2 * kBM) + (int)rank * kBM);
      }
      for (int kb = 0; kb < a.kblocks; ++kb) {
        if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort_flag, a.err, 0x1301)) break;
        uint8_t *sa = smem + (size_t)stage * stage_bytes;
        const uint32_t fb = full0 + (uint32_t)stage * full_stride;
        if (it >= pre) {
          if (leader) mbar_arrive_expect_tx(&ctl->full[stage], both);
          tma_load_2d_pair(sa + a_bytes, &tmB, fb, kb * kBoxBytes, b0);
        }
        tma_load_2d_pair(sa, &tmA, fb, kb * kBoxBytes, a0);
        ++it;
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Give every prefetched weight box its token box, so that each stage armed
    // above can still complete.
    if (units.first < units.total) {
      const int a0 = (units.first / a.b_tiles) * (2 * kBM) + (int)rank * kBM;
      for (; it < pre; ++it, ++issued)
        tma_load_2d_pair(smem + (size_t)it * stage_bytes, &tmA, full0 + (uint32_t)it * full_stride,
                         it * kBoxBytes, a0);
    }
    if (*abort_flag) {
      // This CTA's copies complete on the even CTA's barriers: give the ones
      // in flight time to land before the shared memory is released.
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------- MMA issuer (even CTA) ----------------
    pdl_wait();
    const uint32_t idesc = make_idesc(2, 1, 2 * kBM, kPairBN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int consumed = 0;
    bool ok = true;
    for (int u = units.first; u < units.total && ok; u += units.stride) {
      if (!mbar_wait(&ctl->tmem_empty[acc], acc_phase ^ 1, abort_flag, a.err, 0x1302)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kPairBN);
      for (int kb = 0; kb < a.kblocks; ++kb) {
        if (!mbar_wait(&ctl->full[stage], phase, abort_flag, a.err, 0x1303)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)stage * stage_bytes);
        const uint32_t sb = sa + a_bytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 4 x 32-byte K steps inside the 128-byte atom
          tc_mma_i8_pair(d_tmem, make_sw128_desc(sa + 32 * k), make_sw128_desc(sb + 32 * k), idesc,
                         (kb != 0 || k != 0) ? 1u : 0u);
        tc_commit_pair_both(&ctl->empty[stage]);
        ++consumed;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      tc_commit_pair_both(&ctl->tmem_full[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    ctl->consumed = consumed;
    // No MMA may still write either CTA's TMEM or read shared memory when the
    // pair meets at the final cluster barrier.
    tc_commit_pair(&ctl->drain);
    mbar_wait(&ctl->drain, 0, nullptr, a.err, 0x1304);
  } else if (warp >= kEpiWarp0) {
    // ---------------- epilogue (both CTAs) ----------------
    pdl_wait();
    const int e = warp - kEpiWarp0;
    epilogue_tm<EPI, false, true>(a, ctl, tmem_base,
                                  smem_u32(epi_stage) + (uint32_t)(e * kWarpEpiBytes), e, lane,
                                  abort_flag, a.vec_params != 0, nullptr);
  }

  __syncthreads();
  if (leader && warp == 0 && lane == 0 && *abort_flag) {
    // Stages armed by this CTA but never consumed: wait (bounded) for their
    // bytes, which include the odd CTA's.
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < issued; ++i) {
      // (a stage the odd CTA never filled does not complete: stop there)
      if (i >= ctl->consumed && !mbar_wait(&ctl->full[stage], phase, nullptr, a.err, 0x1305))
        break;
      if (++stage == stages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  tc_fence_before();
  cluster_sync_all();  // neither CTA frees TMEM or leaves while the pair still works
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kCols);
  }
}

// ---------------------------------------------------------------------------
// host-side launcher
// ---------------------------------------------------------------------------
static int round_up32(int x) { return (x + 31) & ~31; }

// Token tile of the channel-major orientation (weights as the MMA's M = 128
// operand, the tokens as its N).
static int cm_token_tile(int M) { return M >= 256 ? 256 : round_up32(M < 32 ? 32 : M); }

// K splits of a channel-major int8 GEMM given a workspace: when the output
// tiles alone cannot occupy the GPU, about one (tile, K range) unit per SM.
// Returns 1 (no split, the workspace is not read) otherwise; *kb_per is the
// number of 128-byte K blocks per split.
static int cm_ksplit(int M, int N, int K, int sm_count, int *kb_per) {
  const int kblocks = (K + kBoxBytes - 1) / kBoxBytes;
  const int BN = cm_token_tile(M);
  const int tiles0 = ((N + kBM - 1) / kBM) * ((M + BN - 1) / BN);
  *kb_per = kblocks;
  if (2 * tiles0 > sm_count || kblocks <= 1) return 1;
  int ks = sm_count / tiles0;
  if (ks > kblocks) ks = kblocks;
  const int per = (kblocks + ks - 1) / ks;
  const int splits = (kblocks + per - 1) / per;
  if (splits > 1) *kb_per = per;
  return splits;
}

template <int KIND, int EPI, bool CM, bool RT = false>
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
  CUtensorMap tmA, tmB, tmR, tmRb;
  memset(&tmR, 0, sizeof(tmR));
  memset(&tmRb, 0, sizeof(tmRb));
  if (CM) {  // A = weights, B = tokens
    a.BN = cm_token_tile(M);
    st = make_tmap_2d(&tmA, W, dt, (uint64_t)N, (uint64_t)K, (uint64_t)K * esz, kBoxBytes / esz,
                      kBM);
    if (st) return st;
    st = make_tmap_2d(&tmB, X, dt, (uint64_t)M, (uint64_t)K, (uint64_t)ldx_elems * esz,
                      kBoxBytes / esz, (uint32_t)a.BN);
    if (st) return st;
    a.a_tiles = (N + kBM - 1) / kBM;
    a.b_tiles = (M + a.BN - 1) / a.BN;
  } else {   // A = tokens, B = weights
    a.BN = N >= 256 ? 256 : round_up32(N);
    st = make_tmap_2d(&tmA, X, dt, (uint64_t)M, (uint64_t)K, (uint64_t)ldx_elems * esz,
                      kBoxBytes / esz, kBM);
    if (st) return st;
    st = make_tmap_2d(&tmB, W, dt, (uint64_t)N, (uint64_t)K, (uint64_t)K * esz, kBoxBytes / esz,
                      (uint32_t)a.BN);
    if (st) return st;
    a.a_tiles = (M + kBM - 1) / kBM;
    a.b_tiles = (N + a.BN - 1) / a.BN;
    if (EPI == EPI_RESID) {  // L2 prefetch of the residual, one 128 x BN box per tile
      st = make_tmap_2d(&tmR, la.R, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)M, (uint64_t)N,
                        (uint64_t)la.ldr * 2, (uint32_t)a.BN, kBM, 0);
      if (st) return st;
    }
    if (RT) {  // the epilogue's 32-row x 16-channel residual blocks
      st = make_tmap_2d(&tmRb, la.R, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)M, (uint64_t)N,
                        (uint64_t)la.ldr * 2, 16, 32, 32);
      if (st) return st;
    }
  }
  const int stage_bytes = (kBM + a.BN) * kBoxBytes;
  const int epi_bytes =
      (!CM && EPI != EPI_S32) ? (RT ? kEpiStageBytesRT : kEpiStageBytes) : 0;
  const int budget = 227 * 1024 - 1024 - epi_bytes - (int)sizeof(SmemCtl) - 64;
  a.stages = budget / stage_bytes;
  if (a.stages > 8) a.stages = 8;
  if (a.stages < 2) return W8A8_ERR_UNSUPPORTED;
  const size_t smem = 1024 + (size_t)a.stages * stage_bytes + epi_bytes + sizeof(SmemCtl);
  // 16-byte vector loads of channel scales and biases (16-channel runs)
  a.vec_params = aligned16(la.sW) && (la.bias == nullptr || aligned16(la.bias));
  a.kblocks = (K * esz + kBoxBytes - 1) / kBoxBytes;
  a.err = ctx->err;
  a.ksplit = 1;
  a.kb_per = a.kblocks;
  a.ws = nullptr;
  a.tickets = nullptr;
  const int tiles0 = a.a_tiles * a.b_tiles;
  if (CM && KIND == 0 && la.workspace &&
      la.workspace_bytes >= linear_workspace_bytes(M, N)) {
    // Too few output tiles to occupy the GPU (decode): split K so that about
    // one unit lands on every SM.
    a.ksplit = cm_ksplit(M, N, K, ctx->sm_count, &a.kb_per);
    if (a.ksplit > 1) {
      uint8_t *w = (uint8_t *)la.workspace;
      a.ws = (int32_t *)w;
      a.tickets = (int *)(w + (((size_t)M * N * 4 + 255) & ~(size_t)255));
    }
  }
  static bool attr_set[64] = {};  // per template instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<KIND, EPI, CM, RT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return W8A8_ERR_CUDA;
    attr_set[dev] = true;
  }
  const int units = tiles0 * a.ksplit;
  const int grid = units < ctx->sm_count ? units : ctx->sm_count;
  launch_pdl(gemm_tc_kernel<KIND, EPI, CM, RT>, dim3(grid), dim3(kThreads), smem, stream, tmA, tmB,
             tmR, tmRb,
             a);
  return check_launch("gemm_tc");
}

// Token-major INT8 GEMM on CTA pairs: a persistent grid of as many 2-CTA
// clusters as can be resident at once (at most one per TPC), each striding
// over the 256 x 256 units.
template <int EPI>
static int launch_pair(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &la,
                       cudaStream_t stream) {
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  GemmArgs a;
  static_cast<LinearArgs &>(a) = la;
  const int M = la.M, N = la.N, K = la.K;
  CUtensorMap tmA, tmB, tmR;
  memset(&tmR, 0, sizeof(tmR));
  a.BN = kPairBN;
  st = make_tmap_2d(&tmA, X, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)M, (uint64_t)K,
                    (uint64_t)ldx, kBoxBytes, kBM);
  if (st) return st;
  st = make_tmap_2d(&tmB, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)N, (uint64_t)K, (uint64_t)K,
                    kBoxBytes, kPairBN / 2);
  if (st) return st;
  a.a_tiles = (M + kBM - 1) / kBM;
  a.b_tiles = (N + kPairBN - 1) / kPairBN;
  if (EPI == EPI_RESID) {  // L2 prefetch of the residual, one 128 x 256 box per CTA and unit
    st = make_tmap_2d(&tmR, la.R, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)M, (uint64_t)N,
                      (uint64_t)la.ldr * 2, (uint32_t)kPairBN, kBM, 0);
    if (st) return st;
  }
  const int stage_bytes = (kBM + kPairBN / 2) * kBoxBytes;
  const int epi_bytes = kEpiStageBytes;
  const int budget = 227 * 1024 - 1024 - epi_bytes - (int)sizeof(SmemCtl) - 64;
  a.stages = budget / stage_bytes;
  if (a.stages > 8) a.stages = 8;
  if (a.stages < 2) return W8A8_ERR_UNSUPPORTED;
  const size_t smem = 1024 + (size_t)a.stages * stage_bytes + epi_bytes + sizeof(SmemCtl);
  a.vec_params = aligned16(la.sW) && (la.bias == nullptr || aligned16(la.bias));
  a.kblocks = (K + kBoxBytes - 1) / kBoxBytes;
  a.err = ctx->err;
  a.ksplit = 1;
  a.kb_per = a.kblocks;
  a.ws = nullptr;
  a.tickets = nullptr;

  static int max_clusters[64] = {};  // per template instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  if (max_clusters[dev] == 0) {
    if (cudaFuncSetAttribute(gemm_tc_pair_kernel<EPI>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      return W8A8_ERR_CUDA;
    cfg.gridDim = dim3(2 * (ctx->sm_count / 2));
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_pair_kernel<EPI>, &cfg) != cudaSuccess ||
        n < 1) {
      cudaGetLastError();
      return W8A8_ERR_UNSUPPORTED;
    }
    max_clusters[dev] = n;
  }
  const int units = ((a.a_tiles + 1) / 2) * a.b_tiles;
  const int clusters = units < max_clusters[dev] ? units : max_clusters[dev];
  cfg.gridDim = dim3(2 * clusters);
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, gemm_tc_pair_kernel<EPI>, tmA, tmB, tmR, a) !=
      cudaSuccess) {
    cudaGetLastError();
    return W8A8_ERR_CUDA;
  }
  return check_launch("gemm_tc_pair");
}

size_t linear_workspace_bytes(int M, int N) {
  const size_t tiles = (size_t)((N + kBM - 1) / kBM) * (size_t)((M + 31) / 32);
  return (((size_t)M * N * 4 + 255) & ~(size_t)255) + tiles * 4;
}

// Token-major needs whole 32-column chunks and 16-byte aligned output rows.
static bool token_major_ok(const LinearArgs &a) {
  if (a.M <= kBM || (a.N & 31)) return false;
  const int esz = a.epi == EPI_S32 ? 4 : 2;
  if (!aligned16(a.Y) || (a.ldy * esz) % 16) return false;
  if (a.epi == EPI_RESID && (!aligned16(a.R) || (a.ldr % 8))) return false;
  if (a.epi == EPI_QKV &&
      (!aligned16(a.Kc) || !aligned16(a.Vc) || (a.dseg & 31) || (a.seq_stride % 8)))
    return false;
  return true;
}

// Decode-sized GEMMs whose 128-channel tiles cannot occupy the GPU take the
// cluster split-K kernel when its operand rules hold.
static bool takes_cluster(const LinearArgs &a, const void *X, int64_t ldx, int sm_count) {
  const int tiles = (a.N + kBM - 1) / kBM;
  return 2 * tiles <= sm_count && cluster_gemm_ok(a, X, ldx);
}

template <int EPI>
static int launch_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
                     cudaStream_t s) {
  if (token_major_ok(a)) {
    // Residual GEMMs with short K (attn_proj): residual blocks by TMA into
    // per-warp slots; the slots leave room for fewer pipeline stages, enough
    // where the residual loads, not the operand loads, set the pace.
    const int kblocks = (a.K + kBoxBytes - 1) / kBoxBytes;
    if constexpr (EPI != EPI_S32) {
      // The longest reductions on CTA pairs, where the main loop sets the
      // pace: W2 of GPT-2 large (K 5120) at 32768 tokens 178 -> 162 us,
      // tensor pipe 65 -> 74% busy. Shorter ones gain nothing or lose, each
      // unit's time being set by the epilogue (~18 us per 128 x 256 residual
      // tile) or the operand round trip: W2 K 4096 122 -> 123 us, K 3072
      // 89 -> 97; K 1280: W_qkv 147 -> 149, attn_proj 75 -> 78, W1 + GELU
      // 267 -> 270.
      if (a.N >= kPairBN && kblocks > kPairMinKBlocks) {
        const int st = launch_pair<EPI>(W, X, ldx, a, s);
        if (st != W8A8_ERR_UNSUPPORTED) return st;
      }
    }
    if (EPI == EPI_RESID && kblocks <= 16)
      return launch_tc<0, EPI, false, EPI == EPI_RESID>(W, X, ldx, a, s);
    return launch_tc<0, EPI, false>(W, X, ldx, a, s);
  }
  // Decode: too few 128-channel tiles to occupy the GPU; split K over a
  // cluster and reduce in distributed shared memory.
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  if (takes_cluster(a, X, ldx, ctx->sm_count)) return gemm_cluster_i8(W, X, ldx, a, s);
  return launch_tc<0, EPI, true>(W, X, ldx, a, s);
}

size_t gemm_i8_workspace_used(const int8_t *X, int64_t ldx, const LinearArgs &a) {
  if (token_major_ok(a)) return 0;
  int st, kb_per;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx || takes_cluster(a, X, ldx, ctx->sm_count)) return 0;
  if (cm_ksplit(a.M, a.N, a.K, ctx->sm_count, &kb_per) <= 1) return 0;
  return linear_workspace_bytes(a.M, a.N);
}

int gemm_tc_i8(const int8_t *W, const int8_t *X, int64_t ldx, const LinearArgs &a,
               cudaStream_t stream) {
  switch (a.epi) {
    case EPI_S32: return launch_i8<EPI_S32>(W, X, ldx, a, stream);
    case EPI_DEQUANT: return launch_i8<EPI_DEQUANT>(W, X, ldx, a, stream);
    case EPI_BIAS: return launch_i8<EPI_BIAS>(W, X, ldx, a, stream);
    case EPI_RESID: return launch_i8<EPI_RESID>(W, X, ldx, a, stream);
    case EPI_GELU: return launch_i8<EPI_GELU>(W, X, ldx, a, stream);
    case EPI_QKV: return launch_i8<EPI_QKV>(W, X, ldx, a, stream);
    default: return W8A8_ERR_INVALID;
  }
}

int gemm_tc_bf16(const uint16_t *W, const uint16_t *X, int64_t ldx, const LinearArgs &a,
                 cudaStream_t stream) {
  if (a.epi != EPI_F32_BF16) return W8A8_ERR_INVALID;
  return launch_tc<1, EPI_F32_BF16, true>(W, X, ldx, a, stream);
}

}  // namespace w8a8
