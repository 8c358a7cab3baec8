// Causal multi-head attention over the bf16 KV cache (head_dim 64).
//
// Reference dataflow per head (gpt2.c:1182-1219 with cuda/softmax.cu:24-92):
//   S   = bf16(alpha * q.k)            cuBLAS bf16 GEMM, fp32 accumulate,
//                                       alpha = 1/sqrt(64) = 0.125 (exact)
//   m   = max_j S_j                     (j <= query position)
//   e_j = expf(S_j - m)                 written as bf16; summed unrounded
//   sum = 256-slot tree of e_j          (thread t of 256 adds j = t, t+256, ..)
//   P_j = bf16(float(bf16(e_j)) * (1/sum))
//   O   = bf16(sum_j P_j V_j)           cuBLAS bf16 GEMM, fp32 accumulate
// These kernels keep every rounding point, and the softmax sum uses the same
// 256-slot tree, so P is bit-identical to the reference for identical S.
// The S and O dot products accumulate in a fixed order of ours (the
// reference's order is cuBLAS's), so S and O agree within rounding.
//
// Prefill: one CTA per (sequence, head, 64-query tile). Scores for the whole
// causal row block live in shared memory as bf16 (<= 128 KB at 1024 keys),
// so softmax needs no online rescaling and P is formed exactly as above.
// Q.K^T and P.V run on mma.sync bf16 tensor-core fragments.
//
// Decode: per (sequence, head), keys split over CTAs when the batch alone
// cannot fill the GPU. Kernel 1 writes bf16 scores to the workspace; kernel 2
// forms P from the full score row (every split recomputes the row's max and
// tree sum, so no split needs another's result) and accumulates its share of
// P.V; the last split to finish (ticket counter, no waiting) adds the partials
// in split order and rounds.
#include "common.cuh"
#include "kernels.cuh"
#include "runtime.cuh"

namespace w8a8 {

constexpr int kHD = 64;  // head_dim of every GPT-2 size (model_config.h: d_model / nof_heads)

// ---------------------------------------------------------------------------
// warp-level helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                          uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool pred) {
  const int sz = pred ? 16 : 0;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Reference softmax sum: 256 partials folded pairwise (s = 128 .. 1). Lane l
// holds slots l + 32*i, i < 8.
__device__ __forceinline__ float tree256(float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] += v[i + 4];
#pragma unroll
  for (int i = 0; i < 2; ++i) v[i] += v[i + 2];
  float x = v[0] + v[1];
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) x += __shfl_down_sync(0xffffffffu, x, s);
  return __shfl_sync(0xffffffffu, x, 0);
}

// In-place softmax of one causal row held as bf16 in shared memory:
// entries [0, n) hold S; on return they hold P, entries [n, n_pad) hold 0.
__device__ __forceinline__ void softmax_row_inplace(uint16_t *row, int n, int n_pad, int lane) {
  float mx = -INFINITY;
  for (int j = lane; j < n; j += 32) mx = fmaxf(mx, bf2f(row[j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float local_sum = 0.0f;
    for (int j = lane + 32 * i; j < n; j += 256) {
      float e = expf(bf2f(row[j]) - mx);
      row[j] = f2bf(e);
      local_sum += e;
    }
    v[i] = local_sum;
  }
  const float sum_exp = tree256(v);
  const float inv_sum = 1.0f / sum_exp;
  __syncwarp();
  for (int j = lane; j < n_pad; j += 32)
    row[j] = j < n ? f2bf(bf2f(row[j]) * inv_sum) : (uint16_t)0;
  __syncwarp();
}

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
constexpr int kQT = 32;          // query rows per CTA
constexpr int kKT = 64;          // keys per K/V tile
constexpr int kTileStride = 72;  // bf16 elements per smem tile row (64 + 8 pad)

struct PrefillArgs {
  const uint16_t *Q;
  int64_t ldq;
  const uint16_t *Kc, *Vc;
  int64_t seq_stride;
  int n_seq, T, n_head, d;
  uint16_t *O;
  int64_t ldo;
  int s_stride;  // bf16 elements per score row in smem
};

// 8 warps per CTA: warp w owns query rows 16*(w%2) .. +15 and, in Q.K^T, keys
// [16*(w/2), +16) of each 64-key tile, in P.V head dims [16*(w/2), +16).
// Every output element is accumulated by one thread in key order. 32-query
// tiles keep the bf16 score rows of a 1024-token causal block in 66 KB of
// shared memory, so two CTAs (16 warps) share an SM at 1024 tokens and four
// at 512.
constexpr int kPrefillThreads = 256;

__global__ void __launch_bounds__(kPrefillThreads)
    attention_prefill_kernel(PrefillArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) uint16_t sm[];
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kQT;
  if (q0 >= a.T) return;
  const int nk = min(q0 + kQT, a.T);  // keys visible to this query tile
  const int n_ktiles = (nk + kKT - 1) / kKT;
  const int nk_pad = n_ktiles * kKT;

  uint16_t *sQ = sm;                            // [32][72]
  uint16_t *sKV = sQ + kQT * kTileStride;       // [2][64][72]
  uint16_t *sS = sKV + 2 * kKT * kTileStride;   // [32][s_stride]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int mt = warp & 1, quarter = warp >> 1;

  const uint16_t *Kb = a.Kc + (int64_t)b * a.seq_stride + h * kHD;
  const uint16_t *Vb = a.Vc + (int64_t)b * a.seq_stride + h * kHD;
  const uint16_t *Qb = a.Q + ((int64_t)b * a.T) * a.ldq + h * kHD;

  // tile loader: rows x 128 bytes in 16 B chunks (64-row K/V tiles: 2 per
  // thread; the 32-row Q tile: 1)
  auto load_tile = [&](uint16_t *dst, const uint16_t *src, int64_t ld, int row0, int nrows,
                       int rows) {
    for (int i = 0; i < rows * 8 / kPrefillThreads; ++i) {
      int c = tid + kPrefillThreads * i;
      int r = c >> 3, cc = (c & 7) * 8;
      bool ok = row0 + r < nrows;
      const uint16_t *g = src + (int64_t)(ok ? row0 + r : 0) * ld + cc;
      cp_async16(dst + r * kTileStride + cc, g, ok);
    }
  };

  load_tile(sQ, Qb, a.ldq, q0, a.T, kQT);
  load_tile(sKV, Kb, a.d, 0, nk, kKT);
  cp_async_commit();

  // Q fragments (rows 16*mt .. +15), 4 k-steps of 16
  uint32_t qa[4][4];
  const int g = lane >> 2, tq = lane & 3;

  // ---- phase A: S = bf16(0.125 * Q K^T) into sS ----
  for (int kt = 0; kt < n_ktiles; ++kt) {
    cp_async_wait_all();
    __syncthreads();
    if (kt + 1 < n_ktiles) {
      load_tile(sKV + ((kt + 1) & 1) * kKT * kTileStride, Kb, a.d, (kt + 1) * kKT, nk, kKT);
      cp_async_commit();
    }
    if (kt == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint16_t *p = sQ + (mt * 16 + (lane & 15)) * kTileStride + ks * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32(p), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    const uint16_t *sK = sKV + (kt & 1) * kKT * kTileStride;
    float c[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) c[nb][i] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {  // the pair of 8-key blocks of this warp's 16 keys
      const int nb2 = quarter;
      const int q = lane >> 3;
      const uint16_t *p =
          sK + (nb2 * 16 + (q >> 1) * 8 + (lane & 7)) * kTileStride + ks * 16 + (q & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(smem_u32(p), b0, b1, b2, b3);
      mma_bf16_16816(c[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      mma_bf16_16816(c[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
    }
    // scale, round, store (columns beyond a row's causal limit are never read)
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      const int col = kt * kKT + quarter * 16 + nb * 8 + 2 * tq;
      const int r0 = mt * 16 + g;
      uint32_t lo = (uint32_t)f2bf(c[nb][0] * 0.125f) | ((uint32_t)f2bf(c[nb][1] * 0.125f) << 16);
      uint32_t hi = (uint32_t)f2bf(c[nb][2] * 0.125f) | ((uint32_t)f2bf(c[nb][3] * 0.125f) << 16);
      *reinterpret_cast<uint32_t *>(sS + r0 * a.s_stride + col) = lo;
      *reinterpret_cast<uint32_t *>(sS + (r0 + 8) * a.s_stride + col) = hi;
    }
  }
  __syncthreads();

  // prefetch V tile 0 while the softmax runs
  load_tile(sKV, Vb, a.d, 0, nk, kKT);
  cp_async_commit();

  // ---- phase B: causal softmax per row (warp w: rows w, w+8, ...) ----
  for (int r = warp; r < kQT; r += kPrefillThreads / 32) {
    const int qpos = q0 + r;
    const int n = qpos < a.T ? qpos + 1 : 0;
    softmax_row_inplace(sS + r * a.s_stride, n, nk_pad, lane);
  }

  // ---- phase C: O = P V (this warp: 16 rows x 16 head dims) ----
  float o[2][4];
#pragma unroll
  for (int nb = 0; nb < 2; ++nb)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[nb][i] = 0.f;
  for (int kt = 0; kt < n_ktiles; ++kt) {
    cp_async_wait_all();
    __syncthreads();
    if (kt + 1 < n_ktiles) {
      load_tile(sKV + ((kt + 1) & 1) * kKT * kTileStride, Vb, a.d, (kt + 1) * kKT, nk, kKT);
      cp_async_commit();
    }
    const uint16_t *sV = sKV + (kt & 1) * kKT * kTileStride;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {  // 16 keys per step
      uint32_t pa0, pa1, pa2, pa3;
      const uint16_t *pp =
          sS + (mt * 16 + (lane & 15)) * a.s_stride + kt * kKT + ks * 16 + (lane >> 4) * 8;
      ldsm_x4(smem_u32(pp), pa0, pa1, pa2, pa3);
      {  // the pair of 8-dim blocks of this warp's 16 dims
        const int nb2 = quarter;
        const int q = lane >> 3;
        const uint16_t *p =
            sV + (ks * 16 + (q & 1) * 8 + (lane & 7)) * kTileStride + nb2 * 16 + (q >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(p), b0, b1, b2, b3);
        mma_bf16_16816(o[0], pa0, pa1, pa2, pa3, b0, b1);
        mma_bf16_16816(o[1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
  }
  // ---- store O ----
  const int r0 = mt * 16 + g;
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
    const int col = h * kHD + quarter * 16 + nb * 8 + 2 * tq;
    if (q0 + r0 < a.T) {
      uint32_t v = (uint32_t)f2bf(o[nb][0]) | ((uint32_t)f2bf(o[nb][1]) << 16);
      *reinterpret_cast<uint32_t *>(a.O + ((int64_t)b * a.T + q0 + r0) * a.ldo + col) = v;
    }
    if (q0 + r0 + 8 < a.T) {
      uint32_t v = (uint32_t)f2bf(o[nb][2]) | ((uint32_t)f2bf(o[nb][3]) << 16);
      *reinterpret_cast<uint32_t *>(a.O + ((int64_t)b * a.T + q0 + r0 + 8) * a.ldo + col) = v;
    }
  }
}

int launch_attention_prefill(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                             const uint16_t *Vc, int64_t seq_stride, int n_seq, int T, int n_head,
                             uint16_t *O, int64_t ldo, cudaStream_t s) {
  if (attention_prefill_tc_ok(Q, ldq, Kc, Vc, seq_stride, T, n_head))
    return launch_attention_prefill_tc(Q, ldq, Kc, Vc, seq_stride, n_seq, T, n_head, O, ldo, s);
  PrefillArgs a;
  a.Q = Q;
  a.ldq = ldq;
  a.Kc = Kc;
  a.Vc = Vc;
  a.seq_stride = seq_stride;
  a.n_seq = n_seq;
  a.T = T;
  a.n_head = n_head;
  a.d = n_head * kHD;
  a.O = O;
  a.ldo = ldo;
  const int max_pad = ((T + kKT - 1) / kKT) * kKT;
  a.s_stride = max_pad + 8;
  size_t smem = (size_t)(kQT * kTileStride + 2 * kKT * kTileStride + kQT * a.s_stride) * 2;
  if (smem > 227 * 1024) return W8A8_ERR_UNSUPPORTED;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaFuncSetAttribute(attention_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         227 * 1024);
    attr[dev & 63] = true;
  }
  dim3 grid((T + kQT - 1) / kQT, n_head, n_seq);
  launch_pdl(attention_prefill_kernel, dim3(grid), dim3(kPrefillThreads), smem, s, a);
  return check_launch("attention_prefill");
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
struct DecodeArgs {
  const uint16_t *Q;
  int64_t ldq;
  const uint16_t *Kc, *Vc;
  int64_t seq_stride;
  int n_seq, n_head, d, max_ctx, splits, keys_per_split;
  const int32_t *n_ctx;  // per-sequence key counts, or NULL: every sequence uses max_ctx
  uint16_t *O;
  int64_t ldo;
  uint16_t *scores;   // [n_seq][n_head][max_ctx]
  float *partials;    // [n_seq][n_head][splits][64]
  int *tickets;       // [n_seq][n_head]
  // optional fused per-token quantization of each sequence's whole output
  // row (all heads): the last (b, h) of sequence b to finish quantizes O[b]
  int8_t *Xq;         // [n_seq][d], NULL: no quantization
  float *sXq;         // [n_seq]
  int *seq_tickets;   // [n_seq], zero between calls
};

// q row of (b, h) in registers: lane part p holds dims 8p .. 8p+7.
__device__ __forceinline__ void load_q8(const DecodeArgs &a, int b, int h, int part, float (&q)[8]) {
  const uint4 qv = *reinterpret_cast<const uint4 *>(a.Q + (int64_t)b * a.ldq + h * kHD + part * 8);
  const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    q[2 * i] = __uint_as_float(w[i] << 16);
    q[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// S_j = bf16(0.125 * q.k_j) for keys [j0, j1), written through `emit(j, s)`.
// 8 lanes cover one 128-byte key row (16 bytes each), a warp 4 keys per
// step; each lane keeps 4 row loads in flight.
template <int U = 4, typename Emit>
__device__ __forceinline__ void score_keys(const DecodeArgs &a, int b, int h, int j0, int j1,
                                           int warp, int nwarps, int lane, Emit emit) {
  const int sub = lane >> 3, part = lane & 7;
  float q[8];
  load_q8(a, b, h, part, q);
  const uint16_t *Kb = a.Kc + (int64_t)b * a.seq_stride + h * kHD + part * 8;
  const int step = nwarps * 4;
  // U row loads in flight per lane (any U: each score is computed alone)
  
  for (int jb = j0 + warp * 4; jb < j1; jb += step * U) {
    uint4 kv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + u * step + sub;
      kv[u] = j < j1 ? __ldg(reinterpret_cast<const uint4 *>(Kb + (int64_t)j * a.d))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + u * step + sub;
      const uint32_t w[4] = {kv[u].x, kv[u].y, kv[u].z, kv[u].w};
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s = fmaf(q[2 * i], __uint_as_float(w[i] << 16), s);
        s = fmaf(q[2 * i + 1], __uint_as_float(w[i] & 0xffff0000u), s);
      }
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      if (part == 0 && j < j1) emit(j, f2bf(s * 0.125f));
    }
  }
}

// Softmax statistics of a full score row (n entries, bf16) with the
// reference's 256-slot tree: slot t adds e_j for j = t, t + 256, ... in
// order, then the slots fold pairwise (s = 128 .. 1). With NT = 128 threads,
// thread t owns slots t and t + 128 (the first fold is its own addition);
// with more than 256, threads 0..255 own the slots and the rest only help
// with the maximum. s_tree holds 256 floats. Returns (max, 1/sum).
template <int NT, typename Load>
__device__ __forceinline__ void row_stats(int n, int tid, Load ld, float *s_red, float *s_tree,
                                          float &mx_out, float &inv_out) {
  static_assert(NT == 128 || NT == 256 || NT == 512, "row_stats: 128, 256 or 512 threads");
  const int warp = tid >> 5, lane = tid & 31;
  float mx = -INFINITY;
  for (int j = tid; j < n; j += NT) mx = fmaxf(mx, bf2f(ld(j)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) mx = fmaxf(mx, s_red[w]);
  float local_sum = 0.0f;
  if (tid < 256)
    for (int j = tid; j < n; j += 256) local_sum += expf(bf2f(ld(j)) - mx);
  if (NT == 128) {
    float hi_sum = 0.0f;
    for (int j = tid + 128; j < n; j += 256) hi_sum += expf(bf2f(ld(j)) - mx);
    local_sum += hi_sum;  // fold s = 128: slot t += slot t + 128
  }
  if (tid < (NT == 128 ? 128 : 256)) s_tree[tid] = local_sum;
  __syncthreads();
  for (int s = (NT == 128 ? 64 : 128); s > 0; s >>= 1) {
    if (tid < s) s_tree[tid] += s_tree[tid + s];
    __syncthreads();
  }
  mx_out = mx;
  inv_out = 1.0f / s_tree[0];
}

// Partial O = sum_{j in [j0, j1)} P_j V_j over NT threads: 8 lanes per
// 128-byte V row (8 dims each), 4 rows per warp step, 4 steps in flight.
// Returns this thread's share for dim `tid` (< 64) after the block reduction.
template <int NT, int U = 4>
__device__ __forceinline__ float pv_range(const DecodeArgs &a, int b, int h, int j0, int j1,
                                          const float *p, float (*s_part)[kHD], int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int sub = lane >> 3, part = lane & 7;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  const uint16_t *Vb = a.Vc + (int64_t)b * a.seq_stride + h * kHD + part * 8;
  // U rows in flight per lane: each lane still adds its rows (j = j0 + warp*4 + sub
  // + NT/8 * k, k = 0, 1, ...) in increasing order, so U does not change the result
  
  constexpr int kRows = NT / 8;  // V rows per step over the block
  for (int jb = j0 + warp * 4 + sub; jb < j1; jb += kRows * U) {
    uint4 vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + kRows * u;
      vv[u] = j < j1 ? __ldg(reinterpret_cast<const uint4 *>(Vb + (int64_t)j * a.d))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + kRows * u;
      const float pj = j < j1 ? p[j - j0] : 0.f;
      const uint32_t w[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(pj, __uint_as_float(w[i] << 16), acc[2 * i]);
        acc[2 * i + 1] = fmaf(pj, __uint_as_float(w[i] & 0xffff0000u), acc[2 * i + 1]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
  }
  if (sub == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) s_part[warp][part * 8 + i] = acc[i];
  }
  __syncthreads();
  float o = 0.f;
  if (tid < kHD) {
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) o += s_part[w][tid];
  }
  return o;
}

// Per-token quantization (activation_quant.cu:75-91) of sequence b's whole
// output row O[b, 0:d) once its last head is written: the CTA that finishes
// the last (b, h) of the sequence (ticket counter, no waiting) reads the row
// back from L2 and writes Xq[b], sXq[b]. Identical to w8a8_quant_rows.
template <int NT>
__device__ __forceinline__ void quant_row_when_complete(const DecodeArgs &a, int b, int tid,
                                                        float *s_red, int *s_flag) {
  __threadfence();
  __syncthreads();
  if (tid == 0) *s_flag = (atomicAdd(&a.seq_tickets[b], 1) == a.n_head - 1);
  __syncthreads();
  if (!*s_flag) return;
  __threadfence();
  const uint16_t *row = a.O + (int64_t)b * a.ldo;
  const int nv = a.d >> 3;
  float m = 0.0f;
  for (int v = tid; v < nv; v += NT) {
    const uint4 x = __ldcg(reinterpret_cast<const uint4 *>(row) + v);
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      m = fmaxf(m, fabsf(__uint_as_float(w[i] << 16)));
      m = fmaxf(m, fabsf(__uint_as_float(w[i] & 0xffff0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) s_red[tid >> 5] = m;
  __syncthreads();
  m = s_red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) m = fmaxf(m, s_red[w]);
  const float scale = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, scale);
  if (tid == 0) {
    a.sXq[b] = scale;
    a.seq_tickets[b] = 0;  // ready for the next call
  }
  for (int v = tid; v < nv; v += NT) {
    const uint4 x = __ldcg(reinterpret_cast<const uint4 *>(row) + v);
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
    uint32_t q8[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = (e & 1) ? __uint_as_float(w[e >> 1] & 0xffff0000u)
                              : __uint_as_float(w[e >> 1] << 16);
      int q = __float2int_rn(__fmul_rn(f, inv));
      q = q > 127 ? 127 : (q < -127 ? -127 : q);
      q8[e >> 2] |= ((uint32_t)(q & 0xff)) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2 *>(a.Xq + (int64_t)b * a.d + 8 * v) = make_uint2(q8[0], q8[1]);
  }
}

// Split path, kernel 1: this split's scores into the workspace row.
__global__ void __launch_bounds__(256) attention_decode_scores_kernel(DecodeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / a.n_head, h = bh - (bh / a.n_head) * a.n_head;
  const int n = a.n_ctx ? a.n_ctx[b] : a.max_ctx;
  const int j0 = split * a.keys_per_split;
  const int j1 = min(n, j0 + a.keys_per_split);
  if (j0 >= j1) return;
  uint16_t *srow = a.scores + ((int64_t)b * a.n_head + h) * a.max_ctx;
  score_keys(a, b, h, j0, j1, threadIdx.x >> 5, 8, threadIdx.x & 31,
             [&](int j, uint16_t s) { srow[j] = s; });
}

// Split path, kernel 2: softmax statistics from the full score row (each
// split recomputes them), P for this split's keys, its share of P.V; the
// last split of (b, h) to finish adds the partials in split order.
__global__ void __launch_bounds__(256) attention_decode_pv_kernel(DecodeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float s_red[8];
  __shared__ float s_tree[256];
  __shared__ float s_part[8][kHD];
  __shared__ float s_p[1024];
  __shared__ int s_last;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / a.n_head, h = bh - (bh / a.n_head) * a.n_head;
  const int n = a.n_ctx ? a.n_ctx[b] : a.max_ctx;
  const int j0 = split * a.keys_per_split;
  const int j1 = min(n, j0 + a.keys_per_split);
  const int tid = threadIdx.x;
  const uint16_t *srow = a.scores + ((int64_t)b * a.n_head + h) * a.max_ctx;
  float mx, inv_sum;
  row_stats<256>(n, tid, [&](int j) { return srow[j]; }, s_red, s_tree, mx, inv_sum);
  for (int j = j0 + tid; j < j1; j += 256)
    s_p[j - j0] = bf2f(f2bf(bf2f(f2bf(expf(bf2f(srow[j]) - mx))) * inv_sum));
  __syncthreads();
  const float o = pv_range<256>(a, b, h, j0, j1, s_p, s_part, tid);
  if (a.splits == 1) {
    if (tid < kHD) a.O[(int64_t)b * a.ldo + h * kHD + tid] = f2bf(o);
    if (a.Xq) quant_row_when_complete<256>(a, b, tid, s_red, &s_last);
    return;
  }
  float *part_out = a.partials + (((int64_t)b * a.n_head + h) * a.splits + split) * kHD;
  if (tid < kHD) part_out[tid] = o;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int ticket = atomicAdd(&a.tickets[b * a.n_head + h], 1);
    s_last = (ticket == a.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < kHD) {
    const float *pp = a.partials + ((int64_t)b * a.n_head + h) * a.splits * kHD;
    float tot = 0.f;
    for (int sidx = 0; sidx < a.splits; ++sidx) tot += __ldcg(pp + sidx * kHD + tid);
    a.O[(int64_t)b * a.ldo + h * kHD + tid] = f2bf(tot);
  }
  if (tid == 0) a.tickets[b * a.n_head + h] = 0;  // ready for the next call
  if (a.Xq) quant_row_when_complete<256>(a, b, tid, s_red, &s_last);
}

// Split path as one launch: the `splits` CTAs of a (b, h) pair form a thread-
// block cluster; CTA r owns keys [r*kps, (r+1)*kps) of the pair's n keys (kps
// = ceil(n / splits)) and everything the two-kernel form exchanges through the
// workspace moves through distributed shared memory instead:
//   scores of its keys (own shared memory) -> its maximum -> the row maximum
//   (every CTA reads all CTAs' maxima) -> e_j = expf(S_j - max) of its keys ->
//   the reference's 256-slot sums (slot t adds e_j, j = t, t + 256, ... in
//   order, read from the CTA holding each j; CTA r sums slots
//   r*256/splits ..) stored in CTA 0 -> every CTA folds the 256 slots with the
//   same tree -> P of its keys -> its P.V partial -> CTA 0 adds the partials
//   in rank order, rounds, stores (and quantizes the sequence's row when it
//   is the last of its heads).
// The same operations as the two kernels above (which split by max_ctx), in
// one launch with no global round trip between the phases.
__global__ void __launch_bounds__(256) attention_decode_cluster_kernel(DecodeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ uint16_t s_s[1024];  // scores of this CTA's keys
  __shared__ float s_e[1024];     // their exponentials, then their P
  __shared__ float s_red[8];
  __shared__ float s_tree[256];
  __shared__ float s_slots[256];  // CTA 0: the 256 slot sums
  __shared__ float s_part[8][kHD];
  __shared__ float s_o[kHD];      // this CTA's P.V partial
  __shared__ float s_cmax;
  __shared__ int s_flag;
  const uint32_t r = cluster_ctarank();
  const int S = a.splits;
  const int bh = blockIdx.x / S;
  const int b = bh / a.n_head, h = bh - (bh / a.n_head) * a.n_head;
  const int n = a.n_ctx ? a.n_ctx[b] : a.max_ctx;
  // the pair's own keys split evenly (at most keys_per_split <= 1024 each)
  const int kps = max(1, (n + S - 1) / S);
  const int j0 = (int)r * kps, j1 = min(n, j0 + kps);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // scores of this CTA's keys
  score_keys(a, b, h, j0, j1, warp, 8, lane, [&](int j, uint16_t sv) { s_s[j - j0] = sv; });
  __syncthreads();
  // row maximum
  float mx = -INFINITY;
  for (int j = j0 + tid; j < j1; j += 256) mx = fmaxf(mx, bf2f(s_s[j - j0]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = s_red[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, s_red[w]);
    s_cmax = m;
  }
  cluster_sync_all();
  if (tid == 0) {
    float m = ld_dsmem_f32(dsmem_addr(&s_cmax, 0));
    for (int q = 1; q < S; ++q) m = fmaxf(m, ld_dsmem_f32(dsmem_addr(&s_cmax, (uint32_t)q)));
    s_red[0] = m;
  }
  __syncthreads();
  mx = s_red[0];
  for (int j = j0 + tid; j < j1; j += 256) s_e[j - j0] = expf(bf2f(s_s[j - j0]) - mx);
  cluster_sync_all();
  // slot sums, in order, over the cluster
  const int per = 256 / S;  // slots per CTA (S <= 8: per >= 32)
  if (tid < per) {
    const int t = (int)r * per + tid;
    float acc = 0.0f;
    int q = 0, off = t;  // e_j lives in CTA q at offset off
    while (off >= kps) {
      off -= kps;
      ++q;
    }
    for (int j = t; j < n; j += 256) {
      acc += ld_dsmem_f32(dsmem_addr(&s_e[off], (uint32_t)q));
      off += 256;
      while (off >= kps) {
        off -= kps;
        ++q;
      }
    }
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dsmem_addr(&s_slots[t], 0)), "f"(acc)
                 : "memory");
  }
  cluster_sync_all();
  s_tree[tid] = ld_dsmem_f32(dsmem_addr(&s_slots[tid], 0));
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) s_tree[tid] += s_tree[tid + s];
    __syncthreads();
  }
  const float inv_sum = 1.0f / s_tree[0];
  for (int j = j0 + tid; j < j1; j += 256)
    s_e[j - j0] = bf2f(f2bf(bf2f(f2bf(s_e[j - j0])) * inv_sum));
  __syncthreads();
  const float o = pv_range<256>(a, b, h, j0, j1, s_e, s_part, tid);
  if (tid < kHD) s_o[tid] = o;
  cluster_sync_all();
  if (r == 0) {
    if (tid < kHD) {
      float tot = 0.f;
      for (int q = 0; q < S; ++q) tot += ld_dsmem_f32(dsmem_addr(&s_o[tid], (uint32_t)q));
      a.O[(int64_t)b * a.ldo + h * kHD + tid] = f2bf(tot);
    }
    if (a.Xq) quant_row_when_complete<256>(a, b, tid, s_red, &s_flag);
  }
  cluster_sync_all();  // no CTA leaves while CTA 0 still reads its partial
}

// Whole-row path: one CTA per (b, h) keeps the scores in shared memory, so K
// and V are each read once and the call is one launch. With enough pairs to
// fill the GPU the CTAs are small (128 threads, 48 registers, ~8 KB of shared
// memory): ten share an SM and a 64-sequence batch of GPT-2 large (1280
// pairs) runs as a single wave. With fewer pairs than SMs (small batches)
// each CTA has 512 threads, so one pair's keys are covered in a few steps.
template <int NT, int U>
__global__ void __launch_bounds__(NT) attention_decode_fused_kernel(DecodeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float s_red[NT / 32];
  __shared__ float s_tree[NT == 128 ? 128 : 256];
  __shared__ float s_part[NT / 32][kHD];
  __shared__ float s_p[1024];
  __shared__ uint16_t s_s[1024];
  __shared__ int s_flag;
  const int bh = blockIdx.x;
  const int b = bh / a.n_head, h = bh - (bh / a.n_head) * a.n_head;
  const int n = a.n_ctx ? a.n_ctx[b] : a.max_ctx;
  const int tid = threadIdx.x;
  score_keys<U>(a, b, h, 0, n, tid >> 5, NT / 32, tid & 31, [&](int j, uint16_t s) { s_s[j] = s; });
  __syncthreads();
  float mx, inv_sum;
  row_stats<NT>(n, tid, [&](int j) { return s_s[j]; }, s_red, s_tree, mx, inv_sum);
  for (int j = tid; j < n; j += NT)
    s_p[j] = bf2f(f2bf(bf2f(f2bf(expf(bf2f(s_s[j]) - mx))) * inv_sum));
  __syncthreads();
  const float o = pv_range<NT, U>(a, b, h, 0, n, s_p, s_part, tid);
  if (tid < kHD) a.O[(int64_t)b * a.ldo + h * kHD + tid] = f2bf(o);
  if (a.Xq) quant_row_when_complete<NT>(a, b, tid, s_red, &s_flag);
}

// One CTA per (sequence, head) unless the pairs cover fewer than a quarter of
// the SMs; then split the keys so that about two CTAs land on every SM, with
// at least 128 keys per split. Measured on decode steps (prompt 512): GPT-2
// large with 1 sequence (20 pairs) 1196 us split / 1362 us whole-row, with 4
// sequences 1755 us split / 1577 us whole-row (512-thread CTAs); GPT-2 medium
// with 1 sequence 789 / 869 us; 8 sequences of GPT-2 large (160 pairs) 15%
// faster whole-row than in 2 splits.
static int decode_splits(int n_seq, int n_head, int max_ctx, int sm_count) {
  const int pairs = n_seq * n_head;
  if (4 * pairs >= sm_count) return 1;
  int splits = 1;
  while (pairs * splits < 2 * sm_count && splits * 2 * 128 <= max_ctx) splits *= 2;
  return splits;
}

// The ticket counters (per (sequence, head) for the split path, per sequence
// for the fused output quantization) live in the last kTicketBytes of the
// caller's workspace: a fixed place for a given buffer whatever the shape of
// the call. Every call leaves them zero (the last CTA resets its counter), so
// a workspace zero-filled once needs no clearing between calls — in a CUDA
// graph, no memset node per layer.
constexpr int kMaxPairTickets = 16384;
constexpr int kMaxSeqTickets = 4096;
constexpr size_t kTicketBytes = (size_t)(kMaxPairTickets + kMaxSeqTickets) * sizeof(int);

int decode_workspace_reset(void *ws, size_t ws_bytes, cudaStream_t s) {
  if (!ws || ws_bytes < kTicketBytes + 16) return W8A8_ERR_INVALID;
  void *t = reinterpret_cast<void *>((((uintptr_t)ws + ws_bytes - kTicketBytes) & ~(uintptr_t)15));
  return cudaMemsetAsync(t, 0, kTicketBytes, s) == cudaSuccess ? W8A8_OK : W8A8_ERR_CUDA;
}

int decode_launches(int n_seq, int n_head, int max_ctx, int sm_count) {
  const int splits = decode_splits(n_seq, n_head, max_ctx, sm_count);
  if (splits == 1) return 1;
  const int kps = (max_ctx + splits - 1) / splits;
  return (kps <= 1024 && kps >= 128 && splits <= 8) ? 1 : 2;  // cluster form: one launch
}

size_t decode_workspace_bytes(int n_seq, int n_head, int max_ctx, int splits) {
  size_t scores = (size_t)n_seq * n_head * max_ctx * 2;
  scores = (scores + 255) & ~(size_t)255;
  size_t parts = (size_t)n_seq * n_head * splits * kHD * 4;
  return scores + parts + 512 + kTicketBytes;  // 512: base alignment slack
}

int launch_attention_decode(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                            const uint16_t *Vc, int64_t seq_stride, int n_seq,
                            const int32_t *n_ctx, int max_ctx, int n_head, uint16_t *O,
                            int64_t ldo, int8_t *Xq, float *sXq, void *ws, size_t ws_bytes,
                            int sm_count, cudaStream_t s) {
  DecodeArgs a;
  a.Q = Q;
  a.ldq = ldq;
  a.Kc = Kc;
  a.Vc = Vc;
  a.seq_stride = seq_stride;
  a.n_seq = n_seq;
  a.n_head = n_head;
  a.d = n_head * kHD;
  a.max_ctx = max_ctx;
  a.n_ctx = n_ctx;
  a.O = O;
  a.ldo = ldo;
  a.splits = decode_splits(n_seq, n_head, max_ctx, sm_count);
  a.keys_per_split = (max_ctx + a.splits - 1) / a.splits;
  if (decode_workspace_bytes(n_seq, n_head, max_ctx, a.splits) > ws_bytes)
    return W8A8_ERR_INVALID;
  uint8_t *w = (uint8_t *)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  a.scores = (uint16_t *)w;
  size_t scores = ((size_t)n_seq * n_head * max_ctx * 2 + 255) & ~(size_t)255;
  a.partials = (float *)(w + scores);
  if (n_seq * n_head > kMaxPairTickets || n_seq > kMaxSeqTickets) return W8A8_ERR_UNSUPPORTED;
  a.tickets = reinterpret_cast<int *>((((uintptr_t)ws + ws_bytes - kTicketBytes) & ~(uintptr_t)15));
  a.seq_tickets = a.tickets + kMaxPairTickets;
  a.Xq = Xq;
  a.sXq = sXq;
  if (a.splits == 1) {
    const int pairs = n_seq * n_head;
    if (pairs >= 8 * sm_count)
      launch_pdl(attention_decode_fused_kernel<128, 4>, dim3(pairs), dim3(128), 0, s, a);
    else if (pairs >= 4 * sm_count)
      launch_pdl(attention_decode_fused_kernel<256, 4>, dim3(pairs), dim3(256), 0, s, a);
    else
      launch_pdl(attention_decode_fused_kernel<512, 4>, dim3(pairs), dim3(512), 0, s, a);
    return check_launch("attention_decode_fused");
  }
  if (a.keys_per_split <= 1024 && a.keys_per_split >= 128 && a.splits <= 8) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_seq * n_head * a.splits);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)a.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, attention_decode_cluster_kernel, a) != cudaSuccess) {
      cudaGetLastError();
      return W8A8_ERR_CUDA;
    }
    return check_launch("attention_decode_cluster");
  }
  dim3 grid(n_seq * n_head, a.splits);
  launch_pdl(attention_decode_scores_kernel, dim3(grid), dim3(256), 0, s, a);
  int st = check_launch("attention_decode_scores");
  if (st) return st;
  launch_pdl(attention_decode_pv_kernel, dim3(grid), dim3(256), 0, s, a);
  return check_launch("attention_decode_pv");
}

}  // namespace w8a8
