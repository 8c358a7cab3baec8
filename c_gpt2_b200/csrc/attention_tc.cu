// Causal prefill attention on the 5th-generation tensor cores: tcgen05.mma
// kind::f16 (bf16 operands, fp32 accumulators in TMEM), operands staged by
// TMA, and the reference's exact two-pass softmax (gpt2.c:1205-1217 with
// cuda/softmax.cu:24-92):
//   S_j = bf16(0.125 * q.k_j)               (alpha = 1/sqrt(64), exact)
//   m   = max_{j <= i} S_j
//   e_j = expf(S_j - m), summed unrounded in 256 slots (slot t adds
//         j = t, t+256, ... in order), the slots folded pairwise (h = 128..1)
//   P_j = bf16(float(bf16(e_j)) * (1 / sum)),  P_j = 0 for j > i
//   O   = bf16(sum_j P_j V_j)                (fp32 accumulate)
// so P is bit-identical to the reference's for identical S; the S and O dot
// products sum in the tensor core's order (the reference's is cuBLAS's).
//
// One CTA per (128-query tile, head, sequence), heaviest tiles first. The
// CTA's key tiles (128 keys x 64 dims, <= 8 of them: prompts up to 1024
// tokens) stay in shared memory; V tiles stream through two slots.
//   warp 16  TMA: Q tile, every K tile, V tiles
//   warp 17  TMEM owner and MMA issuer: S = Q K^T into one of two 128-column
//            TMEM buffers, three times per key tile (pass 1: row maxima;
//            pass 2: slot sums; pass 3: P), and O += P V into 64 columns
//   warps 0-15  softmax: TMEM lane (query row) = 32 * (warp % 4) + lane,
//            columns [32 * (warp / 4), +32) of every key tile. Pass 2 visits
//            even tiles, then odd tiles: slot t (t < 128) only sums even
//            tiles' column t, slot t + 128 odd tiles' column t, so each slot
//            keeps the reference's order and each thread holds 32 slot sums
//            at a time. Recomputing S costs tensor-core time the kernel has
//            to spare; storing it would not fit on chip at 1024 keys.
// The softmax warps first scale the Q tile by 0.125 in shared memory (exact:
// a power of two), so S = bf16(acc) needs no multiply; scores stay packed as
// bf16x2 until an exponential needs them, and only the diagonal key tile
// (kt == query tile) pays for the causal mask (a warp whose 32 keys are all
// masked there skips them). This three-pass kernel serves prompts of 513 to
// 1024 tokens; up to 512 tokens attention_prefill_tc_e_kernel (below) keeps
// the exponentials on chip instead of recomputing S a third time.
// Every wait is bounded and records an error instead of hanging.
#include "common.cuh"
#include "runtime.cuh"

#include <math.h>

namespace w8a8 {

namespace {

constexpr int kAQ = 128;      // query rows per CTA (TMEM lanes)
constexpr int kAK = 128;      // keys per tile
constexpr int kAMaxKT = 8;    // key tiles of a 1024-token prompt
constexpr int kSoftWarps = 16;
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kTmaWarp = 16, kMmaWarp = 17;
constexpr int kAThreads = 18 * 32;
constexpr uint32_t kATile = 128 * 128;   // [128 rows][64 bf16], 128-byte swizzle
constexpr uint32_t kAP = 2 * kATile;     // P: [128 rows][128 keys] as two 64-key atoms
constexpr int kSoftBar = 1;
constexpr uint32_t kTmemS = 0;           // two 128-column score buffers
constexpr uint32_t kTmemO = 256;         // 64 columns
constexpr uint32_t kTmemSlots = 320;     // 4 x 32 columns: slot sums of the even tiles
constexpr uint32_t kTmemCols = 512;

struct AttnCtl {
  uint64_t q_full, q_ready;
  uint64_t k_full[kAMaxKT];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  float row_max[4][kAQ];
  float row_inv[kAQ];
};

struct AttnTcArgs {
  int T, n_qt;
  int p_bufs;     // 1 or 2 P buffers
  uint16_t *O;
  int64_t ldo;
  int vec_store;  // O rows 16-byte aligned
  int *err;
};

// One key tile's 32 scores of this thread as bf16 pairs: S = bf16(acc) (the
// 0.125 is in Q already).
__device__ __forceinline__ void scores_bf2(const uint32_t (&v)[32], uint32_t (&p)[16]) {
#pragma unroll
  for (int c = 0; c < 16; ++c)
    p[c] = pack_bf2(__uint_as_float(v[2 * c]), __uint_as_float(v[2 * c + 1]));
}
__device__ __forceinline__ float lo_f(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float hi_f(uint32_t p) { return __uint_as_float(p & 0xffff0000u); }
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

}  // namespace

__global__ void __launch_bounds__(kAThreads, 1)
    attention_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                const __grid_constant__ CUtensorMap tmK,
                                const __grid_constant__ CUtensorMap tmV, AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int qt = a.n_qt - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kAQ;
  const int nk = min(q0 + kAQ, a.T);
  const int n_kt = (nk + kAK - 1) / kAK;
  uint8_t *sQ = smem;
  uint8_t *sK = sQ + kATile;
  uint8_t *sV = sK + (size_t)a.n_qt * kATile;
  uint8_t *sP = sV + 2 * kATile;
  AttnCtl *ctl = reinterpret_cast<AttnCtl *>(sP + (size_t)a.p_bufs * kAP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->q_full, 1);
    mbar_init(&ctl->q_ready, 1);
    for (int i = 0; i < kAMaxKT; ++i) mbar_init(&ctl->k_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->v_full[i], 1);
      mbar_init(&ctl->v_empty[i], 1);
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], kSoftWarps);
      mbar_init(&ctl->p_full[i], kSoftWarps);
      mbar_init(&ctl->p_empty[i], 1);
    }
    mbar_init(&ctl->o_full, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int *abort_flag = &ctl->abort_flag;
  // Q, K and V are the previous kernel's output.
  pdl_wait();

  if (warp == kTmaWarp) {
    // ---------------- TMA ----------------
    if (lane == 0) {
      int k_issued = 0, v_issued = 0;
      mbar_arrive_expect_tx(&ctl->q_full, kATile);
      tma_load_3d(sQ, &tmQ, &ctl->q_full, h * 64, q0, b);
      for (int kt = 0; kt < n_kt; ++kt, ++k_issued) {
        mbar_arrive_expect_tx(&ctl->k_full[kt], kATile);
        tma_load_3d(sK + (size_t)kt * kATile, &tmK, &ctl->k_full[kt], h * 64, kt * kAK, b);
      }
      for (int kt = 0; kt < n_kt; ++kt) {
        const int vb = kt & 1;
        if (!mbar_wait(&ctl->v_empty[vb], ((kt >> 1) & 1) ^ 1, abort_flag, a.err, 0x1401)) break;
        mbar_arrive_expect_tx(&ctl->v_full[vb], kATile);
        tma_load_3d(sV + (size_t)vb * kATile, &tmV, &ctl->v_full[vb], h * 64, kt * kAK, b);
        ++v_issued;
      }
      if (*abort_flag) {
        // no bulk copy may still be writing shared memory when the CTA exits
        mbar_wait(&ctl->q_full, 0, nullptr, a.err, 0x1402);
        for (int kt = 0; kt < k_issued; ++kt) mbar_wait(&ctl->k_full[kt], 0, nullptr, a.err, 0x1402);
        for (int i = (v_issued > 2 ? v_issued - 2 : 0); i < v_issued; ++i)
          mbar_wait(&ctl->v_full[i & 1], (i >> 1) & 1, nullptr, a.err, 0x1402);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idS = make_idesc(1, 1, kAQ, kAK);
      const uint32_t idO = make_idesc_bmn(1, 1, kAQ, 64);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV),
                     p_addr = smem_u32(sP);
      bool ok = mbar_wait(&ctl->q_ready, 0, abort_flag, a.err, 0x1403);
      tc_fence_after();
      int sidx = 0;
      uint32_t k_seen = 0;
      auto issue_s = [&](int kt) -> bool {
        const int buf = sidx & 1;
        if (!mbar_wait(&ctl->s_empty[buf], ((sidx >> 1) & 1) ^ 1, abort_flag, a.err, 0x1404))
          return false;
        if (!(k_seen & (1u << kt))) {
          if (!mbar_wait(&ctl->k_full[kt], 0, abort_flag, a.err, 0x1405)) return false;
          k_seen |= 1u << kt;
        }
        tc_fence_after();
        const uint32_t d = tmem + kTmemS + (uint32_t)(buf * kAK);
        const uint32_t kb = k_addr + (uint32_t)kt * kATile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_bf16(d, make_sw128_desc(q_addr + 32 * k), make_sw128_desc(kb + 32 * k), idS,
                      k > 0);
        tc_commit(&ctl->s_full[buf]);
        ++sidx;
        return true;
      };
      // pass 1 (maxima) in tile order, pass 2 (slot sums) even tiles then odd
      for (int kt = 0; kt < n_kt && ok; ++kt) ok = issue_s(kt);
      for (int par = 0; par < 2 && ok; ++par)
        for (int kt = par; kt < n_kt && ok; kt += 2) ok = issue_s(kt);
      // pass 3: S of the next tile is issued before P V of this one
      if (ok) ok = issue_s(0);
      for (int kt = 0; kt < n_kt && ok; ++kt) {
        if (kt + 1 < n_kt && !(ok = issue_s(kt + 1))) break;
        const int vb = kt & 1;
        const int pb = a.p_bufs == 2 ? (kt & 1) : 0;
        const uint32_t pph = (uint32_t)((a.p_bufs == 2 ? kt >> 1 : kt) & 1);
        if (!(ok = mbar_wait(&ctl->p_full[pb], pph, abort_flag, a.err, 0x1406))) break;
        if (!(ok = mbar_wait(&ctl->v_full[vb], (kt >> 1) & 1, abort_flag, a.err, 0x1407))) break;
        tc_fence_after();
        const uint32_t vbase = v_addr + (uint32_t)vb * kATile;
        const uint32_t pbase = p_addr + (uint32_t)pb * kAP;
#pragma unroll
        for (int ks = 0; ks < kAK / 16; ++ks)
          tc_mma_bf16(tmem + kTmemO,
                      make_sw128_desc(pbase + (uint32_t)(ks >> 2) * kATile + 32 * (ks & 3)),
                      make_sw128_mn_desc(vbase + (uint32_t)ks * 2048), idO, (kt > 0) || (ks > 0));
        tc_commit(&ctl->p_empty[pb]);
        tc_commit(&ctl->v_empty[vb]);
      }
      if (ok) {
        tc_commit(&ctl->o_full);
      } else {
        // no MMA may still be writing TMEM when it is released
        tc_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, a.err, 0x1408);
      }
    }
  } else {
    // ---------------- softmax warps ----------------
    const int qd = warp & 3, cq = warp >> 2;
    const int r = qd * 32 + lane;      // query row of the tile = TMEM lane
    const int qpos = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    const int col0 = cq * 32;          // this thread's columns of each key tile
    // Q *= 0.125 in place (exact for bf16: a power of two), then the MMA may start
    {
      mbar_wait(&ctl->q_full, 0, abort_flag, a.err, 0x140C);
      uint4 *q4 = reinterpret_cast<uint4 *>(sQ) + threadIdx.x * 2;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint4 v = q4[i];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = pack_bf2(lo_f(w[j]) * 0.125f, hi_f(w[j]) * 0.125f);
        q4[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      named_barrier_sync(kSoftBar, kSoftThreads);
      if (threadIdx.x == 0) mbar_arrive(&ctl->q_ready);
    }
    int sidx = 0;
    // Wait for the next score tile, copy this thread's 32 columns, release it.
    auto next_scores = [&](uint32_t (&p)[16]) {
      const int buf = sidx & 1;
      mbar_wait(&ctl->s_full[buf], (sidx >> 1) & 1, abort_flag, a.err, 0x1409);
      tc_fence_after();
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + kTmemS + (uint32_t)(buf * kAK + col0), v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->s_empty[buf]);
      ++sidx;
      scores_bf2(v, p);
    };

    // ---- pass 1: row maximum ----
    uint32_t mx2 = 0xff80ff80u;  // (-inf, -inf)
    float m = -INFINITY;
    // On the diagonal key tile (kt == qt) this warp's 32 keys lie past all
    // of its rows' positions when cq > qd, before all of them when cq < qd.
    for (int kt = 0; kt < n_kt; ++kt) {
      uint32_t p[16];
      next_scores(p);
      if (kt < qt || cq < qd) {  // every key visible
#pragma unroll
        for (int c = 0; c < 16; ++c) mx2 = bf2_max(mx2, p[c]);
      } else if (cq == qd) {
        const int lim = qpos - (kt * kAK + col0);  // columns c <= lim are causal
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float x = (c & 1) ? hi_f(p[c >> 1]) : lo_f(p[c >> 1]);
          if (c <= lim) m = fmaxf(m, x);
        }
      }
    }
    m = fmaxf(m, fmaxf(lo_f(mx2), hi_f(mx2)));
    ctl->row_max[cq][r] = m;
    named_barrier_sync(kSoftBar, kSoftThreads);
    m = fmaxf(fmaxf(ctl->row_max[0][r], ctl->row_max[1][r]),
              fmaxf(ctl->row_max[2][r], ctl->row_max[3][r]));

    // ---- pass 2: slot sums (even tiles, then odd tiles) ----
    float sl[32];
    for (int par = 0; par < 2; ++par) {
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = 0.0f;
      for (int kt = par; kt < n_kt; kt += 2) {
        uint32_t p[16];
        next_scores(p);
        if (kt < qt || cq < qd) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            sl[2 * c] = sl[2 * c] + expf(lo_f(p[c]) - m);
            sl[2 * c + 1] = sl[2 * c + 1] + expf(hi_f(p[c]) - m);
          }
        } else if (cq == qd) {
          const int lim = qpos - (kt * kAK + col0);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float x = (c & 1) ? hi_f(p[c >> 1]) : lo_f(p[c >> 1]);
            if (c <= lim) sl[c] = sl[c] + expf(x - m);
          }
        }
      }
      if (par == 0) {  // park the even slots in TMEM
        uint32_t u[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) u[c] = __float_as_uint(sl[c]);
        tmem_st_32x32b_x32(trow + kTmemSlots + (uint32_t)col0, u);
        tmem_st_wait();
      }
    }
    // fold h = 128: slot t (even tiles) + slot t + 128 (odd tiles), thread-local
    {
      uint32_t u[32];
      tmem_ld_32x32b_x32(trow + kTmemSlots + (uint32_t)col0, u);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = __uint_as_float(u[c]) + sl[c];
    }
    // h = 64 and h = 32 across the four threads of a row, through shared
    // memory (the first P buffer, unused until pass 3)
    float *xs = reinterpret_cast<float *>(sP);  // [2][32][128]
    if (cq >= 2) {
#pragma unroll
      for (int c = 0; c < 32; ++c) xs[((cq - 2) * 32 + c) * kAQ + r] = sl[c];
    }
    named_barrier_sync(kSoftBar, kSoftThreads);
    if (cq < 2) {
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = sl[c] + xs[(cq * 32 + c) * kAQ + r];
    }
    named_barrier_sync(kSoftBar, kSoftThreads);
    if (cq == 1) {
#pragma unroll
      for (int c = 0; c < 32; ++c) xs[c * kAQ + r] = sl[c];
    }
    named_barrier_sync(kSoftBar, kSoftThreads);
    if (cq == 0) {
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = sl[c] + xs[c * kAQ + r];
#pragma unroll
      for (int hh = 16; hh > 0; hh >>= 1)
#pragma unroll
        for (int c = 0; c < hh; ++c) sl[c] = sl[c] + sl[c + hh];
      ctl->row_inv[r] = 1.0f / sl[0];
    }
    named_barrier_sync(kSoftBar, kSoftThreads);
    const float inv = ctl->row_inv[r];

    // ---- pass 3: P into shared memory (128-byte swizzle), one tile at a time ----
    for (int kt = 0; kt < n_kt; ++kt) {
      uint32_t p[16];
      next_scores(p);
      uint32_t pk[16];
      if (kt < qt || cq < qd) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint32_t e2 = pack_bf2(expf(lo_f(p[c]) - m), expf(hi_f(p[c]) - m));
          pk[c] = pack_bf2(lo_f(e2) * inv, hi_f(e2) * inv);
        }
      } else if (cq > qd) {  // every key masked: P = 0
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = 0u;
      } else {
        const int lim = qpos - (kt * kAK + col0);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float p0 = 0.0f, p1 = 0.0f;
          if (2 * c <= lim) p0 = round_bf(expf(lo_f(p[c]) - m)) * inv;
          if (2 * c + 1 <= lim) p1 = round_bf(expf(hi_f(p[c]) - m)) * inv;
          pk[c] = pack_bf2(p0, p1);
        }
      }
      const int pb = a.p_bufs == 2 ? (kt & 1) : 0;
      const int use = a.p_bufs == 2 ? kt >> 1 : kt;  // earlier fills of this buffer
      if (use > 0) mbar_wait(&ctl->p_empty[pb], (uint32_t)((use - 1) & 1), abort_flag, a.err, 0x140A);
      uint8_t *prow = sP + (size_t)pb * kAP + (size_t)(cq >> 1) * kATile + (size_t)r * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int unit = ((cq & 1) * 4 + i) ^ (r & 7);
        *reinterpret_cast<uint4 *>(prow + unit * 16) =
            make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->p_full[pb]);
    }

    // ---- O: this thread's 16 head dims of its row ----
    const bool ok = mbar_wait(&ctl->o_full, 0, abort_flag, a.err, 0x140B);
    tc_fence_after();
    uint32_t o[16];
    tmem_ld_32x32b_x16(trow + kTmemO + (uint32_t)(16 * cq), o);
    tmem_ld_wait();
    if (ok && !*abort_flag && qpos < a.T) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = pack_bf2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
      uint16_t *dst = a.O + ((int64_t)b * a.T + qpos) * a.ldo + h * 64 + 16 * cq;
      if (a.vec_store) {
        reinterpret_cast<uint4 *>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4 *>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<uint32_t *>(dst)[i] = w[i];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Prompts up to 512 tokens (at most four key tiles): the exponentials fit on
// chip. Pass 2 writes bf16(e_j) for every key tile into shared memory, laid
// out as the P operand, so pass 3 is P_j = bf16(float(bf16(e_j)) * inv) in
// place: no third S = Q K^T and no second expf. The K tiles are dead after
// pass 2, and the V tiles are loaded into their space.
//   shared memory: Q 16 KB | K tiles, then V tiles, 16 KB each | E / P tiles,
//   32 KB each (128 rows x 128 keys bf16 as two 64-key 128-byte-swizzle atoms)
//   TMEM: S buffers 0-255, O 256-319, slot sums 320-447, exchange 448-511
// Every rounding point and sum order is the three-pass kernel's.
// ---------------------------------------------------------------------------
namespace {

constexpr int kEMaxKT = 4;
constexpr uint32_t kTmemX = 448;  // cross-thread exchange columns (64)

struct AttnCtlE {
  uint64_t q_full, q_ready;
  uint64_t k_full[kEMaxKT], v_full[kEMaxKT], p_full[kEMaxKT];
  uint64_t s_full[2], s_empty[2];
  uint64_t k_dead, o_full, drain;
  uint32_t tmem_base;
  int abort_flag;
};

// this thread's 16-byte units of row r in a P-layout tile: keys [32*cq, +32)
__device__ __forceinline__ uint4 *p_unit(uint8_t *tile, int r, int cq, int i) {
  const int unit = ((cq & 1) * 4 + i) ^ (r & 7);
  return reinterpret_cast<uint4 *>(tile + (size_t)(cq >> 1) * kATile + (size_t)r * 128 +
                                   unit * 16);
}

// Exchange through TMEM columns of this thread's lane: other warps of the
// same lane quadrant read what a warp wrote after a named barrier.
__device__ __forceinline__ void xchg_barrier() {
  tc_fence_before();
  named_barrier_sync(kSoftBar, kSoftThreads);
  tc_fence_after();
}

}  // namespace

__global__ void __launch_bounds__(kAThreads, 1)
    attention_prefill_tc_e_kernel(const __grid_constant__ CUtensorMap tmQ,
                                  const __grid_constant__ CUtensorMap tmK,
                                  const __grid_constant__ CUtensorMap tmV, AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int qt = a.n_qt - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kAQ;
  const int nk = min(q0 + kAQ, a.T);
  const int n_kt = (nk + kAK - 1) / kAK;
  uint8_t *sQ = smem;
  uint8_t *sKV = sQ + kATile;                          // [n_qt] K tiles, then V tiles
  uint8_t *sE = sKV + (size_t)a.n_qt * kATile;         // [n_qt] E / P tiles
  AttnCtlE *ctl = reinterpret_cast<AttnCtlE *>(sE + (size_t)a.n_qt * kAP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->q_full, 1);
    mbar_init(&ctl->q_ready, 1);
    for (int i = 0; i < kEMaxKT; ++i) {
      mbar_init(&ctl->k_full[i], 1);
      mbar_init(&ctl->v_full[i], 1);
      mbar_init(&ctl->p_full[i], kSoftWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], kSoftWarps);
    }
    mbar_init(&ctl->k_dead, 1);
    mbar_init(&ctl->o_full, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int *abort_flag = &ctl->abort_flag;
  pdl_wait();  // Q, K and V are the previous kernel's output

  if (warp == kTmaWarp) {
    // ---------------- TMA ----------------
    if (lane == 0) {
      int v_issued = 0;
      mbar_arrive_expect_tx(&ctl->q_full, kATile);
      tma_load_3d(sQ, &tmQ, &ctl->q_full, h * 64, q0, b);
      for (int kt = 0; kt < n_kt; ++kt) {
        mbar_arrive_expect_tx(&ctl->k_full[kt], kATile);
        tma_load_3d(sKV + (size_t)kt * kATile, &tmK, &ctl->k_full[kt], h * 64, kt * kAK, b);
      }
      // the V tiles, once no MMA reads the K tiles any more
      if (mbar_wait(&ctl->k_dead, 0, abort_flag, a.err, 0x1421)) {
        for (int kt = 0; kt < n_kt; ++kt, ++v_issued) {
          mbar_arrive_expect_tx(&ctl->v_full[kt], kATile);
          tma_load_3d(sKV + (size_t)kt * kATile, &tmV, &ctl->v_full[kt], h * 64, kt * kAK, b);
        }
      }
      if (*abort_flag) {
        // no bulk copy may still be writing shared memory when the CTA exits
        mbar_wait(&ctl->q_full, 0, nullptr, a.err, 0x1422);
        for (int kt = 0; kt < n_kt; ++kt) mbar_wait(&ctl->k_full[kt], 0, nullptr, a.err, 0x1422);
        for (int kt = 0; kt < v_issued; ++kt) mbar_wait(&ctl->v_full[kt], 0, nullptr, a.err, 0x1422);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idS = make_idesc(1, 1, kAQ, kAK);
      const uint32_t idO = make_idesc_bmn(1, 1, kAQ, 64);
      const uint32_t q_addr = smem_u32(sQ), kv_addr = smem_u32(sKV), e_addr = smem_u32(sE);
      bool ok = mbar_wait(&ctl->q_ready, 0, abort_flag, a.err, 0x1423);
      tc_fence_after();
      int sidx = 0;
      uint32_t k_seen = 0;
      auto issue_s = [&](int kt) -> bool {
        const int buf = sidx & 1;
        if (!mbar_wait(&ctl->s_empty[buf], ((sidx >> 1) & 1) ^ 1, abort_flag, a.err, 0x1424))
          return false;
        if (!(k_seen & (1u << kt))) {
          if (!mbar_wait(&ctl->k_full[kt], 0, abort_flag, a.err, 0x1425)) return false;
          k_seen |= 1u << kt;
        }
        tc_fence_after();
        const uint32_t d = tmem + kTmemS + (uint32_t)(buf * kAK);
        const uint32_t kb = kv_addr + (uint32_t)kt * kATile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_bf16(d, make_sw128_desc(q_addr + 32 * k), make_sw128_desc(kb + 32 * k), idS,
                      k > 0);
        tc_commit(&ctl->s_full[buf]);
        ++sidx;
        return true;
      };
      for (int kt = 0; kt < n_kt && ok; ++kt) ok = issue_s(kt);
      for (int par = 0; par < 2 && ok; ++par)
        for (int kt = par; kt < n_kt && ok; kt += 2) ok = issue_s(kt);
      tc_commit(&ctl->k_dead);  // completes once every S MMA has read its K tile
      for (int kt = 0; kt < n_kt && ok; ++kt) {
        if (!(ok = mbar_wait(&ctl->p_full[kt], 0, abort_flag, a.err, 0x1426))) break;
        if (!(ok = mbar_wait(&ctl->v_full[kt], 0, abort_flag, a.err, 0x1427))) break;
        tc_fence_after();
        const uint32_t vbase = kv_addr + (uint32_t)kt * kATile;
        const uint32_t pbase = e_addr + (uint32_t)kt * kAP;
#pragma unroll
        for (int ks = 0; ks < kAK / 16; ++ks)
          tc_mma_bf16(tmem + kTmemO,
                      make_sw128_desc(pbase + (uint32_t)(ks >> 2) * kATile + 32 * (ks & 3)),
                      make_sw128_mn_desc(vbase + (uint32_t)ks * 2048), idO, (kt > 0) || (ks > 0));
      }
      if (ok) {
        tc_commit(&ctl->o_full);
      } else {
        tc_commit(&ctl->drain);
        mbar_wait(&ctl->drain, 0, nullptr, a.err, 0x1428);
      }
    }
  } else {
    // ---------------- softmax warps ----------------
    const int qd = warp & 3, cq = warp >> 2;
    const int r = qd * 32 + lane;
    const int qpos = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    const int col0 = cq * 32;
    {  // Q *= 0.125 in place (exact), then the MMA may start
      mbar_wait(&ctl->q_full, 0, abort_flag, a.err, 0x1429);
      uint4 *q4 = reinterpret_cast<uint4 *>(sQ) + threadIdx.x * 2;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint4 v = q4[i];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = pack_bf2(lo_f(w[j]) * 0.125f, hi_f(w[j]) * 0.125f);
        q4[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      named_barrier_sync(kSoftBar, kSoftThreads);
      if (threadIdx.x == 0) mbar_arrive(&ctl->q_ready);
    }
    int sidx = 0;
    auto next_scores = [&](uint32_t (&pp)[16]) {
      const int buf = sidx & 1;
      mbar_wait(&ctl->s_full[buf], (sidx >> 1) & 1, abort_flag, a.err, 0x142A);
      tc_fence_after();
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + kTmemS + (uint32_t)(buf * kAK + col0), v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->s_empty[buf]);
      ++sidx;
      scores_bf2(v, pp);
    };

    // ---- pass 1: row maximum ----
    uint32_t mx2 = 0xff80ff80u;
    float m = -INFINITY;
    // On the diagonal key tile (kt == qt) this warp's 32 keys lie past all
    // of its rows' positions when cq > qd, before all of them when cq < qd.
    for (int kt = 0; kt < n_kt; ++kt) {
      uint32_t pp[16];
      next_scores(pp);
      if (kt < qt || cq < qd) {
#pragma unroll
        for (int c = 0; c < 16; ++c) mx2 = bf2_max(mx2, pp[c]);
      } else if (cq == qd) {
        const int lim = qpos - (kt * kAK + col0);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float x = (c & 1) ? hi_f(pp[c >> 1]) : lo_f(pp[c >> 1]);
          if (c <= lim) m = fmaxf(m, x);
        }
      }
    }
    m = fmaxf(m, fmaxf(lo_f(mx2), hi_f(mx2)));
    tmem_st_32x32b_x1(trow + kTmemX + (uint32_t)cq, __float_as_uint(m));
    tmem_st_wait();
    xchg_barrier();
    {
      uint32_t mm[4];
      tmem_ld_32x32b_x4(trow + kTmemX, mm);
      tmem_ld_wait();
      m = fmaxf(fmaxf(__uint_as_float(mm[0]), __uint_as_float(mm[1])),
                fmaxf(__uint_as_float(mm[2]), __uint_as_float(mm[3])));
    }
    xchg_barrier();  // every lane has read the maxima before the columns are reused

    // ---- pass 2: slot sums and bf16(e) into the E tiles ----
    float sl[32];
    for (int par = 0; par < 2; ++par) {
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = 0.0f;
      for (int kt = par; kt < n_kt; kt += 2) {
        uint32_t pp[16];
        next_scores(pp);
        uint8_t *tile = sE + (size_t)kt * kAP;
        if (kt == qt && cq > qd) {  // every key masked: e = 0
#pragma unroll
          for (int i = 0; i < 4; ++i) *p_unit(tile, r, cq, i) = make_uint4(0u, 0u, 0u, 0u);
          continue;
        }
        // keys past the row's own position (diagonal tile only) give e = 0
        const int lim = (kt < qt || cq < qd) ? 31 : qpos - (kt * kAK + col0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // one 16-byte unit (8 keys) at a time
          uint32_t e2[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = 4 * i + j;
            float e0 = 0.0f, e1 = 0.0f;
            if (2 * c <= lim) {
              e0 = expf(lo_f(pp[c]) - m);
              sl[2 * c] = sl[2 * c] + e0;
            }
            if (2 * c + 1 <= lim) {
              e1 = expf(hi_f(pp[c]) - m);
              sl[2 * c + 1] = sl[2 * c + 1] + e1;
            }
            e2[j] = pack_bf2(e0, e1);
          }
          *p_unit(tile, r, cq, i) = make_uint4(e2[0], e2[1], e2[2], e2[3]);
        }
      }
      if (par == 0) {
        uint32_t u[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) u[c] = __float_as_uint(sl[c]);
        tmem_st_32x32b_x32(trow + kTmemSlots + (uint32_t)col0, u);
        tmem_st_wait();
      }
    }
    {  // fold h = 128, thread-local
      uint32_t u[32];
      tmem_ld_32x32b_x32(trow + kTmemSlots + (uint32_t)col0, u);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; ++c) sl[c] = __uint_as_float(u[c]) + sl[c];
    }
    // h = 64 (thread cq + 2 -> cq) and h = 32 (thread 1 -> 0) through TMEM
    if (cq >= 2) {
      uint32_t u[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) u[c] = __float_as_uint(sl[c]);
      tmem_st_32x32b_x32(trow + kTmemX + (uint32_t)(32 * (cq - 2)), u);
      tmem_st_wait();
    }
    xchg_barrier();
    if (cq < 2) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t u[16];
        tmem_ld_32x32b_x16(trow + kTmemX + (uint32_t)(32 * cq + 16 * half), u);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 16; ++c) sl[16 * half + c] = sl[16 * half + c] + __uint_as_float(u[c]);
      }
    }
    xchg_barrier();
    if (cq == 1) {
      uint32_t u[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) u[c] = __float_as_uint(sl[c]);
      tmem_st_32x32b_x32(trow + kTmemX, u);
      tmem_st_wait();
    }
    xchg_barrier();
    if (cq == 0) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t u[16];
        tmem_ld_32x32b_x16(trow + kTmemX + (uint32_t)(16 * half), u);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 16; ++c) sl[16 * half + c] = sl[16 * half + c] + __uint_as_float(u[c]);
      }
#pragma unroll
      for (int hh = 16; hh > 0; hh >>= 1)
#pragma unroll
        for (int c = 0; c < hh; ++c) sl[c] = sl[c] + sl[c + hh];
      tmem_st_32x32b_x1(trow + kTmemX + 32u, __float_as_uint(1.0f / sl[0]));
      tmem_st_wait();
    }
    xchg_barrier();
    float inv;
    {
      uint32_t u[4];
      tmem_ld_32x32b_x4(trow + kTmemX + 32u, u);
      tmem_ld_wait();
      inv = __uint_as_float(u[0]);
    }

    // ---- pass 3: P = bf16(bf16(e) * inv) in place ----
    for (int kt = 0; kt < n_kt; ++kt) {
      uint8_t *tile = sE + (size_t)kt * kAP;
      if (!(kt == qt && cq > qd)) {  // (a masked quarter holds zeros already)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 *u = p_unit(tile, r, cq, i);
          uint4 v = *u;
          uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) w[j] = pack_bf2(lo_f(w[j]) * inv, hi_f(w[j]) * inv);
          *u = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->p_full[kt]);
    }

    // ---- O: this thread's 16 head dims of its row ----
    const bool ok = mbar_wait(&ctl->o_full, 0, abort_flag, a.err, 0x142B);
    tc_fence_after();
    uint32_t o[16];
    tmem_ld_32x32b_x16(trow + kTmemO + (uint32_t)(16 * cq), o);
    tmem_ld_wait();
    if (ok && !*abort_flag && qpos < a.T) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = pack_bf2(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1]));
      uint16_t *dst = a.O + ((int64_t)b * a.T + qpos) * a.ldo + h * 64 + 16 * cq;
      if (a.vec_store) {
        reinterpret_cast<uint4 *>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4 *>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<uint32_t *>(dst)[i] = w[i];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

bool attention_prefill_tc_ok(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                             const uint16_t *Vc, int64_t seq_stride, int T, int n_head) {
  return T >= 1 && T <= kAMaxKT * kAK && n_head >= 1 && aligned16(Q) && aligned16(Kc) &&
         aligned16(Vc) && ldq % 8 == 0 && seq_stride % 8 == 0;
}

int launch_attention_prefill_tc(const uint16_t *Q, int64_t ldq, const uint16_t *Kc,
                                const uint16_t *Vc, int64_t seq_stride, int n_seq, int T,
                                int n_head, uint16_t *O, int64_t ldo, cudaStream_t stream) {
  int st;
  DeviceCtx *ctx = device_ctx(&st);
  if (!ctx) return st;
  const int d = n_head * 64;
  CUtensorMap tmQ, tmK, tmV;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  st = make_tmap_3d(&tmQ, Q, bf, (uint64_t)n_seq, (uint64_t)T, (uint64_t)d, (uint64_t)ldq * 2,
                    (uint64_t)T * ldq * 2, 64, kAQ);
  if (st) return st;
  st = make_tmap_3d(&tmK, Kc, bf, (uint64_t)n_seq, (uint64_t)T, (uint64_t)d, (uint64_t)d * 2,
                    (uint64_t)seq_stride * 2, 64, kAK);
  if (st) return st;
  st = make_tmap_3d(&tmV, Vc, bf, (uint64_t)n_seq, (uint64_t)T, (uint64_t)d, (uint64_t)d * 2,
                    (uint64_t)seq_stride * 2, 64, kAK);
  if (st) return st;
  AttnTcArgs a;
  a.T = T;
  a.n_qt = (T + kAQ - 1) / kAQ;
  a.O = O;
  a.ldo = ldo;
  a.vec_store = aligned16(O) && ldo % 8 == 0;
  a.err = ctx->err;
  a.p_bufs = 1;
  static bool attr[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return W8A8_ERR_CUDA;
  const dim3 grid(a.n_qt, n_head, n_seq);
  if (a.n_qt <= kEMaxKT) {
    // exponentials kept on chip: Q | K, then V | E tiles
    size_t smem = 1024 + (size_t)kATile * (1 + a.n_qt) + (size_t)kAP * a.n_qt + sizeof(AttnCtlE);
    // at least half of the SM's shared memory: one CTA per SM, which owns all
    // 512 TMEM columns
    if (smem < 116 * 1024) smem = 116 * 1024;
    if (!attr[dev][1]) {
      if (cudaFuncSetAttribute(attention_prefill_tc_e_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
          cudaSuccess)
        return W8A8_ERR_CUDA;
      attr[dev][1] = true;
    }
    launch_pdl(attention_prefill_tc_e_kernel, grid, dim3(kAThreads), smem, stream, tmQ, tmK, tmV,
               a);
    return check_launch("attention_prefill_tc_e");
  }
  const size_t base = 1024 + (size_t)kATile * (1 + a.n_qt + 2) + sizeof(AttnCtl);
  a.p_bufs = base + 2 * kAP <= 227 * 1024 ? 2 : 1;
  size_t smem = base + (size_t)a.p_bufs * kAP;
  if (smem < 116 * 1024) smem = 116 * 1024;
  if (!attr[dev][0]) {
    if (cudaFuncSetAttribute(attention_prefill_tc_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess)
      return W8A8_ERR_CUDA;
    attr[dev][0] = true;
  }
  launch_pdl(attention_prefill_tc_kernel, grid, dim3(kAThreads), smem, stream, tmQ, tmK, tmV, a);
  return check_launch("attention_prefill_tc");
}

}  // namespace w8a8
