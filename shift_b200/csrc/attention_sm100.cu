// Causal flash attention on the 5th-generation tensor cores (sm_100a).
//
// Layout: q/k/v are read straight from the fused QKV projection
// [T, (Hq + 2 Hkv) * 64] with TMA (one 2D map over the whole activation), the
// output O is written as [T, Hq * 64].  head_dim = 64, tiles of 128 queries x
// 128 keys, GQA by mapping query head h to kv head h / (Hq / Hkv).  The
// softmax runs in base 2 on scores pre-multiplied by scale*log2(e); the
// per-row log-sum-exp (base 2) is saved for the backward.
//
// Forward (one CTA per 128 queries of one head; default form `fwd_split_kernel`):
//   warp 0   TMA: Q once, then K_j and V_j into separate 3-stage rings
//   warp 1   TMEM allocation + single-thread tcgen05.mma issue:
//              S_j = Q K_j^T   (128x128x64, TMEM, triple-buffered)
//              O  += P_j V_j   (128x64x128, TMEM, one accumulator per block parity)
//   warps 2-9 softmax, two warps per query row group (= TMEM lane quarter)
//              taking alternate key blocks: each reads whole rows of S_j with
//              tcgen05.ld, keeps its own online max / sum, writes P_j (bf16)
//              into 128B-swizzled shared memory for the next MMA and rescales
//              its O in TMEM only when the row max rises by more than 2^8; the
//              two partial results are merged once at the end.
//   Two older forms stay selectable (SHIFT_ATTN_FWD=fold | tmem): the pair
//   shares each key block (half the columns each) and O is folded into
//   registers or accumulated in TMEM.
// Backward (deterministic, no atomics):
//   dkdv kernel: one CTA per 128 keys of one KV head, looping over every
//              query head of the group and every query block at or after the
//              diagonal: S^T = K Q^T, dP^T = V dO^T (TMEM); P^T and
//              dS^T = P^T (dP^T - delta) go to shared memory; dV += P^T dO,
//              dK += dS^T Q accumulate in TMEM for the whole loop.
//   dq kernel:   one CTA per 128 queries of one head, looping over key blocks:
//              S = Q K^T, dP = dO V^T, dS -> shared memory, dQ += dS K in TMEM.
//   The same 128B-swizzled tile of Q, dO or K serves both as a K-major and as
//   an MN-major MMA operand, so each is loaded once.
// Every mbarrier wait is bounded; on expiry the kernel records a status code
// and winds down (waits for its own MMAs, frees TMEM) instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"

namespace sb {
namespace fa {

constexpr int D = 64;
constexpr int BM = 128;
constexpr int BN = 128;
// warp 0: TMA producer, warp 1: TMEM owner + MMA issuer, then the softmax /
// epilogue warps.  Forward: two softmax warps share each TMEM lane quarter
// (warp % 4) and split the 128 columns of a tile (half = (warp - 2) / 4).
// Backward: four warps per quarter, each taking 16 of a 64-column sub-block
// (no cross-warp reductions there: lse and delta are given), which gives the
// SM four times the warps to hide TMEM-load and exponent latencies.  (Four
// warps per quarter in the forward measured slower -- 0.312 vs 0.257 ms at
// B 8, S 2048 -- its row max / sum exchange spans twice the warps.)
constexpr int kThreads = 320;
constexpr int kSoftThreads = 256;
constexpr int kTile = 128 * 128;   // bytes of one 128 x 64 bf16 tile
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  int B, S, Hq, Hkv;
  float scale_log2, scale;
  __nv_bfloat16* o;
  float* lse;
  const float* delta;
  __nv_bfloat16* dqkv;
  int dqkv_stride;
  int o_stride;
  int* status;
  int hsplit;        // dK/dV: CTAs per (key block, kv head), each over group/hsplit query heads
  float* ws;         // hsplit > 1: fp32 partials [B, Hkv, hsplit, S, 2*D] (dK scaled | dV)
};

SB_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA and integer pipes, for x <= 127, to take part of the
// softmax's exponentials off the 16-per-clock MUFU unit.  Cody-Waite style
// range reduction: x = j + r with j = round(x) (the 1.5 * 2^23 shifter puts j
// in the low mantissa bits of t) and r in [-1/2, 1/2]; 2^r from a cubic fitted
// here by iteratively re-weighted least squares on the relative error (max
// relative error 7.5e-5, far below the bf16 rounding of P); j is added to the
// exponent field with an integer add.  Inputs below -126 are clamped (their
// probabilities are below bf16's smallest normal anyway).
SB_DEVICE float ex2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float r = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.055171531f, r, 0.24261111f), r, 0.69326103f), r, 0.99992806f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));   // unsigned: wraps, no overflow
}

// 16-byte chunk c (0..15) of row r of a [128 x 128] bf16 operand stored as two
// K-major 128B-swizzled halves of 64 columns (16 KB each).
SB_DEVICE uint8_t* swz_chunk(uint8_t* base, int r, int c) {
  return base + (c >> 3) * kTile + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

SB_DEVICE uint64_t kdesc(uint32_t addr) { return make_sw128_desc(addr, 16, 1024); }
SB_DEVICE uint64_t mndesc(uint32_t addr) { return make_sw128_desc(addr, 8192, 1024); }

SB_DEVICE void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Work order of the causal grids: a (row block, head, batch) tile's cost grows
// with its distance from the diagonal, so the launch order is re-mapped to put
// the costliest blocks of every head and batch first (longest-processing-time
// first): the last wave then holds the cheap blocks instead of a few long
// ones, which matters most when B x heads is small (one sequence per
// pipeline microbatch).  Returns the block index along x, counted from the
// costliest; y and z are the remaining coordinates.
SB_DEVICE void lpt_coords(int& costliest_rank, int& y, int& z) {
  const int yz = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  costliest_rank = lin / yz;
  const int r = lin % yz;
  y = r % gridDim.y;
  z = r / gridDim.y;
}

// ============================ forward ============================
constexpr int kFwdStages = 2;
constexpr int kFwdSmem = 1024 + kTile /*Q*/ + 2 * kFwdStages * kTile /*K,V*/ + 2 * 2 * kTile /*P x2*/ + 256 +
                         (2 * 2 * 128 + 2 * 128) * 4 /*row max / sum exchange*/;

// kTmemO: O accumulates in TMEM across the key blocks and the softmax warps
// keep a running row max that may be stale by up to 2^kRescaleLog2: O (and the
// row sum) are rescaled in place only when a row's max rises by more than
// that, which on these shapes happens in the first blocks of a row and rarely
// after, so the common block costs no TMEM read of O and no rescale FMAs.
// Otherwise (kTmemO false) every block's P V lands in a fresh TMEM block that
// the softmax warps fold into registers with the running rescale.
constexpr float kRescaleLog2 = 8.f;

template <bool kTmemO>
__global__ void __launch_bounds__(kThreads, 1)
fwd_kernel(const __grid_constant__ CUtensorMap tm, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + kTile;
  uint8_t* sV = sK + kFwdStages * kTile;
  uint8_t* sP = sV + kFwdStages * kTile;      // 2 buffers x 32 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 4 * kTile);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;
  uint64_t* kv_empty = kv_full + kFwdStages;
  uint64_t* s_full = kv_empty + kFwdStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* drain = o_full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  // row-max exchange between the two softmax warps of a lane quarter,
  // double-buffered by block parity: [parity][half][row]; then the row sums
  float* s_max = reinterpret_cast<float*>(tslot + 4);
  float* s_sum = s_max + 2 * 2 * BM;

  int rank_x, h, b;
  lpt_coords(rank_x, h, b);
  const int qb = gridDim.x - 1 - rank_x;     // query block qb sees qb + 1 key blocks
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = qb * BM;
  const int tok0 = b * p.S;
  const int n_kv = qb + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kSoftThreads);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_2d(sQ, &tm, q_full, h * D, tok0 + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % kFwdStages;
        if (!mbar_wait(&kv_empty[st], ((j / kFwdStages) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
        tma_load_2d(sK + st * kTile, &tm, &kv_full[st], (p.Hq + kvh) * D, tok0 + j * BN);
        tma_load_2d(sV + st * kTile, &tm, &kv_full[st], (p.Hq + p.Hkv + kvh) * D, tok0 + j * BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t idO = make_idesc_bf16(BM, D, 0, 1);
      const uint32_t qa = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.status);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kFwdStages;
        if (!mbar_wait(&kv_full[st], (j / kFwdStages) & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + st * kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tbase + (j & 1) * BN, kdesc(qa + kk * 32), kdesc(ka + kk * 32), idS, kk > 0);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status)) break;
        tc_fence_after();
        const int st = j % kFwdStages;
        const uint32_t pa = smem_u32(sP + (j & 1) * 2 * kTile);
        const uint32_t va = smem_u32(sV + st * kTile);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16(kTmemO ? tbase + 256 : tbase + 256 + (j & 1) * D,
                   kdesc(pa + (kk >> 2) * kTile + (kk & 3) * 32), mndesc(va + kk * 2048), idO,
                   kTmemO ? (j > 0 || kk > 0) : kk > 0);
        umma_commit(&o_full[j & 1]);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else if (kTmemO) {
    // -------------------- softmax, O accumulated in TMEM --------------------
    const int quarter = warp % 4;
    const int half = (warp - 2) / 4;          // columns [64*half, 64*half+64) of S, [32*half, +32) of O
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int pair_bar = 1 + quarter;
    const uint32_t to = tbase + 256 + half * 32 + lane_off;   // this warp's 32 columns of O
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (ok && !mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.status)) ok = false;
      ok = __all_sync(0xffffffffu, ok);       // warp-uniform before the warp-collective TMEM accesses
      if (ok) tc_fence_after();
      const uint32_t ts = tbase + (j & 1) * BN + lane_off;
      const bool diag = (j == qb);
      uint32_t v[64];
      float mraw = -INFINITY;
      const int c_lo = half * 64;
      if (ok) {
        tmem_ld_32x32b_x32(ts + c_lo, v);
        tmem_ld_32x32b_x32(ts + c_lo + 32, v + 32);
        tmem_wait_ld();
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (diag) {
          const int lim = q - j * BN - c_lo;
#pragma unroll
          for (int t = 0; t < 64; ++t)
            if (t <= lim) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 64; ++t) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
        }
        mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      float mx = fmaxf(m_run, mraw * p.scale_log2);
      s_max[((j & 1) * 2 + half) * BM + row] = mx;
      named_bar(pair_bar, 64);
      if (!ok) continue;
      mx = fmaxf(mx, s_max[((j & 1) * 2 + (half ^ 1)) * BM + row]);
      // the two warps of a pair hold the same rows and maxima, so they take the
      // same branch; each rescales its own 32 columns of O
      bool waited_prev = false;
      if (__any_sync(0xffffffffu, mx > m_run + kRescaleLog2)) {
        if (j > 0) {
          // O must hold every earlier block before it is read and rewritten
          if (!__all_sync(0xffffffffu, mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status))) {
            ok = false;
            continue;
          }
          waited_prev = true;
          tc_fence_after();
          const float a = ex2(m_run - mx);
          uint32_t o[32];
          tmem_ld_32x32b_x32(to, o);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * a);
          tmem_st_32x32b_x16(to, o);
          tmem_st_32x32b_x16(to + 16, o + 16);
          tmem_wait_st();
          l_run *= a;
        }
        m_run = mx;
      }
      // this block's P buffer was last read by the PV product of block j - 2
      if (j >= 2 && !waited_prev &&
          !__all_sync(0xffffffffu, mbar_wait(&o_full[j & 1], ((j - 2) >> 1) & 1, p.status))) {
        ok = false;
        continue;
      }
      uint8_t* pbuf = sP + (j & 1) * 2 * kTile;
      const float nmx = -m_run;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float pr[32];
        if (diag) {
          const int lim = q - j * BN - c_lo - cc * 32;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            pr[t] = (t > lim) ? 0.f : ex2(fmaf(__uint_as_float(v[cc * 32 + t]), p.scale_log2, nmx));
            l4[t & 3] += pr[t];
          }
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            pr[t] = ex2(fmaf(__uint_as_float(v[cc * 32 + t]), p.scale_log2, nmx));
            l4[t & 3] += pr[t];
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          bf16x8 pk = float_to_bf16x8(pr + 8 * u);
          *reinterpret_cast<uint4*>(swz_chunk(pbuf, row, ((c_lo + cc * 32) >> 3) + u)) =
              make_uint4(pk.w[0], pk.w[1], pk.w[2], pk.w[3]);
        }
      }
      l_run += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    s_sum[half * BM + row] = l_run;
    named_bar(pair_bar, 64);
    l_run += s_sum[(half ^ 1) * BM + row];
    if (ok) ok = mbar_wait(&o_full[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, p.status);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      uint32_t o[32];
      tmem_ld_32x32b_x32(to, o);
      tmem_wait_ld();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = p.o + static_cast<long>(tok0 + q) * p.o_stride + h * D + half * 32;
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float t8[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) t8[t] = __uint_as_float(o[c + t]) * inv;
        *reinterpret_cast<bf16x8*>(orow + c) = float_to_bf16x8(t8);
      }
      if (half == 0) p.lse[(static_cast<long>(b) * p.Hq + h) * p.S + q] = m_run + log2f(l_run);
    }
  } else {
    // ----------------------------- softmax -----------------------------
    const int quarter = warp % 4;
    const int half = (warp - 2) / 4;          // columns [64*half, 64*half+64) of S, [32*half, +32) of O
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int pair_bar = 1 + quarter;         // named barrier of the two warps of this quarter
    float m_run = -INFINITY, l_run = 0.f, m_fold = -INFINITY;
    float o_acc[D / 2];
#pragma unroll
    for (int i = 0; i < D / 2; ++i) o_acc[i] = 0.f;
    bool ok = true;
    auto fold = [&](int i, float m_i) -> bool {
      if (!mbar_wait(&o_full[i & 1], (i >> 1) & 1, p.status)) return false;
      tc_fence_after();
      const float a = (m_fold == -INFINITY) ? 0.f : ex2(m_fold - m_i);
      uint32_t v[32];
      tmem_ld_32x32b_x32(tbase + 256 + (i & 1) * D + half * 32 + lane_off, v);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 32; ++t) o_acc[t] = o_acc[t] * a + __uint_as_float(v[t]);
      m_fold = m_i;
      return true;
    };
    // Both warps of a pair run every iteration's named barrier even after a
    // bounded wait failed (they then skip the work), so a failure in one warp
    // can never leave its partner blocked on the barrier.
    for (int j = 0; j < n_kv; ++j) {
      if (ok && !mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.status)) ok = false;
      if (ok) tc_fence_after();
      const uint32_t ts = tbase + (j & 1) * BN + lane_off;
      const bool diag = (j == qb);
      // pass 1: this warp's 64 columns of S come out of TMEM once (two loads,
      // one wait) and stay in registers for pass 2.  Row max over them (the
      // causal mask only exists on the diagonal tile) in four independent
      // chains, scaled once, then combined with the partner warp's.
      uint32_t v[64];
      float mraw = -INFINITY;
      const int c_lo = half * 64;
      if (ok) {
        tmem_ld_32x32b_x32(ts + c_lo, v);
        tmem_ld_32x32b_x32(ts + c_lo + 32, v + 32);
        tmem_wait_ld();
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (diag) {
          const int lim = q - j * BN - c_lo;       // columns t <= lim are visible
#pragma unroll
          for (int t = 0; t < 64; ++t)
            if (t <= lim) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 64; ++t) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
        }
        mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      float mx = fmaxf(m_run, mraw * p.scale_log2);
      s_max[((j & 1) * 2 + half) * BM + row] = mx;
      named_bar(pair_bar, 64);
      if (!ok) continue;
      mx = fmaxf(mx, s_max[((j & 1) * 2 + (half ^ 1)) * BM + row]);
      const float m_prev = m_run;
      m_run = mx;
      // pass 2: probabilities -> shared memory (bf16, swizzled); the row sum
      // of this tile in four independent chains
      uint8_t* pbuf = sP + (j & 1) * 2 * kTile;
      const float nmx = -mx;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float pr[32];
        if (diag) {
          const int lim = q - j * BN - c_lo - cc * 32;
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            pr[t] = (t > lim) ? 0.f : ex2(fmaf(__uint_as_float(v[cc * 32 + t]), p.scale_log2, nmx));
            l4[t & 3] += pr[t];
          }
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            pr[t] = ex2(fmaf(__uint_as_float(v[cc * 32 + t]), p.scale_log2, nmx));
            l4[t & 3] += pr[t];
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          bf16x8 pk = float_to_bf16x8(pr + 8 * u);
          *reinterpret_cast<uint4*>(swz_chunk(pbuf, row, ((c_lo + cc * 32) >> 3) + u)) =
              make_uint4(pk.w[0], pk.w[1], pk.w[2], pk.w[3]);
        }
      }
      l_run = ((m_prev == -INFINITY) ? 0.f : l_run * ex2(m_prev - mx)) + ((l4[0] + l4[1]) + (l4[2] + l4[3]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      if (j >= 1 && !fold(j - 1, m_prev)) ok = false;
    }
    if (ok) ok = fold(n_kv - 1, m_run);
    // row sum = both halves' partial sums (same running max)
    s_sum[half * BM + row] = l_run;
    named_bar(pair_bar, 64);
    l_run += s_sum[(half ^ 1) * BM + row];
    if (ok) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = p.o + static_cast<long>(tok0 + q) * p.o_stride + h * D + half * 32;
#pragma unroll
      for (int c = 0; c < D / 2; c += 8) {
        float t8[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) t8[t] = o_acc[c + t] * inv;
        *reinterpret_cast<bf16x8*>(orow + c) = float_to_bf16x8(t8);
      }
      if (half == 0) p.lse[(static_cast<long>(b) * p.Hq + h) * p.S + q] = m_run + log2f(l_run);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ------------------- forward, key blocks split between the pair -------------------
// The two softmax warps of a TMEM lane quarter take alternate key blocks
// (warp parity 0: j = 0, 2, 4, ...; parity 1: j = 1, 3, 5, ...) and each owns
// whole 128-column rows of S, so they need no exchange per block: they drift
// apart, and one warp's exponent phase overlaps the other's TMEM-load / row-max
// phase on the same scheduler, which keeps the MUFU pipe busy (with a shared
// block the pair reached every phase together).  Each parity keeps its own
// online-softmax state and its own O accumulator in TMEM (P V accumulates; O is
// rescaled in place only when the row max rises by more than 2^kRescaleLog2);
// the two partial results are merged once at the end.  S is triple-buffered in
// TMEM (3 x 128 columns + 2 x 64 for the O blocks = all 512), and K / V have
// separate three-stage rings, so the tensor core runs ahead of both warps.
constexpr int kSplitStages = 3;
constexpr int kSplitSmem = 1024 + kTile /*Q*/ + 2 * kSplitStages * kTile /*K,V*/ + 2 * 2 * kTile /*P x2*/ + 256 +
                           2 * 2 * BM * 4 /*partner m, l*/;

// kFma: how many of every 8 probabilities are computed with ex2_fma instead of
// the MUFU exponent (0 = all on MUFU).
template <int kFma>
__global__ void __launch_bounds__(kThreads, 1)
fwd_split_kernel(const __grid_constant__ CUtensorMap tm, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + kTile;
  uint8_t* sV = sK + kSplitStages * kTile;
  uint8_t* sP = sV + kSplitStages * kTile;    // 2 buffers x 32 KB, buffer = block parity
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 4 * kTile);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;
  uint64_t* k_empty = k_full + kSplitStages;
  uint64_t* v_full = k_empty + kSplitStages;
  uint64_t* v_empty = v_full + kSplitStages;
  uint64_t* s_full = v_empty + kSplitStages;  // S buffer j % 3
  uint64_t* p_full = s_full + kSplitStages;   // P buffer j & 1
  uint64_t* o_full = p_full + 2;              // P V of a block of parity j & 1 done
  uint64_t* drain = o_full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_ml = reinterpret_cast<float*>(tslot + 4);   // [parity][m | l][row]

  int rank_x, h, b;
  lpt_coords(rank_x, h, b);
  const int qb = gridDim.x - 1 - rank_x;
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = qb * BM;
  const int tok0 = b * p.S;
  const int n_kv = qb + 1;
  constexpr uint32_t kOCol = 3 * BN;          // O block of parity r at kOCol + r * D

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kSplitStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], kSoftThreads / 2);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_2d(sQ, &tm, q_full, h * D, tok0 + q0);
      // K runs one block ahead of V: K_j is free once S_j is computed, V_j only
      // after P_j V_j
      auto load = [&](int j, bool is_v) -> bool {
        const int st = j % kSplitStages;
        uint64_t* empty = is_v ? &v_empty[st] : &k_empty[st];
        uint64_t* full = is_v ? &v_full[st] : &k_full[st];
        if (!mbar_wait(empty, ((j / kSplitStages) & 1) ^ 1, p.status)) return false;
        mbar_arrive_expect_tx(full, kTile);
        tma_load_2d((is_v ? sV : sK) + st * kTile, &tm, full, (p.Hq + (is_v ? p.Hkv : 0) + kvh) * D,
                    tok0 + j * BN);
        return true;
      };
      bool ok = load(0, false);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv) ok = load(j + 1, false);
        if (ok) ok = load(j, true);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t idO = make_idesc_bf16(BM, D, 0, 1);
      const uint32_t qa = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.status);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kSplitStages;
        if (!mbar_wait(&k_full[st], (j / kSplitStages) & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + st * kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tbase + st * BN, kdesc(qa + kk * 32), kdesc(ka + kk * 32), idS, kk > 0);
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      for (int j = 0; j < kSplitStages && j < n_kv && ok; ++j) ok = issue_s(j);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.status)) break;
        const int st = j % kSplitStages;
        if (!mbar_wait(&v_full[st], (j / kSplitStages) & 1, p.status)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sP + (j & 1) * 2 * kTile);
        const uint32_t va = smem_u32(sV + st * kTile);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16(tbase + kOCol + (j & 1) * D, kdesc(pa + (kk >> 2) * kTile + (kk & 3) * 32),
                   mndesc(va + kk * 2048), idO, (j >= 2 || kk > 0));
        umma_commit(&o_full[j & 1]);
        umma_commit(&v_empty[st]);
        // P_j written means S_j has been read: its buffer takes S_{j+3}
        if (j + kSplitStages < n_kv && !issue_s(j + kSplitStages)) break;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    const int quarter = warp % 4;
    const int par = (warp - 2) / 4;
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t to = tbase + kOCol + par * D + lane_off;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int last = -1;
    for (int j = par; j < n_kv; j += 2) {
      const int st = j % kSplitStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[st], (j / kSplitStages) & 1, p.status))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tbase + st * BN + lane_off;
      const bool diag = (j == qb);
      // the whole 128-column row of S stays in registers for both passes
      uint32_t v[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) tmem_ld_32x32b_x32(ts + c, v + c);
      tmem_wait_ld();
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (diag) {
#pragma unroll
        for (int t = 0; t < BN; ++t)
          if (t <= row) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
      } else {
#pragma unroll
        for (int t = 0; t < BN; ++t) m4[t & 3] = fmaxf(m4[t & 3], __uint_as_float(v[t]));
      }
      const float mx = fmaxf(m_run, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2);
      // P V of this parity's previous block must be complete before its P
      // buffer is rewritten or its O block rescaled
      if (j >= 2) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[par], ((j - 2) >> 1) & 1, p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, mx > m_run + kRescaleLog2)) {
        if (j >= 2) {
          const float a = ex2(m_run - mx);
#pragma unroll
          for (int c = 0; c < D; c += 32) {         // 32 columns at a time: S is still live
            uint32_t o[32];
            tmem_ld_32x32b_x32(to + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * a);
            tmem_st_32x32b_x16(to + c, o);
            tmem_st_32x32b_x16(to + c + 16, o + 16);
          }
          tmem_wait_st();
          l_run *= a;
        }
        m_run = mx;
      }
      uint8_t* pbuf = sP + par * 2 * kTile;
      const float nmx = -m_run;
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < BN; c += 8) {
        float pr[8];                              // probabilities overwrite S eight at a time
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float z = fmaf(__uint_as_float(v[c + t]), p.scale_log2, nmx);
          pr[t] = (diag && c + t > row) ? 0.f : (t >= 8 - kFma ? ex2_fma(z) : ex2(z));
          l4[t & 3] += pr[t];
        }
        bf16x8 pk = float_to_bf16x8(pr);
        *reinterpret_cast<uint4*>(swz_chunk(pbuf, row, c >> 3)) = make_uint4(pk.w[0], pk.w[1], pk.w[2], pk.w[3]);
      }
      l_run += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[par]);
      last = j;
    }
    if (ok && last >= 0) ok = mbar_wait(&o_full[par], (last >> 1) & 1, p.status);
    ok = __all_sync(0xffffffffu, ok);
    s_ml[(par * 2) * BM + row] = ok ? m_run : NAN;
    s_ml[(par * 2 + 1) * BM + row] = l_run;
    named_bar(1 + quarter, 64);
    if (par == 0) {
      const float mb = s_ml[2 * BM + row], lb = s_ml[3 * BM + row];
      // the partner had no block (a single-block row) or ran out of a wait
      ok = ok && __all_sync(0xffffffffu, !isnan(mb));
      if (ok) {
        const float m = fmaxf(m_run, mb);
        const float aa = ex2(m_run - m);
        const float ab = (mb == -INFINITY) ? 0.f : ex2(mb - m);
        const float l = l_run * aa + lb * ab;
        const bool has_b = n_kv > 1;
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* orow = p.o + static_cast<long>(tok0 + q) * p.o_stride + h * D;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t oa[32], ob[32];
          tmem_ld_32x32b_x32(to + c0, oa);
          if (has_b) tmem_ld_32x32b_x32(to + D + c0, ob);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float t8[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              t8[t] = (__uint_as_float(oa[c + t]) * aa + (has_b ? __uint_as_float(ob[c + t]) * ab : 0.f)) * inv;
            *reinterpret_cast<bf16x8*>(orow + c0 + c) = float_to_bf16x8(t8);
          }
        }
        p.lse[(static_cast<long>(b) * p.Hq + h) * p.S + q] = m + log2f(l);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ============================ backward: dK, dV ============================
// One CTA per (key block of 128, kv head [, head split], batch).  The query
// blocks of every head of the group are walked in 64-query sub-blocks k:
//   S^T_k = K Q_k^T and dP^T_k = V dO_k^T  -> TMEM buffer k & 1 (64 columns each)
//   softmax warps: P^T = exp2(S^T * scale - lse), dS^T = P^T (dP^T - delta)
//                  -> swizzled smem buffer k & 1 (bf16, 128 keys x 64 queries)
//   dV += P^T dO_k, dK += dS^T Q_k  (accumulated in TMEM across all k)
// With two S/dP buffers the tensor core computes S_{k+1} while the softmax
// warps work on k, and the dV/dK update of k-1 overlaps the softmax of k.
constexpr int kBwdStages = 2;
// as in the forward: four softmax warps per TMEM lane quarter, each taking 16
// of a 64-column sub-block, 16 softmax warps in all
constexpr int kBwdSplit = 4;
constexpr int kBwdSoft = 128 * kBwdSplit;
constexpr int kBwdThreads = 64 + kBwdSoft;
constexpr int kBwdCols = 64 / kBwdSplit;              // columns of a sub-block per softmax warp
constexpr int kBwdOut = D / kBwdSplit;                // dK / dV / dQ columns per softmax warp in the epilogue
constexpr int kDkdvSmem = 1024 + 2 * kTile /*K,V*/ + 2 * kBwdStages * kTile /*Q,dO*/ + 4 * kTile /*P^T,dS^T x2*/ +
                          2 * BM * 4 * 2 /*lse,delta*/ + 256;

__global__ void __launch_bounds__(kBwdThreads, 1)
dkdv_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sK = sm;
  uint8_t* sV = sK + kTile;
  uint8_t* sQ = sV + kTile;                       // stages x kTile (128 queries x 64 d)
  uint8_t* sO = sQ + kBwdStages * kTile;          // dO, stages x kTile
  uint8_t* sP = sO + kBwdStages * kTile;          // P^T  [2 buffers] x (128 keys x 64 queries)
  uint8_t* sS = sP + 2 * kTile;                   // dS^T [2 buffers]
  float* s_lse = reinterpret_cast<float*>(sS + 2 * kTile);   // [2][BM], by iteration parity
  float* s_del = s_lse + 2 * BM;                               // [2][BM]
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_del + 2 * BM);
  uint64_t* kv_full = bar;
  uint64_t* qo_full = bar + 1;
  uint64_t* qo_empty = qo_full + kBwdStages;
  uint64_t* sdp_full = qo_empty + kBwdStages;     // [2]
  uint64_t* sdp_empty = sdp_full + 2;             // [2]
  uint64_t* ds_full = sdp_empty + 2;              // [2]
  uint64_t* pds_empty = ds_full + 2;              // [2]
  uint64_t* acc_done = pds_empty + 2;
  uint64_t* drain = acc_done + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);

  // At small batch a causal key block near the start of the sequence is the
  // critical path (it meets every later query block of every head of its
  // group); with hsplit > 1 the group's query heads are spread over hsplit
  // CTAs whose fp32 partials are summed in a fixed order afterwards.
  int kb, yy, b;
  lpt_coords(kb, yy, b);                     // key block kb is seen by S/BM - kb query blocks
  const int kvh = yy / p.hsplit, part_h = yy % p.hsplit;
  const int group = p.Hq / p.Hkv / p.hsplit;     // query heads handled by this CTA
  const int h_first = kvh * (p.Hq / p.Hkv) + part_h * group;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int k0 = kb * BN;
  const int tok0 = b * p.S;
  const int n_q = p.S / BM;
  const int per_head = n_q - kb;
  const int n_it = group * per_head;              // 128-query blocks
  const int n_sub = 2 * n_it;                     // 64-query sub-blocks

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&qo_full[s], 1);
      mbar_init(&qo_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&sdp_empty[i], kBwdSoft);
      mbar_init(&ds_full[i], kBwdSoft);
      mbar_init(&pds_empty[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  // S^T / dP^T double buffers of 64 columns, then the dV / dK accumulators
  const uint32_t tS0 = tbase, tdP0 = tbase + 128, tdV = tbase + 256, tdK = tbase + 320;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      tma_prefetch_desc(&tmo);
      mbar_arrive_expect_tx(kv_full, 2 * kTile);
      tma_load_2d(sK, &tm, kv_full, (p.Hq + kvh) * D, tok0 + k0);
      tma_load_2d(sV, &tm, kv_full, (p.Hq + p.Hkv + kvh) * D, tok0 + k0);
      for (int it = 0; it < n_it; ++it) {
        const int h = h_first + it / per_head;
        const int qb = kb + it % per_head;
        const int st = it % kBwdStages;
        if (!mbar_wait(&qo_empty[st], ((it / kBwdStages) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&qo_full[st], 2 * kTile);
        tma_load_2d(sQ + st * kTile, &tm, &qo_full[st], h * D, tok0 + qb * BM);
        tma_load_2d(sO + st * kTile, &tmo, &qo_full[st], h * D, tok0 + qb * BM);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BN, 64, 0, 0);   // [keys x 64 queries], K = d
      constexpr uint32_t idG = make_idesc_bf16(BN, D, 0, 1);    // [keys x d], K = 64 queries
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, p.status);
      // k: issue S/dP of sub-block k (k < n_sub), then dV/dK of sub-block k-1
      for (int k = 0; k <= n_sub && ok; ++k) {
        if (k < n_sub) {
          const int it = k >> 1, hh = k & 1, st = it % kBwdStages;
          if (hh == 0 && !mbar_wait(&qo_full[st], (it / kBwdStages) & 1, p.status)) break;
          if (k >= 2 && !mbar_wait(&sdp_empty[k & 1], ((k - 2) >> 1) & 1, p.status)) break;
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ + st * kTile) + hh * 8192, oa = smem_u32(sO + st * kTile) + hh * 8192;
          const uint32_t ts = tS0 + (k & 1) * 64, tp = tdP0 + (k & 1) * 64;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            umma_f16(ts, kdesc(ka + kk * 32), kdesc(qa + kk * 32), idS, kk > 0);
            umma_f16(tp, kdesc(va + kk * 32), kdesc(oa + kk * 32), idS, kk > 0);
          }
          umma_commit(&sdp_full[k & 1]);
        }
        if (k >= 1) {
          const int kp = k - 1, it = kp >> 1, hh = kp & 1, st = it % kBwdStages;
          if (!mbar_wait(&ds_full[kp & 1], (kp >> 1) & 1, p.status)) break;
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ + st * kTile), oa = smem_u32(sO + st * kTile);
          const uint32_t pa = smem_u32(sP + (kp & 1) * kTile), da = smem_u32(sS + (kp & 1) * kTile);
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk) {
            const uint32_t acc = (kp > 0 || kk > 0) ? 1u : 0u;
            umma_f16(tdV, kdesc(pa + kk * 32), mndesc(oa + (hh * 4 + kk) * 2048), idG, acc);
            umma_f16(tdK, kdesc(da + kk * 32), mndesc(qa + (hh * 4 + kk) * 2048), idG, acc);
          }
          umma_commit(&pds_empty[kp & 1]);
          if (hh == 1) umma_commit(&qo_empty[st]);     // both halves of this Q / dO stage consumed
        }
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    const int quarter = warp % 4;
    const int part = (warp - 2) / 4;         // columns [16*part, +16) of a 64-query sub-block; of dK/dV
    const int row = quarter * 32 + lane;     // key row within the block
    const int key = k0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int sm_tid = threadIdx.x - 64;     // 0..kBwdSoft-1
    bool ok = true;
    // lse / delta of the 128-query block of iteration it live in buffer it & 1;
    // the next iteration's values are loaded into registers during the
    // current one and published by the barrier that ends it.  Every softmax
    // warp runs every barrier, also after a bounded wait failed (it then
    // skips the work), so no warp is left blocked on a barrier.
    auto li_of = [&](int it) -> long {
      const int hh = h_first + it / per_head;
      const int qq = kb + it % per_head;
      return (static_cast<long>(b) * p.Hq + hh) * p.S + qq * BM + sm_tid;
    };
    if (sm_tid < BM) {
      s_lse[sm_tid] = p.lse[li_of(0)];
      s_del[sm_tid] = p.delta[li_of(0)];
    }
    named_bar(1, kBwdSoft);
    for (int it = 0; it < n_it; ++it) {
      const int qb = kb + it % per_head;
      const int buf = it & 1;
      float nl = 0.f, nd = 0.f;
      const bool pre = sm_tid < BM && it + 1 < n_it;
      if (pre) {
        nl = p.lse[li_of(it + 1)];
        nd = p.delta[li_of(it + 1)];
      }
      const float* cl = s_lse + buf * BM;
      const float* cd = s_del + buf * BM;
      for (int hh = 0; hh < 2; ++hh) {
        const int k = 2 * it + hh;
        const int q0 = qb * BM + hh * 64;              // first query of the sub-block
        if (ok && !mbar_wait(&sdp_full[k & 1], (k >> 1) & 1, p.status)) ok = false;
        if (!ok) continue;
        tc_fence_after();
        uint32_t vs[kBwdCols], vd[kBwdCols];
        tmem_ld_32x32b_x16(tS0 + (k & 1) * 64 + part * kBwdCols + lane_off, vs);
        tmem_ld_32x32b_x16(tdP0 + (k & 1) * 64 + part * kBwdCols + lane_off, vd);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&sdp_empty[k & 1]);                 // S/dP buffer may be overwritten by S_{k+2}
        const int c0 = hh * 64 + part * kBwdCols;       // column of the 128-query block
        float pt[kBwdCols], dst[kBwdCols];
        // lse / delta of the 16 queries: four 16-byte broadcast loads each
        // (c0 is a multiple of 16 floats; the arrays start 1024-byte aligned)
        const float4* cl4 = reinterpret_cast<const float4*>(cl + c0);
        const float4* cd4 = reinterpret_cast<const float4*>(cd + c0);
#pragma unroll
        for (int u = 0; u < kBwdCols / 4; ++u) {
          const float4 l = cl4[u], d = cd4[u];
          const float la[4] = {l.x, l.y, l.z, l.w}, da[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 4 * u + e;
            const float pv = ex2(fmaf(__uint_as_float(vs[t]), p.scale_log2, -la[e]));
            pt[t] = pv;
            dst[t] = pv * (__uint_as_float(vd[t]) - da[e]);
          }
        }
        if (qb == kb) {             // causal mask only on the diagonal block
#pragma unroll
          for (int t = 0; t < kBwdCols; ++t)
            if (key > q0 + part * kBwdCols + t) pt[t] = dst[t] = 0.f;
        }
        if (k >= 2 && !mbar_wait(&pds_empty[k & 1], ((k - 2) >> 1) & 1, p.status)) {
          ok = false;
          continue;
        }
        uint8_t* pb = sP + (k & 1) * kTile;
        uint8_t* db = sS + (k & 1) * kTile;
#pragma unroll
        for (int u = 0; u < kBwdCols / 8; ++u) {
          bf16x8 a = float_to_bf16x8(pt + 8 * u);
          bf16x8 d = float_to_bf16x8(dst + 8 * u);
          const int ch = part * (kBwdCols / 8) + u;
          *reinterpret_cast<uint4*>(swz_chunk(pb, row, ch)) = make_uint4(a.w[0], a.w[1], a.w[2], a.w[3]);
          *reinterpret_cast<uint4*>(swz_chunk(db, row, ch)) = make_uint4(d.w[0], d.w[1], d.w[2], d.w[3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&ds_full[k & 1]);
      }
      if (pre) {
        s_lse[(buf ^ 1) * BM + sm_tid] = nl;
        s_del[(buf ^ 1) * BM + sm_tid] = nd;
      }
      named_bar(1, kBwdSoft);   // next buffer written; everyone done with this one
    }
    if (ok && p.hsplit > 1 && mbar_wait(acc_done, 0, p.status)) {
      tc_fence_after();
      uint32_t v[kBwdOut];
      float* wrow = p.ws + ((((static_cast<long>(b) * p.Hkv + kvh) * p.hsplit + part_h) * p.S) + key) * (2 * D);
      {
        const int c = part * kBwdOut;
        tmem_ld_32x32b_x16(tdK + c + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < kBwdOut; t += 4)
          *reinterpret_cast<float4*>(wrow + c + t) =
              make_float4(__uint_as_float(v[t]) * p.scale, __uint_as_float(v[t + 1]) * p.scale,
                          __uint_as_float(v[t + 2]) * p.scale, __uint_as_float(v[t + 3]) * p.scale);
        tmem_ld_32x32b_x16(tdV + c + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < kBwdOut; t += 4)
          *reinterpret_cast<float4*>(wrow + D + c + t) = make_float4(
              __uint_as_float(v[t]), __uint_as_float(v[t + 1]), __uint_as_float(v[t + 2]), __uint_as_float(v[t + 3]));
      }
    } else if (ok && mbar_wait(acc_done, 0, p.status)) {
      tc_fence_after();
      uint32_t v[kBwdOut];
      __nv_bfloat16* krow = p.dqkv + static_cast<long>(tok0 + key) * p.dqkv_stride + (p.Hq + kvh) * D;
      __nv_bfloat16* vrow = p.dqkv + static_cast<long>(tok0 + key) * p.dqkv_stride + (p.Hq + p.Hkv + kvh) * D;
      {
        const int c = part * kBwdOut;
        float f[kBwdOut];
        tmem_ld_32x32b_x16(tdK + c + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < kBwdOut; ++t) f[t] = __uint_as_float(v[t]) * p.scale;
#pragma unroll
        for (int u = 0; u < kBwdOut / 8; ++u) reinterpret_cast<bf16x8*>(krow + c)[u] = float_to_bf16x8(f + 8 * u);
        tmem_ld_32x32b_x16(tdV + c + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < kBwdOut; ++t) f[t] = __uint_as_float(v[t]);
#pragma unroll
        for (int u = 0; u < kBwdOut / 8; ++u) reinterpret_cast<bf16x8*>(vrow + c)[u] = float_to_bf16x8(f + 8 * u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ============================ backward: dQ ============================
// One CTA per (query block of 128, head, batch), walking the causal key
// blocks in 64-key sub-blocks k with double-buffered S / dP in TMEM:
//   S_k = Q K_k^T, dP_k = dO V_k^T -> buffer k & 1;  dS_k -> smem buffer k & 1;
//   dQ += dS_k K_k (TMEM accumulator)
constexpr int kDqSmem = 1024 + 2 * kTile /*Q,dO*/ + 2 * kBwdStages * kTile /*K,V*/ + 2 * kTile /*dS x2*/ + 256;

__global__ void __launch_bounds__(kBwdThreads, 1)
dq_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tmo, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* sQ = sm;
  uint8_t* sO = sQ + kTile;
  uint8_t* sK = sO + kTile;
  uint8_t* sV = sK + kBwdStages * kTile;
  uint8_t* sS = sV + kBwdStages * kTile;          // dS [2 buffers] x (128 queries x 64 keys)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sS + 2 * kTile);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;
  uint64_t* kv_empty = kv_full + kBwdStages;
  uint64_t* sdp_full = kv_empty + kBwdStages;     // [2]
  uint64_t* sdp_empty = sdp_full + 2;             // [2]
  uint64_t* ds_full = sdp_empty + 2;              // [2]
  uint64_t* ds_empty = ds_full + 2;               // [2]
  uint64_t* acc_done = ds_empty + 2;
  uint64_t* drain = acc_done + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);

  int rank_x, h, b;
  lpt_coords(rank_x, h, b);
  const int qb = gridDim.x - 1 - rank_x;     // query block qb sees qb + 1 key blocks
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q0 = qb * BM;
  const int tok0 = b * p.S;
  const int n_kv = qb + 1;
  const int n_sub = 2 * n_kv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&sdp_empty[i], kBwdSoft);
      mbar_init(&ds_full[i], kBwdSoft);
      mbar_init(&ds_empty[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t tS0 = tbase, tdP0 = tbase + 128, tdQ = tbase + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      tma_prefetch_desc(&tmo);
      mbar_arrive_expect_tx(q_full, 2 * kTile);
      tma_load_2d(sQ, &tm, q_full, h * D, tok0 + q0);
      tma_load_2d(sO, &tmo, q_full, h * D, tok0 + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % kBwdStages;
        if (!mbar_wait(&kv_empty[st], ((j / kBwdStages) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
        tma_load_2d(sK + st * kTile, &tm, &kv_full[st], (p.Hq + kvh) * D, tok0 + j * BN);
        tma_load_2d(sV + st * kTile, &tm, &kv_full[st], (p.Hq + p.Hkv + kvh) * D, tok0 + j * BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = make_idesc_bf16(BM, 64, 0, 0);   // [queries x 64 keys], K = d
      constexpr uint32_t idG = make_idesc_bf16(BM, D, 0, 1);    // [queries x d], K = 64 keys
      const uint32_t qa = smem_u32(sQ), oa = smem_u32(sO);
      bool ok = mbar_wait(q_full, 0, p.status);
      for (int k = 0; k <= n_sub && ok; ++k) {
        if (k < n_sub) {
          const int j = k >> 1, hh = k & 1, st = j % kBwdStages;
          if (hh == 0 && !mbar_wait(&kv_full[st], (j / kBwdStages) & 1, p.status)) break;
          if (k >= 2 && !mbar_wait(&sdp_empty[k & 1], ((k - 2) >> 1) & 1, p.status)) break;
          tc_fence_after();
          const uint32_t ka = smem_u32(sK + st * kTile) + hh * 8192, va = smem_u32(sV + st * kTile) + hh * 8192;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            umma_f16(tS0 + (k & 1) * 64, kdesc(qa + kk * 32), kdesc(ka + kk * 32), idS, kk > 0);
            umma_f16(tdP0 + (k & 1) * 64, kdesc(oa + kk * 32), kdesc(va + kk * 32), idS, kk > 0);
          }
          umma_commit(&sdp_full[k & 1]);
        }
        if (k >= 1) {
          const int kp = k - 1, j = kp >> 1, hh = kp & 1, st = j % kBwdStages;
          if (!mbar_wait(&ds_full[kp & 1], (kp >> 1) & 1, p.status)) break;
          tc_fence_after();
          const uint32_t ka = smem_u32(sK + st * kTile), da = smem_u32(sS + (kp & 1) * kTile);
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk)
            umma_f16(tdQ, kdesc(da + kk * 32), mndesc(ka + (hh * 4 + kk) * 2048), idG,
                     (kp > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&ds_empty[kp & 1]);
          if (hh == 1) umma_commit(&kv_empty[st]);     // both halves of this K / V stage consumed
        }
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    const int quarter = warp % 4;
    const int part = (warp - 2) / 4;          // columns [16*part, +16) of a 64-key sub-block; of dQ
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const long li = (static_cast<long>(b) * p.Hq + h) * p.S + q;
    const float nlse = -p.lse[li];
    const float del = p.delta[li];
    bool ok = true;
    for (int k = 0; k < n_sub; ++k) {
      const int j = k >> 1, hh = k & 1;
      if (!mbar_wait(&sdp_full[k & 1], (k >> 1) & 1, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t vs[kBwdCols], vd[kBwdCols];
      tmem_ld_32x32b_x16(tS0 + (k & 1) * 64 + part * kBwdCols + lane_off, vs);
      tmem_ld_32x32b_x16(tdP0 + (k & 1) * 64 + part * kBwdCols + lane_off, vd);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sdp_empty[k & 1]);
      float ds[kBwdCols];
#pragma unroll
      for (int t = 0; t < kBwdCols; ++t)
        ds[t] = ex2(fmaf(__uint_as_float(vs[t]), p.scale_log2, nlse)) * (__uint_as_float(vd[t]) - del);
      if (j == qb) {             // causal mask only on the diagonal block
        const int key0 = j * BN + hh * 64 + part * kBwdCols;
#pragma unroll
        for (int t = 0; t < kBwdCols; ++t)
          if (key0 + t > q) ds[t] = 0.f;
      }
      if (k >= 2 && !mbar_wait(&ds_empty[k & 1], ((k - 2) >> 1) & 1, p.status)) {
        ok = false;
        break;
      }
      uint8_t* db = sS + (k & 1) * kTile;
#pragma unroll
      for (int u = 0; u < kBwdCols / 8; ++u) {
        bf16x8 d = float_to_bf16x8(ds + 8 * u);
        *reinterpret_cast<uint4*>(swz_chunk(db, row, part * (kBwdCols / 8) + u)) =
            make_uint4(d.w[0], d.w[1], d.w[2], d.w[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&ds_full[k & 1]);
    }
    if (ok && mbar_wait(acc_done, 0, p.status)) {
      tc_fence_after();
      uint32_t v[kBwdOut];
      __nv_bfloat16* qrow = p.dqkv + static_cast<long>(tok0 + q) * p.dqkv_stride + h * D;
      {
        const int c = part * kBwdOut;
        float f[kBwdOut];
        tmem_ld_32x32b_x16(tdQ + c + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < kBwdOut; ++t) f[t] = __uint_as_float(v[t]) * p.scale;
#pragma unroll
        for (int u = 0; u < kBwdOut / 8; ++u) reinterpret_cast<bf16x8*>(qrow + c)[u] = float_to_bf16x8(f + 8 * u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// delta[b,h,q] = sum_d dO * O
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                             float* __restrict__ delta, int B, int S, int Hq) {
  const long i = static_cast<long>(blockIdx.x) * (blockDim.x / 8) + threadIdx.x / 8;
  const int sub = threadIdx.x % 8;
  const long n = static_cast<long>(B) * S * Hq;
  if (i >= n) return;
  const long tok = i / Hq;
  const int h = static_cast<int>(i % Hq);
  const long off = tok * Hq * D + h * D + sub * 8;
  float a[8], g[8];
  bf16x8_to_float(*reinterpret_cast<const bf16x8*>(o + off), a);
  bf16x8_to_float(*reinterpret_cast<const bf16x8*>(dout + off), g);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += a[j] * g[j];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  if (sub == 0) {
    const long bb = tok / S, q = tok % S;
    delta[(bb * Hq + h) * S + q] = s;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr, "cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// [rows, cols] bf16 row-major with row stride ld; box 64 x 128, 128B swizzle.
static CUtensorMap tile_map(const void* base, int64_t rows, int64_t cols, int64_t ld) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (ld * 2) % 16 == 0, "attention: TMA alignment");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "attention: cuTensorMapEncodeTiled failed ", static_cast<int>(r));
  return m;
}

// dK/dV of a head split: sum the hsplit partials in order, write bf16.
// One thread per (b, key, kv head, 8 values of the 2*D row).
__global__ void dkdv_reduce_kernel(const float* __restrict__ ws, int B, int S, int Hq, int Hkv, int hsplit,
                                   __nv_bfloat16* __restrict__ dqkv, int stride) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long per_row = 2 * D / 8;
  const long total = static_cast<long>(B) * Hkv * S * per_row;
  if (i >= total) return;
  const int c8 = static_cast<int>(i % per_row);
  const long r = i / per_row;                 // (b, kvh, key)
  const int key = static_cast<int>(r % S);
  const int kvh = static_cast<int>((r / S) % Hkv);
  const int b = static_cast<int>(r / (static_cast<long>(S) * Hkv));
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int pt = 0; pt < hsplit; ++pt) {
    const float* src = ws + ((((static_cast<long>(b) * Hkv + kvh) * hsplit + pt) * S) + key) * (2 * D) + c8 * 8;
    const float4 a = reinterpret_cast<const float4*>(src)[0], c = reinterpret_cast<const float4*>(src)[1];
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += c.x; acc[5] += c.y; acc[6] += c.z; acc[7] += c.w;
  }
  const int col = (c8 * 8 < D) ? (Hq + kvh) * D + c8 * 8 : (Hq + Hkv + kvh) * D + (c8 * 8 - D);
  *reinterpret_cast<bf16x8*>(dqkv + (static_cast<long>(b) * S + key) * stride + col) = float_to_bf16x8(acc);
}

static Params base_params(const at::Tensor& qkv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale,
                          const at::Tensor& status) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1, "attention: bf16 qkv");
  TORCH_CHECK(qkv.size(-1) == (Hq + 2 * Hkv) * D, "attention: qkv width must be (Hq + 2 Hkv) * 64");
  TORCH_CHECK(Hq % Hkv == 0, "attention: Hq % Hkv");
  TORCH_CHECK(S % 128 == 0, "attention: sequence length must be a multiple of 128");
  TORCH_CHECK(qkv.numel() / qkv.size(-1) == B * S, "attention: token count");
  Params p{};
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale) * kLog2e;
  p.status = status.data_ptr<int>();
  p.hsplit = 1;
  p.ws = nullptr;
  return p;
}

std::vector<at::Tensor> fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale,
                            const at::Tensor& status) {
  const at::cuda::CUDAGuard guard(qkv.device());
  Params p = base_params(qkv, B, S, Hq, Hkv, scale, status);
  auto o = at::empty({B * S, Hq * D}, qkv.options());
  auto lse = at::empty({B, Hq, S}, qkv.options().dtype(at::kFloat));
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.o_stride = static_cast<int>(Hq * D);
  p.lse = lse.data_ptr<float>();
  CUtensorMap tm = tile_map(qkv.data_ptr(), B * S, qkv.size(-1), qkv.stride(-2));
  static bool cfg = false;
  // SHIFT_ATTN_FWD selects the forward form: unset or "split" (key blocks
  // alternate between the warps of a pair, O in TMEM: 0.188 ms at B 8, S 2048,
  // 16 / 4 heads), "split_fma" (the same with 2 of every 8 exponentials on the
  // FMA pipe), "fold" (the pair shares each key block, O folded into
  // registers: 0.213 ms) or "tmem" (shared block, O in TMEM: 0.225 ms)
  static const int form = [] {
    const char* e = std::getenv("SHIFT_ATTN_FWD");
    const std::string v = e ? e : "split";
    return v == "fold" ? 0 : v == "tmem" ? 1 : v == "split_fma" ? 3 : 2;
  }();
  if (!cfg) {
    cudaFuncSetAttribute(fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
    cudaFuncSetAttribute(fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
    cudaFuncSetAttribute(fwd_split_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmem);
    cudaFuncSetAttribute(fwd_split_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmem);
    cfg = true;
  }
  dim3 grid(static_cast<unsigned>(S / BM), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (form == 2) fwd_split_kernel<0><<<grid, kThreads, kSplitSmem, stream>>>(tm, p);
  else if (form == 3) fwd_split_kernel<2><<<grid, kThreads, kSplitSmem, stream>>>(tm, p);
  else if (form == 1) fwd_kernel<true><<<grid, kThreads, kFwdSmem, stream>>>(tm, p);
  else fwd_kernel<false><<<grid, kThreads, kFwdSmem, stream>>>(tm, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

at::Tensor bwd(const at::Tensor& qkv, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dout, int64_t B,
               int64_t S, int64_t Hq, int64_t Hkv, double scale, const at::Tensor& status) {
  const at::cuda::CUDAGuard guard(qkv.device());
  TORCH_CHECK(dout.is_contiguous() && o.is_contiguous(), "attention bwd: contiguous O / dO");
  Params p = base_params(qkv, B, S, Hq, Hkv, scale, status);
  auto dqkv = at::empty({B * S, (Hq + 2 * Hkv) * D}, qkv.options());
  auto delta = at::empty({B, Hq, S}, qkv.options().dtype(at::kFloat));
  p.lse = const_cast<float*>(lse.data_ptr<float>());
  p.delta = delta.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.dqkv_stride = static_cast<int>(dqkv.stride(-2));
  auto stream = at::cuda::getCurrentCUDAStream();
  const long n = B * S * Hq;
  delta_kernel<<<(n + 31) / 32, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
                                                  reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                                                  delta.data_ptr<float>(), (int)B, (int)S, (int)Hq);
  CUtensorMap tm = tile_map(qkv.data_ptr(), B * S, qkv.size(-1), qkv.stride(-2));
  CUtensorMap tmo = tile_map(dout.data_ptr(), B * S, dout.size(-1), dout.stride(-2));
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDkdvSmem);
    cudaFuncSetAttribute(dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem);
    cfg = true;
  }
  // head split when the dK/dV grid would leave most SMs idle (small batch)
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int group = static_cast<int>(Hq / Hkv);
  const long ctas = (S / BN) * Hkv * B;
  int hs = 1;
  while (hs < group && group % (hs * 2) == 0 && ctas * hs * 2 <= 2L * sms) hs *= 2;
  at::Tensor ws;
  if (hs > 1) {
    ws = at::empty({B * Hkv * hs * S * 2 * D}, qkv.options().dtype(at::kFloat));
    p.hsplit = hs;
    p.ws = ws.data_ptr<float>();
  }
  dim3 g1(static_cast<unsigned>(S / BN), static_cast<unsigned>(Hkv * hs), static_cast<unsigned>(B));
  dkdv_kernel<<<g1, kBwdThreads, kDkdvSmem, stream>>>(tm, tmo, p);
  if (hs > 1) {
    const long total = B * Hkv * S * (2 * D / 8);
    dkdv_reduce_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
        p.ws, (int)B, (int)S, (int)Hq, (int)Hkv, hs, p.dqkv, p.dqkv_stride);
  }
  dim3 g2(static_cast<unsigned>(S / BM), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  dq_kernel<<<g2, kBwdThreads, kDqSmem, stream>>>(tm, tmo, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace fa
}  // namespace sb
