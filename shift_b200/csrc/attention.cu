// Causal flash attention (forward / backward) with grouped-query heads.
//
// Reads q/k/v straight out of the fused QKV projection [T, (Hq + 2*Hkv) * D]
// (no re-layout) and writes O as [T, Hq * D], which is exactly the input of
// the output projection.  head_dim = 64.  Online softmax in base 2; the
// per-row log-sum-exp (base 2) is saved for the backward.
//
// The backward is deterministic: one kernel owns a block of keys and loops
// over every query block (and every query head of its KV group) to build
// dK/dV in registers; a second kernel owns a block of queries and loops over
// key blocks to build dQ.  No atomics.
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) with
// ldmatrix from XOR-swizzled shared memory, cp.async double buffering.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace sb {
namespace attn {

constexpr int D = 64;
constexpr int BQ = 64;     // queries per CTA (4 warps x 16)
constexpr int BKV = 64;    // keys per block
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const __nv_bfloat16* qkv;  // [T, row_stride]
  __nv_bfloat16* o;          // [T, Hq*D]
  float* lse;                // [B, Hq, S] base-2 log-sum-exp
  const __nv_bfloat16* dout; // [T, Hq*D]
  const float* delta;        // [B, Hq, S]
  __nv_bfloat16* dqkv;       // [T, row_stride]
  int B, S, Hq, Hkv, row_stride;
  float scale_log2;          // softmax_scale * log2(e)
  float scale;
};

// ---- smem tile: 64 rows x 64 bf16, 16-byte chunks XOR-swizzled by row ----
SB_DEVICE uint32_t swz(int row, int col) {  // col in elements (multiple of 8)
  return static_cast<uint32_t>(row * 128 + ((((col >> 3) ^ (row & 7))) << 4));
}

SB_DEVICE void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
SB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SB_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Load a 64x64 tile whose row r starts at src + r*stride (elements).
SB_DEVICE void load_tile(uint32_t sbase, const __nv_bfloat16* src, long stride, int rows_valid) {
  for (int i = threadIdx.x; i < 64 * 8; i += kThreads) {
    const int r = i / 8, c = (i % 8) * 8;
    if (r < rows_valid) cp_async16(sbase + swz(r, c), src + r * stride + c);
  }
}

SB_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
SB_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
SB_DEVICE void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragments (16 rows x 64 cols) for the warp's 16 rows starting at row0 of a tile.
SB_DEVICE void load_a_frags(uint32_t sbase, int row0, uint32_t (&a)[4][4]) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int r = row0 + (lane % 8) + 8 * ((lane / 8) % 2);
    const int c = ks * 16 + 8 * (lane / 16);
    ldsm_x4(sbase + swz(r, c), a[ks][0], a[ks][1], a[ks][2], a[ks][3]);
  }
}

// acc[8 n-tiles][4] += A(16x64, regs) * B where B[k][n] = tile[n][k] (tile rows are n).
SB_DEVICE void mma_a_tileT(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t tile) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int np = 0; np < 4; ++np) {      // pairs of n-tiles (16 rows of tile)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int r = np * 16 + (lane % 8) + 8 * (lane / 16);
      const int c = ks * 16 + 8 * ((lane / 8) % 2);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(tile + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * np], a[ks], b0, b1);
      mma16816(acc[2 * np + 1], a[ks], b2, b3);
    }
  }
}

// acc[8 n-tiles over D][4] += P(16 x 64 keys as bf16 A frags) * tile (rows = k, cols = n).
SB_DEVICE void mma_p_tile(float (&acc)[8][4], const uint32_t (&p)[4][4], uint32_t tile) {
  const int lane = threadIdx.x % 32;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int r = ks * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
      const int c = np * 16 + 8 * (lane / 16);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(tile + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * np], p[ks], b0, b1);
      mma16816(acc[2 * np + 1], p[ks], b2, b3);
    }
  }
}

// Convert fp32 accumulators (16 x 64 over 8 n-tiles) into bf16 A fragments (4 k-steps).
SB_DEVICE void acc_to_a(const float (&s)[8][4], uint32_t (&p)[4][4]) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    p[ks][0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
    p[ks][1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
    p[ks][2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
    p[ks][3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
  }
}

SB_DEVICE void zero_acc(float (&a)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) a[i][j] = 0.f;
}

// ============================ forward ============================
__global__ void __launch_bounds__(kThreads)
fwd_kernel(Params p) {
  __shared__ __align__(128) uint8_t smem[5 * 8192];  // Q, K[2], V[2]
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + 8192, sQ + 16384};
  const uint32_t sV[2] = {sQ + 24576, sQ + 32768};
  const long tok0 = static_cast<long>(b) * p.S;
  const int q0 = qb * BQ;
  const __nv_bfloat16* qptr = p.qkv + (tok0 + q0) * p.row_stride + h * D;
  const __nv_bfloat16* kptr = p.qkv + tok0 * p.row_stride + (p.Hq + kvh) * D;
  const __nv_bfloat16* vptr = p.qkv + tok0 * p.row_stride + (p.Hq + p.Hkv + kvh) * D;
  const int rows_q = min(BQ, p.S - q0);
  load_tile(sQ, qptr, p.row_stride, rows_q);
  load_tile(sK[0], kptr, p.row_stride, min(BKV, p.S));
  load_tile(sV[0], vptr, p.row_stride, min(BKV, p.S));
  cp_async_commit();
  const int n_kv = min((q0 + BQ + BKV - 1) / BKV, (p.S + BKV - 1) / BKV);

  uint32_t qa[4][4];
  float o[8][4];
  zero_acc(o);
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int row_a = q0 + warp * 16 + lane / 4;  // query index of c0/c1 rows; +8 for c2/c3

  for (int kb = 0; kb < n_kv; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kv) {
      const int k1 = (kb + 1) * BKV;
      load_tile(sK[buf ^ 1], kptr + static_cast<long>(k1) * p.row_stride, p.row_stride, min(BKV, p.S - k1));
      load_tile(sV[buf ^ 1], vptr + static_cast<long>(k1) * p.row_stride, p.row_stride, min(BKV, p.S - k1));
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) load_a_frags(sQ, warp * 16, qa);
    float s[8][4];
    zero_acc(s);
    mma_a_tileT(s, qa, sK[buf]);
    const int kbase = kb * BKV;
    const bool diag = (kbase + BKV > q0);
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + j * 8 + (lane % 4) * 2 + (e & 1);
        const int q = row_a + (e >> 1) * 8;
        float v = s[j][e] * p.scale_log2;
        if ((diag && key > q) || key >= p.S) v = -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) corr[r] = (m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - mx[r]);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = (mx[e >> 1] == -INFINITY) ? 0.f : exp2f(s[j][e] - mx[e >> 1]);
        s[j][e] = pv;
        rs[e >> 1] += pv;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * corr[r] + rs[r];
      m_r[r] = mx[r];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    uint32_t pa[4][4];
    acc_to_a(s, pa);
    mma_p_tile(o, pa, sV[buf]);
    __syncthreads();
  }
  // epilogue: normalise, write O and LSE
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = row_a + r * 8;
    if (q >= p.S) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    __nv_bfloat16* orow = p.o + (tok0 + q) * (static_cast<long>(p.Hq) * D) + h * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + (lane % 4) * 2;
      *reinterpret_cast<uint32_t*>(orow + c) = pack_bf16x2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
    }
    if (lane % 4 == 0) p.lse[(static_cast<long>(b) * p.Hq + h) * p.S + q] = m_r[r] + log2f(l_r[r]);
  }
}

// delta[b,h,q] = sum_d dO * O
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                             float* __restrict__ delta, int B, int S, int Hq) {
  const long i = static_cast<long>(blockIdx.x) * (blockDim.x / 8) + threadIdx.x / 8;  // (token, head)
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
    const long b = tok / S, q = tok % S;
    delta[(b * Hq + h) * S + q] = s;
  }
}

// ============================ backward: dK, dV ============================
// CTA owns 64 keys of one KV head; warp w owns keys [16w, 16w+16).
__global__ void __launch_bounds__(kThreads)
bwd_dkdv_kernel(Params p) {
  __shared__ __align__(128) uint8_t smem[4 * 8192];   // K, V, Q, dO
  __shared__ float s_lse[BQ], s_delta[BQ];
  const int kb = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t sK = smem_u32(smem), sV = sK + 8192, sQ = sK + 16384, sO = sK + 24576;
  const long tok0 = static_cast<long>(b) * p.S;
  const int k0 = kb * BKV;
  const int rows_k = min(BKV, p.S - k0);
  load_tile(sK, p.qkv + (tok0 + k0) * p.row_stride + (p.Hq + kvh) * D, p.row_stride, rows_k);
  load_tile(sV, p.qkv + (tok0 + k0) * p.row_stride + (p.Hq + p.Hkv + kvh) * D, p.row_stride, rows_k);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t ka[4][4], va[4][4];
  load_a_frags(sK, warp * 16, ka);
  load_a_frags(sV, warp * 16, va);
  float dk[8][4], dv[8][4];
  zero_acc(dk);
  zero_acc(dv);
  const int key_a = k0 + warp * 16 + lane / 4;  // key of c0/c1 rows (+8 for c2/c3)
  const int n_q = (p.S + BQ - 1) / BQ;
  for (int hh = 0; hh < group; ++hh) {
    const int h = kvh * group + hh;
    for (int qb = kb; qb < n_q; ++qb) {  // causal: queries >= keys
      const int q0 = qb * BQ;
      __syncthreads();
      load_tile(sQ, p.qkv + (tok0 + q0) * p.row_stride + h * D, p.row_stride, min(BQ, p.S - q0));
      load_tile(sO, p.dout + (tok0 + q0) * (static_cast<long>(p.Hq) * D) + h * D, static_cast<long>(p.Hq) * D,
                min(BQ, p.S - q0));
      cp_async_commit();
      if (threadIdx.x < BQ) {
        const int q = q0 + threadIdx.x;
        const long idx = (static_cast<long>(b) * p.Hq + h) * p.S + q;
        s_lse[threadIdx.x] = q < p.S ? p.lse[idx] : 0.f;
        s_delta[threadIdx.x] = q < p.S ? p.delta[idx] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      // S^T (keys x queries) = K Q^T
      float st[8][4], dpt[8][4];
      zero_acc(st);
      zero_acc(dpt);
      mma_a_tileT(st, ka, sQ);
      mma_a_tileT(dpt, va, sO);   // dP^T = V dO^T
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = j * 8 + (lane % 4) * 2 + (e & 1);
          const int q = q0 + ql;
          const int key = key_a + (e >> 1) * 8;
          float pv = exp2f(st[j][e] * p.scale_log2 - s_lse[ql]);
          if (key > q || q >= p.S || key >= p.S) pv = 0.f;
          st[j][e] = pv;                                   // P^T
          dpt[j][e] = pv * (dpt[j][e] - s_delta[ql]);       // dS^T
        }
      uint32_t pa[4][4], dsa[4][4];
      acc_to_a(st, pa);
      acc_to_a(dpt, dsa);
      mma_p_tile(dv, pa, sO);   // dV += P^T dO
      mma_p_tile(dk, dsa, sQ);  // dK += dS^T Q
    }
  }
  // write dK (scaled) and dV into the dqkv buffer
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key_a + r * 8;
    if (key >= p.S) continue;
    __nv_bfloat16* krow = p.dqkv + (tok0 + key) * p.row_stride + (p.Hq + kvh) * D;
    __nv_bfloat16* vrow = p.dqkv + (tok0 + key) * p.row_stride + (p.Hq + p.Hkv + kvh) * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + (lane % 4) * 2;
      *reinterpret_cast<uint32_t*>(krow + c) = pack_bf16x2(dk[j][2 * r] * p.scale, dk[j][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(vrow + c) = pack_bf16x2(dv[j][2 * r], dv[j][2 * r + 1]);
    }
  }
}

// ============================ backward: dQ ============================
__global__ void __launch_bounds__(kThreads)
bwd_dq_kernel(Params p) {
  __shared__ __align__(128) uint8_t smem[4 * 8192];   // Q, dO, K, V
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t sQ = smem_u32(smem), sO = sQ + 8192, sK = sQ + 16384, sV = sQ + 24576;
  const long tok0 = static_cast<long>(b) * p.S;
  const int q0 = qb * BQ;
  const int rows_q = min(BQ, p.S - q0);
  load_tile(sQ, p.qkv + (tok0 + q0) * p.row_stride + h * D, p.row_stride, rows_q);
  load_tile(sO, p.dout + (tok0 + q0) * (static_cast<long>(p.Hq) * D) + h * D, static_cast<long>(p.Hq) * D, rows_q);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t qa[4][4], oa[4][4];
  load_a_frags(sQ, warp * 16, qa);
  load_a_frags(sO, warp * 16, oa);
  const int row_a = q0 + warp * 16 + lane / 4;
  float lse[2], dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = row_a + r * 8;
    const long idx = (static_cast<long>(b) * p.Hq + h) * p.S + q;
    lse[r] = q < p.S ? p.lse[idx] : 0.f;
    dl[r] = q < p.S ? p.delta[idx] : 0.f;
  }
  float dq[8][4];
  zero_acc(dq);
  const int n_kv = min((q0 + BQ + BKV - 1) / BKV, (p.S + BKV - 1) / BKV);
  for (int kb = 0; kb < n_kv; ++kb) {
    const int k0 = kb * BKV;
    __syncthreads();
    load_tile(sK, p.qkv + (tok0 + k0) * p.row_stride + (p.Hq + kvh) * D, p.row_stride, min(BKV, p.S - k0));
    load_tile(sV, p.qkv + (tok0 + k0) * p.row_stride + (p.Hq + p.Hkv + kvh) * D, p.row_stride, min(BKV, p.S - k0));
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float s[8][4], dp[8][4];
    zero_acc(s);
    zero_acc(dp);
    mma_a_tileT(s, qa, sK);
    mma_a_tileT(dp, oa, sV);  // dP = dO V^T
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + (lane % 4) * 2 + (e & 1);
        const int q = row_a + (e >> 1) * 8;
        float pv = exp2f(s[j][e] * p.scale_log2 - lse[e >> 1]);
        if (key > q || key >= p.S || q >= p.S) pv = 0.f;
        s[j][e] = pv * (dp[j][e] - dl[e >> 1]);  // dS
      }
    uint32_t dsa[4][4];
    acc_to_a(s, dsa);
    mma_p_tile(dq, dsa, sK);  // dQ += dS K
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = row_a + r * 8;
    if (q >= p.S) continue;
    __nv_bfloat16* row = p.dqkv + (tok0 + q) * p.row_stride + h * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + (lane % 4) * 2;
      *reinterpret_cast<uint32_t*>(row + c) = pack_bf16x2(dq[j][2 * r] * p.scale, dq[j][2 * r + 1] * p.scale);
    }
  }
}

// ---------------------------------------------------------------------------
static Params make_params(const at::Tensor& qkv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1, "attention: bf16 qkv");
  TORCH_CHECK(qkv.size(-1) == (Hq + 2 * Hkv) * D, "attention: qkv width must be (Hq + 2 Hkv) * 64");
  TORCH_CHECK(Hq % Hkv == 0, "attention: Hq % Hkv");
  TORCH_CHECK(S % 64 == 0, "attention: sequence length must be a multiple of 64");
  TORCH_CHECK(qkv.numel() / qkv.size(-1) == B * S, "attention: token count");
  Params p{};
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.row_stride = static_cast<int>(qkv.stride(-2));
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale) * kLog2e;
  return p;
}

// Returns (O [T, Hq*64], LSE [B, Hq, S] base 2).
std::vector<at::Tensor> attn_fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale) {
  const at::cuda::CUDAGuard guard(qkv.device());
  Params p = make_params(qkv, B, S, Hq, Hkv, scale);
  auto o = at::empty({B * S, Hq * D}, qkv.options());
  auto lse = at::empty({B, Hq, S}, qkv.options().dtype(at::kFloat));
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  dim3 grid((S + BQ - 1) / BQ, Hq, B);
  fwd_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

// Returns dqkv [T, (Hq+2Hkv)*64].
at::Tensor attn_bwd(const at::Tensor& qkv, const at::Tensor& o, const at::Tensor& lse, const at::Tensor& dout,
                    int64_t B, int64_t S, int64_t Hq, int64_t Hkv, double scale) {
  const at::cuda::CUDAGuard guard(qkv.device());
  TORCH_CHECK(dout.is_contiguous() && o.is_contiguous(), "attention bwd: contiguous O / dO");
  Params p = make_params(qkv, B, S, Hq, Hkv, scale);
  auto dqkv = at::empty({B * S, (Hq + 2 * Hkv) * D}, qkv.options());
  auto delta = at::empty({B, Hq, S}, qkv.options().dtype(at::kFloat));
  p.lse = const_cast<float*>(lse.data_ptr<float>());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.delta = delta.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.row_stride = static_cast<int>(qkv.stride(-2));
  TORCH_CHECK(dqkv.stride(-2) == p.row_stride, "attention bwd: dqkv stride must match qkv");
  auto stream = at::cuda::getCurrentCUDAStream();
  const long n = B * S * Hq;
  delta_kernel<<<(n + 31) / 32, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), p.dout,
                                                  delta.data_ptr<float>(), (int)B, (int)S, (int)Hq);
  dim3 g1((S + BKV - 1) / BKV, Hkv, B);
  bwd_dkdv_kernel<<<g1, kThreads, 0, stream>>>(p);
  dim3 g2((S + BQ - 1) / BQ, Hq, B);
  bwd_dq_kernel<<<g2, kThreads, 0, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

}  // namespace attn
}  // namespace sb
