// tcgen05 GEMM kernel template (included by the per-tile-width translation
// units gemm_bn*.cu).  Documentation of the kernel is in gemm_sm100.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace sb {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 128;

template <int BN>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;   // 16 KB
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN == 256) ? 4 : (BN == 192 ? 4 : 5);
  static constexpr int kTmemCols = 512;          // two accumulators of <= 256 columns
  // Epilogue staging for TMA stores: per epilogue warp two buffers of 32 rows
  // x 64 bf16 (128 B rows, 128-byte swizzle) and, below BN 256, two SwiGLU
  // activation buffers of 32 rows x 32 bf16 (64 B rows, 64-byte swizzle).
  static constexpr bool kD2Staged = BN != 256;
  static constexpr int kEpiD = 32 * 128;
  static constexpr int kEpiD2 = kD2Staged ? 32 * 64 : 0;
  static constexpr int kEpiWarpBytes = 2 * (kEpiD + kEpiD2);
  static constexpr int kEpiBytes = 4 * kEpiWarpBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 /*align*/ + 256 /*barriers*/ +
                                    2 * (kMaxGroups + 1) * 4;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Params {
  int M, N, K;       // per-group problem: rows(M) x cols(N), contraction K
  int G;
  int mode;          // kRowGroups / kKGroups
  int epi;           // Epilogue
  const int* offs;   // [G+1] segment offsets (device); nullptr => [0, M] / [0, K]
  void* D;
  void* D2;          // second output (SwiGLU activation)
  int ldd, ldd2;
  float alpha;
  int* status;
  // ---- tensor-parallel exchange (all optional; see Xchg in common.cuh) ----
  Xchg xc;           // wait before gathered rows / signal after the last store; peer_out = D_peer
  int wait_lo, wait_hi;   // gathered index range that needs the wait: A rows (row mode) or K rows (k mode)
  int m_rot;         // row mode, G == 1: row-tile order rotated by m_rot tiles
  int peer_lo, peer_hi;   // output rows in [peer_lo, peer_hi) go to xc.peer_out at row - peer_lo
  int d_row_off;     // the other output rows go to D at row - d_row_off
  int use_tma_store; // tmD (and tmD2 for SwiGLU) describe D / D2: bf16 tiles leave through TMA
  int d_rows;        // rows of the tensor tmD describes
};

struct TileInfo {
  int a_x, a_y;      // TMA coordinates of A for k-block 0 (x inner)
  int b_x, b_y;      // TMA coordinates of B for k-block 0
  int out_row0;      // first output row
  int n0;            // first output column
  int m_valid;       // rows of this tile that are real
  int kb;            // number of k-blocks
  int k0;            // first contraction index (k mode)
};

template <int BN, bool A_MN, bool B_MN>
__device__ __forceinline__ bool decode_tile(const Params& p, const int* s_prefix, const int* s_offs, int tile,
                                            TileInfo& t) {
  const int tiles_n = (p.N + BN - 1) / BN;
  if (p.mode == kRowGroups) {
    // find group: s_prefix[g] <= tile < s_prefix[g+1]
    int g = 0;
    while (g + 1 < p.G && s_prefix[g + 1] <= tile) ++g;
    const int local = tile - s_prefix[g];
    int tm = local / tiles_n;
    const int tn = local % tiles_n;
    const int seg0 = s_offs[g], seg1 = s_offs[g + 1];
    if (p.m_rot != 0) {
      const int tiles_m = (seg1 - seg0 + BM - 1) / BM;
      tm = (tm + p.m_rot) % tiles_m;
    }
    const int m0 = seg0 + tm * BM;
    t.out_row0 = m0;
    t.m_valid = min(BM, seg1 - m0);
    t.n0 = tn * BN;
    t.kb = (p.K + BK - 1) / BK;
    t.k0 = 0;
    if (!A_MN) { t.a_x = 0; t.a_y = m0; }
    else       { t.a_x = m0; t.a_y = 0; }
    if (!B_MN) { t.b_x = 0; t.b_y = g * p.N + t.n0; }
    else       { t.b_x = t.n0; t.b_y = g * p.K; }
  } else {
    const int tiles_m = (p.M + BM - 1) / BM;
    const int per = tiles_m * tiles_n;
    const int g = tile / per;
    const int local = tile - g * per;
    const int tm = local / tiles_n, tn = local % tiles_n;
    const int k0 = s_offs[g], k1 = s_offs[g + 1];
    t.out_row0 = g * p.M + tm * BM;
    t.m_valid = min(BM, p.M - tm * BM);
    t.n0 = tn * BN;
    t.kb = (k1 - k0 + BK - 1) / BK;
    t.k0 = k0;
    // A: MN-major [K, M] -> x = m, y = k ; K-major [M, K] -> x = k, y = m (not used for k-groups)
    if (A_MN) { t.a_x = tm * BM; t.a_y = k0; }
    else      { t.a_x = k0; t.a_y = g * p.M + tm * BM; }
    if (B_MN) { t.b_x = t.n0; t.b_y = k0; }
    else      { t.b_x = k0; t.b_y = g * p.N + t.n0; }
  }
  return true;
}

// x * sigmoid(x) with the fast reciprocal-based division (the epilogue is
// issue-bound; an IEEE division per activation dominated it)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD2, Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* tiles = smem;
  uint8_t* epi_stage = smem + C::kStages * C::kStageBytes;   // 1024-aligned (stage sizes are)
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + C::kEpiBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tmem_full = empty + C::kStages;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* s_offs = reinterpret_cast<int*>(tmem_base_slot + 4);
  int* s_prefix = s_offs + (kMaxGroups + 1);  // lives in the extra tail
  __shared__ int s_total_tiles;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // ---- set-up: segment table and tile prefix -------------------------------
  if (threadIdx.x == 0) {
    const int tiles_n = (p.N + BN - 1) / BN;
    int total = 0;
    for (int g = 0; g <= p.G; ++g) {
      int o;
      if (p.offs) o = p.offs[g];
      else o = (g == 0) ? 0 : (p.mode == kRowGroups ? p.M : p.K);
      s_offs[g] = o;
    }
    if (p.mode == kRowGroups) {
      for (int g = 0; g < p.G; ++g) {
        s_prefix[g] = total;
        const int rows = max(0, s_offs[g + 1] - s_offs[g]);
        total += ((rows + BM - 1) / BM) * tiles_n;
      }
      s_prefix[p.G] = total;
    } else {
      const int tiles_m = (p.M + BM - 1) / BM;
      total = p.G * tiles_m * tiles_n;
    }
    s_total_tiles = total;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int total_tiles = s_total_tiles;

  if (warp == 0) {
    // ===================== TMA producer =====================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool waited = (p.xc.wait_flag == nullptr);
      // Gathered operand rows written by the TP peer: wait (bounded) for its
      // flag before the first TMA load that reads them, then order the
      // async-proxy loads after the acquire.
      auto peer_wait = [&](int lo, int hi) -> bool {
        if (waited || hi <= p.wait_lo || lo >= p.wait_hi) return true;
        if (!wait_flag_ge(p.xc.wait_flag, p.xc.sdev[0] + p.xc.wait_delta, p.status, kPeerWaitNs)) return false;
        asm volatile("fence.proxy.async.global;" ::: "memory");
        waited = true;
        return true;
      };
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        TileInfo t;
        decode_tile<BN, A_MN, B_MN>(p, s_prefix, s_offs, tile, t);
        if (p.mode == kRowGroups && !peer_wait(t.out_row0, t.out_row0 + BM)) { ok = false; break; }
        for (int kb = 0; kb < t.kb; ++kb) {
          if (p.mode == kKGroups && !peer_wait(t.k0 + kb * BK, t.k0 + (kb + 1) * BK)) { ok = false; break; }
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status)) { ok = false; break; }
          uint8_t* sA = tiles + stage * C::kStageBytes;
          uint8_t* sB = sA + C::kABytes;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], t.a_x + kb * BK, t.a_y);
          } else {
            tma_load_2d(sA, &tmA, &full[stage], t.a_x, t.a_y + kb * BK);
            tma_load_2d(sA + 8192, &tmA, &full[stage], t.a_x + 64, t.a_y + kb * BK);
          }
          if (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], t.b_x + kb * BK, t.b_y);
          } else {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h)
              tma_load_2d(sB + h * 8192, &tmB, &full[stage], t.b_x + h * 64, t.b_y + kb * BK);
          }
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Drain: wait (briefly) for every stage's outstanding load so that no
        // TMA write lands after the CTA exits.
        for (int s = 0; s < C::kStages; ++s) mbar_wait(&full[s], phase ^ (s < stage ? 0 : 1), nullptr, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ===================== MMA issuer =====================
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        TileInfo t;
        decode_tile<BN, A_MN, B_MN>(p, s_prefix, s_offs, tile, t);
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < t.kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + stage * C::kStageBytes);
          const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t ad, bd;
            if (!A_MN) ad = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            else       ad = make_sw128_desc(a_addr + kk * 2048, 8192, 1024);
            if (!B_MN) bd = make_sw128_desc(b_addr + kk * 32, 16, 1024);
            else       bd = make_sw128_desc(b_addr + kk * 2048, 8192, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Make sure every MMA this thread issued has completed before TMEM is freed.
      umma_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    // ===================== epilogue =====================
    const int quarter = warp % 4;              // TMEM lanes [32*quarter, 32*quarter+32)
    const int r = quarter * 32 + lane;         // row within tile
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t epi_slab = 0;                     // staging double-buffer counter (TMA-store path)
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      TileInfo t;
      decode_tile<BN, A_MN, B_MN>(p, s_prefix, s_offs, tile, t);
      if (!mbar_wait(&tmem_full[acc], acc_phase, p.status)) break;
      tc_fence_after();
      // ---- TMA-store path: bf16 / SwiGLU outputs of local destinations.  The
      // tile's accumulator slab (32 rows x 64 columns per warp) is converted
      // and written to swizzled shared memory, then one lane stores it with
      // TMA: whole 128-byte row segments instead of one row per thread.
      // Tiles owned by the tensor-parallel peer take the same staging but
      // leave through coalesced SM stores into the peer's receive buffer
      // (whole 512-byte row runs per warp instruction, over NVLink).
      const bool tile_to_peer = p.xc.peer_out != nullptr && t.out_row0 >= p.peer_lo && t.out_row0 < p.peer_hi;
      const bool tma_ok = t.kb > 0 &&
                          ((p.use_tma_store && !tile_to_peer &&
                            (t.m_valid == BM || t.out_row0 - p.d_row_off + t.m_valid >= p.d_rows) &&
                            (p.epi == kEpiBF16 || (p.epi == kEpiSwiGLU && C::kD2Staged))) ||
                           (tile_to_peer && p.epi == kEpiBF16 && (p.ldd % 8) == 0));
      if (tma_ok) {
        const int drow0 = tile_to_peer ? t.out_row0 - p.peer_lo + quarter * 32
                                       : t.out_row0 - p.d_row_off + quarter * 32;
        const int rows_here = min(32, t.m_valid - quarter * 32);
        uint8_t* wbuf = epi_stage + (warp - 2) * C::kEpiWarpBytes;
        const int nslabs = min(BN, p.N - t.n0 + 63) / 64;
#pragma unroll 1
        for (int sb = 0; sb < nslabs; ++sb) {
          const int c = sb * 64;
          uint32_t v[64];
          tmem_ld_32x32b_x32(tmem_base + acc * BN + c + ((quarter * 32) << 16), v);
          tmem_ld_32x32b_x32(tmem_base + acc * BN + c + 32 + ((quarter * 32) << 16), v + 32);
          tmem_wait_ld();
          if (sb == nslabs - 1) {        // accumulator fully read: hand it back to the MMA warp
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
          }
          uint8_t* bd = wbuf + (epi_slab & 1) * (C::kEpiD + C::kEpiD2);
          uint8_t* bd2 = bd + C::kEpiD;
          ++epi_slab;
          if (lane == 0) bulk_wait_group_read<1>();   // this buffer's previous store has read it
          __syncwarp();
          float f[64];
#pragma unroll
          for (int i = 0; i < 64; ++i) f[i] = __uint_as_float(v[i]) * p.alpha;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<bf16x8*>(bd + lane * 128 + ((j ^ (lane & 7)) * 16)) = float_to_bf16x8(f + 8 * j);
          if (C::kD2Staged && p.epi == kEpiSwiGLU) {
            // columns [c, c+64) = (16 gate, 16 up) x 2 -> 32 activations
            float a[32];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float g = __bfloat162float(__float2bfloat16(f[32 * h + i]));
                const float u = __bfloat162float(__float2bfloat16(f[32 * h + 16 + i]));
                a[16 * h + i] = silu_f(g) * u;
              }
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<bf16x8*>(bd2 + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) = float_to_bf16x8(a + 8 * j);
          }
          if (tile_to_peer) {
            __syncwarp();
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.xc.peer_out);
            const int col_lim = p.N - (t.n0 + c);
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int ch = it * 32 + lane;        // 16-byte chunk of the warp's 32 x 128 B slab
              const int rr = ch >> 3, j = ch & 7;
              if (rr < rows_here && j * 8 < col_lim)
                *reinterpret_cast<uint4*>(dst + static_cast<long>(drow0 + rr) * p.ldd + t.n0 + c + j * 8) =
                    *reinterpret_cast<const uint4*>(bd + rr * 128 + ((j ^ (rr & 7)) * 16));
            }
            __syncwarp();
            continue;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmD, bd, t.n0 + c, drow0);
            if (C::kD2Staged && p.epi == kEpiSwiGLU) tma_store_2d(&tmD2, bd2, (t.n0 + c) / 2, drow0);
            bulk_commit_group();
          }
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        continue;
      }
      const bool row_ok = r < t.m_valid;
      const long grow = static_cast<long>(t.out_row0) + r;
      // destination: the TP peer's receive buffer for its rows, D otherwise
      const bool to_peer = p.xc.peer_out != nullptr && grow >= p.peer_lo && grow < p.peer_hi;
      void* const Dst = to_peer ? p.xc.peer_out : p.D;
      const long row = to_peer ? grow - p.peer_lo : grow - p.d_row_off;
      const bool empty_k = (t.kb == 0);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + acc * BN + c + ((quarter * 32) << 16), v);
        tmem_wait_ld();
        const int col = t.n0 + c;
        if (!row_ok || col >= p.N) continue;
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = empty_k ? 0.0f : __uint_as_float(v[i]) * p.alpha;
        const int ncols = min(32, p.N - col);  // N is a multiple of 32 for all callers except tails
        switch (p.epi) {
          case kEpiBF16: {
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(Dst) + row * p.ldd + col;
            if (ncols == 32) {
#pragma unroll
              for (int q = 0; q < 4; ++q) reinterpret_cast<bf16x8*>(out)[q] = float_to_bf16x8(f + 8 * q);
            } else {
              for (int i = 0; i < ncols; ++i) out[i] = __float2bfloat16(f[i]);
            }
          } break;
          case kEpiF32: {
            float* out = reinterpret_cast<float*>(Dst) + row * p.ldd + col;
            if (ncols == 32) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                reinterpret_cast<float4*>(out)[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
            } else {
              for (int i = 0; i < ncols; ++i) out[i] = f[i];
            }
          } break;
          case kEpiAccBF16: {
            if (empty_k) break;
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(Dst) + row * p.ldd + col;
            if (ncols == 32) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                float old[8];
                bf16x8_to_float(reinterpret_cast<bf16x8*>(out)[q], old);
#pragma unroll
                for (int i = 0; i < 8; ++i) old[i] += f[8 * q + i];
                reinterpret_cast<bf16x8*>(out)[q] = float_to_bf16x8(old);
              }
            } else {
              for (int i = 0; i < ncols; ++i) out[i] = __float2bfloat16(__bfloat162float(out[i]) + f[i]);
            }
          } break;
          case kEpiAccF32: {
            if (empty_k) break;
            float* out = reinterpret_cast<float*>(Dst) + row * p.ldd + col;
            if (ncols == 32) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 o = reinterpret_cast<float4*>(out)[q];
                o.x += f[4 * q]; o.y += f[4 * q + 1]; o.z += f[4 * q + 2]; o.w += f[4 * q + 3];
                reinterpret_cast<float4*>(out)[q] = o;
              }
            } else {
              for (int i = 0; i < ncols; ++i) out[i] += f[i];
            }
          } break;
          case kEpiSwiGLU: {
            // columns [col, col+32) hold 16 gate then 16 up values of features col/2 .. col/2+15
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(Dst) + row * p.ldd + col;
#pragma unroll
            for (int q = 0; q < 4; ++q) reinterpret_cast<bf16x8*>(out)[q] = float_to_bf16x8(f + 8 * q);
            float a[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              // activation is computed from the bf16-rounded pre-activations so that
              // the backward (which re-reads them) sees exactly the same values
              const float g = __bfloat162float(__float2bfloat16(f[i]));
              const float u = __bfloat162float(__float2bfloat16(f[16 + i]));
              a[i] = silu_f(g) * u;
            }
            __nv_bfloat16* out2 = reinterpret_cast<__nv_bfloat16*>(p.D2) + grow * p.ldd2 + col / 2;
            reinterpret_cast<bf16x8*>(out2)[0] = float_to_bf16x8(a);
            reinterpret_cast<bf16x8*>(out2)[1] = float_to_bf16x8(a + 8);
          } break;
          case kEpiSwiGLUBwd: {
            // accumulator columns [col, col+32) = d(activation) of features col..col+31,
            // i.e. h / dh columns [2 col, 2 col + 64): two 16-feature groups of
            // (16 gate, 16 up)
            const __nv_bfloat16* hrow = reinterpret_cast<const __nv_bfloat16*>(p.D2) + row * p.ldd2 + 2 * col;
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(Dst) + row * p.ldd + 2 * col;
#pragma unroll
            for (int gq = 0; gq < 2; ++gq) {
              float g[16], u[16], dg[16], du[16];
              bf16x8_to_float(reinterpret_cast<const bf16x8*>(hrow + 32 * gq)[0], g);
              bf16x8_to_float(reinterpret_cast<const bf16x8*>(hrow + 32 * gq)[1], g + 8);
              bf16x8_to_float(reinterpret_cast<const bf16x8*>(hrow + 32 * gq)[2], u);
              bf16x8_to_float(reinterpret_cast<const bf16x8*>(hrow + 32 * gq)[3], u + 8);
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float d = f[16 * gq + q];
                const float sg = __fdividef(1.f, 1.f + __expf(-g[q]));
                du[q] = d * g[q] * sg;
                dg[q] = d * u[q] * sg * (1.f + g[q] * (1.f - sg));
              }
              bf16x8* o = reinterpret_cast<bf16x8*>(out + 32 * gq);
              o[0] = float_to_bf16x8(dg);
              o[1] = float_to_bf16x8(dg + 8);
              o[2] = float_to_bf16x8(du);
              o[3] = float_to_bf16x8(du + 8);
            }
          } break;
          default: break;
        }
      }
      tc_fence_before();
      mbar_arrive(&tmem_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // every TMA store of this warp has written global memory before the CTA
    // finishes (and before a tensor-parallel signal)
    if (lane == 0) {
      bulk_wait_group<0>();
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
  xchg_signal(p.xc);
}


int num_sms();

template <int BN, bool A_MN, bool B_MN>
inline void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& td2,
                   const Params& p, int total_tiles_hint, cudaStream_t stream) {
  using C = Cfg<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    configured = true;
  }
  int grid = std::min(num_sms(), std::max(1, total_tiles_hint));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(ta, tb, td, td2, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace gemm
}  // namespace sb
