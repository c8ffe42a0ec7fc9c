// MoE routing, stable bucket sort, token permutation and combine for sm_100a.
//
// Router: one warp per token computes the E router logits (router weight held
// in shared memory), softmax in fp32, deterministic top-k (ties go to the
// lower expert index) and renormalised weights.
//
// Bucket sort: a stable counting sort of integer keys into bins, built from
// per-chunk ranks so that every output position is a pure function of the
// input (no atomics decide order).  It serves both the expert permutation
// (bins = experts, segments padded to the GEMM tile) and the embedding
// gradient (bins = vocabulary ids).
//
// Parity: the reference's model uses FLASH's patch_moe dispatcher around HF
// Qwen2-MoE experts (shift_full/train.py:214, gate at :233-247).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "xchg.h"

namespace sb {
namespace moe {

constexpr int kChunk = 256;

// ---------------------------------------------------------------------------
// Router: logits = x @ Wr^T, probs = softmax(logits), top-k, renormalise.
// ---------------------------------------------------------------------------
template <int NV, int E>
__global__ void __launch_bounds__(256)
router_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ wr, int T, int k,
              int normalize, float* __restrict__ probs, int* __restrict__ topk_idx, float* __restrict__ topk_w) {
  constexpr int H = NV * 256;
  extern __shared__ uint8_t smem[];
  bf16x8* sw = reinterpret_cast<bf16x8*>(smem);  // [E][H/8]
  for (int i = threadIdx.x; i < E * H / 8; i += blockDim.x) sw[i] = reinterpret_cast<const bf16x8*>(wr)[i];
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  // the next token's row is loaded while this one is computed
  bf16x8 xn[NV];
  if (warp < T) {
#pragma unroll
    for (int i = 0; i < NV; ++i) xn[i] = reinterpret_cast<const bf16x8*>(x + static_cast<long>(warp) * H)[i * 32 + lane];
  }
  for (int t = warp; t < T; t += nwarps) {
    float xv[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) bf16x8_to_float(xn[i], xv[i]);
    if (t + nwarps < T) {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        xn[i] = reinterpret_cast<const bf16x8*>(x + static_cast<long>(t + nwarps) * H)[i * 32 + lane];
    }
    float logit[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float wv[8];
        bf16x8_to_float(sw[e * (H / 8) + i * 32 + lane], wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc += xv[i][j] * wv[j];
      }
      logit[e] = warp_sum(acc);
    }
    float mx = logit[0];
#pragma unroll
    for (int e = 1; e < E; ++e) mx = fmaxf(mx, logit[e]);
    float p[E], s = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      p[e] = __expf(logit[e] - mx);
      s += p[e];
    }
    const float inv = 1.f / s;
#pragma unroll
    for (int e = 0; e < E; ++e) p[e] *= inv;
    // lane e < E holds p[e] and its rank: the number of experts before it in
    // the order (larger probability first, lower index on ties); the top k are
    // the lanes of rank < k, and lane j < k writes the pick of rank j.
    float mine = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) if (e == lane) mine = p[e];
    int rank = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) rank += (p[e] > mine || (p[e] == mine && e < lane)) ? 1 : 0;
    if (lane < E) probs[static_cast<long>(t) * E + lane] = mine;
    // picks in rank order, and their sum in that order in every lane
    float wsum = 0.f, my_sel = 0.f;
    int my_idx = 0;
    for (int j = 0; j < k; ++j) {
      const unsigned m = __ballot_sync(0xffffffffu, lane < E && rank == j);
      const int src = __ffs(m) - 1;
      const float v = __shfl_sync(0xffffffffu, mine, src);
      wsum += v;
      if (lane == j) {
        my_sel = v;
        my_idx = src;
      }
    }
    const float norm = normalize ? 1.f / wsum : 1.f;
    if (lane < k) {
      topk_idx[static_cast<long>(t) * k + lane] = my_idx;
      topk_w[static_cast<long>(t) * k + lane] = my_sel * norm;
    }
  }
}

std::vector<at::Tensor> router_fwd(const at::Tensor& x, const at::Tensor& wr, int64_t k, bool normalize) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && wr.scalar_type() == at::kBFloat16, "router: bf16");
  TORCH_CHECK(x.is_contiguous() && wr.is_contiguous(), "router: contiguous");
  const at::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(x.size(-1));
  const int T = static_cast<int>(x.numel() / H);
  const int E = static_cast<int>(wr.size(0));
  TORCH_CHECK(k >= 1 && k <= E && k <= 16, "router: bad k");
  auto probs = at::empty({T, E}, x.options().dtype(at::kFloat));
  auto idx = at::empty({T, k}, x.options().dtype(at::kInt));
  auto w = at::empty({T, k}, x.options().dtype(at::kFloat));
  const int smem = E * H * 2;
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = std::max(1, std::min((T + 7) / 8, sms * 2));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(wr.data_ptr());
#define SB_R(NV, EV)                                                                                     \
  {                                                                                                      \
    auto kern = router_kernel<NV, EV>;                                                                   \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                      \
    kern<<<blocks, 256, smem, stream>>>(xp, wp, T, (int)k, normalize ? 1 : 0, probs.data_ptr<float>(),  \
                                        idx.data_ptr<int>(), w.data_ptr<float>());                       \
  }
  if (H == 1024 && E == 16) SB_R(4, 16)
  else if (H == 1024 && E == 8) SB_R(4, 8)
  else if (H == 256 && E == 8) SB_R(1, 8)
  else if (H == 256 && E == 16) SB_R(1, 16)
  else if (H == 512 && E == 8) SB_R(2, 8)
  else TORCH_CHECK(false, "router: unsupported (H, E)");
#undef SB_R
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {probs, idx, w};
}

// d_logits from d(topk weights) and the auxiliary-loss gradient on probs.
//   dprob[sel] = (dw_j - sum_l dw_l * w_l) / S  (renormalised) or dw_j
//   dprob[e]  += aux_coef_e     (per-expert constant: coef * E * f_e / T)
//   dlogit     = p * (dprob - sum(p * dprob))
__global__ void router_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ topk_idx,
                                  const float* __restrict__ topk_w, const float* __restrict__ d_topk_w,
                                  const float* __restrict__ aux_grad, int T, int E, int k, int normalize,
                                  float* __restrict__ d_logits) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float dp[32];
  float p[32];
  for (int e = 0; e < E; ++e) {
    p[e] = probs[static_cast<long>(t) * E + e];
    dp[e] = aux_grad ? aux_grad[e] : 0.f;
  }
  float S = 0.f, dot = 0.f;
  for (int j = 0; j < k; ++j) {
    S += p[topk_idx[static_cast<long>(t) * k + j]];
    dot += d_topk_w[static_cast<long>(t) * k + j] * topk_w[static_cast<long>(t) * k + j];
  }
  for (int j = 0; j < k; ++j) {
    const int e = topk_idx[static_cast<long>(t) * k + j];
    const float dw = d_topk_w[static_cast<long>(t) * k + j];
    dp[e] += normalize ? (dw - dot) / S : dw;
  }
  float sdot = 0.f;
  for (int e = 0; e < E; ++e) sdot += p[e] * dp[e];
  for (int e = 0; e < E; ++e) d_logits[static_cast<long>(t) * E + e] = p[e] * (dp[e] - sdot);
}

at::Tensor router_bwd(const at::Tensor& probs, const at::Tensor& topk_idx, const at::Tensor& topk_w,
                      const at::Tensor& d_topk_w, const c10::optional<at::Tensor>& aux_grad, bool normalize) {
  const at::cuda::CUDAGuard guard(probs.device());
  const int T = static_cast<int>(probs.size(0)), E = static_cast<int>(probs.size(1));
  const int k = static_cast<int>(topk_idx.size(1));
  TORCH_CHECK(E <= 32, "router_bwd: E <= 32");
  auto dl = at::empty_like(probs);
  router_bwd_kernel<<<(T + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      probs.data_ptr<float>(), topk_idx.data_ptr<int>(), topk_w.data_ptr<float>(), d_topk_w.data_ptr<float>(),
      aux_grad.has_value() ? aux_grad->data_ptr<float>() : nullptr, T, E, k, normalize ? 1 : 0,
      dl.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dl;
}

// dx[t] += dlogits[t] @ Wr  (one warp per token, Wr staged in shared memory).
template <int NV, int E>
__global__ void __launch_bounds__(256)
router_dgrad_kernel(const __nv_bfloat16* __restrict__ wr, const float* __restrict__ dlogits,
                    __nv_bfloat16* __restrict__ dx, int T, int peer_lo, int peer_hi, Xchg xc) {
  // Rows in [peer_lo, peer_hi) are finished partial sums that belong to the
  // tensor-parallel peer: they are stored into its receive buffer
  // (xc.peer_out, row t - peer_lo) instead of dx -- the reduce-scatter's
  // transfer fused into the last kernel that writes them.
  constexpr int H = NV * 256;
  __nv_bfloat16* dpeer = reinterpret_cast<__nv_bfloat16*>(xc.peer_out);
  extern __shared__ uint8_t smem[];
  bf16x8* sw = reinterpret_cast<bf16x8*>(smem);
  for (int i = threadIdx.x; i < E * H / 8; i += blockDim.x) sw[i] = reinterpret_cast<const bf16x8*>(wr)[i];
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  // the next token's dx row and dlogits are loaded while this one is computed
  bf16x8 dn[NV];
  float dl_next = 0.f;
  if (warp < T) {
#pragma unroll
    for (int i = 0; i < NV; ++i) dn[i] = reinterpret_cast<const bf16x8*>(dx + static_cast<long>(warp) * H)[i * 32 + lane];
    dl_next = lane < E ? dlogits[static_cast<long>(warp) * E + lane] : 0.f;
  }
  for (int t = warp; t < T; t += nwarps) {
    float dxv[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) bf16x8_to_float(dn[i], dxv[i]);
    const float my_dl = dl_next;
    if (t + nwarps < T) {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        dn[i] = reinterpret_cast<const bf16x8*>(dx + static_cast<long>(t + nwarps) * H)[i * 32 + lane];
      dl_next = lane < E ? dlogits[static_cast<long>(t + nwarps) * E + lane] : 0.f;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float dl = __shfl_sync(0xffffffffu, my_dl, e);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float wv[8];
        bf16x8_to_float(sw[e * (H / 8) + i * 32 + lane], wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) dxv[i][j] += dl * wv[j];
      }
    }
    __nv_bfloat16* dst = (dpeer != nullptr && t >= peer_lo && t < peer_hi)
                             ? dpeer + static_cast<long>(t - peer_lo) * H
                             : dx + static_cast<long>(t) * H;
#pragma unroll
    for (int i = 0; i < NV; ++i) reinterpret_cast<bf16x8*>(dst)[i * 32 + lane] = float_to_bf16x8(dxv[i]);
  }
  xchg_signal(xc);
}

// partial[c, e*H + h] = sum_{t in chunk c} dlogits[t, e] * x[t, h]; one block per
// chunk of kWgChunk tokens, each thread owns 4 columns.
constexpr int kWgChunk = 128;
template <int E>
__global__ void __launch_bounds__(256)
router_wgrad_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ dlogits, int T, int H,
                    float* __restrict__ partial, int chunk) {
  __shared__ float sdl[kWgChunk][E];
  const int t0 = blockIdx.x * chunk;
  const int nt = min(chunk, T - t0);
  for (int i = threadIdx.x; i < chunk * E; i += blockDim.x) {
    const int tt = i / E, e = i % E;
    sdl[tt][e] = tt < nt ? dlogits[static_cast<long>(t0 + tt) * E + e] : 0.f;
  }
  __syncthreads();
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float acc[E][4];
#pragma unroll
    for (int e = 0; e < E; ++e)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[e][q] = 0.f;
    // eight tokens' loads in flight at a time (the accumulation order over
    // tokens is unchanged)
    constexpr int U = 8;
    for (int tb = 0; tb < nt; tb += U) {
      uint2 raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        raw[u] = tb + u < nt ? *reinterpret_cast<const uint2*>(x + static_cast<long>(t0 + tb + u) * H + h)
                             : make_uint2(0u, 0u);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (tb + u >= nt) break;
        const float2 a = unpack_bf16x2(raw[u].x), b = unpack_bf16x2(raw[u].y);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float dl = sdl[tb + u][e];
          acc[e][0] += dl * a.x;
          acc[e][1] += dl * a.y;
          acc[e][2] += dl * b.x;
          acc[e][3] += dl * b.y;
        }
      }
    }
    float* out = partial + static_cast<long>(blockIdx.x) * E * H;
#pragma unroll
    for (int e = 0; e < E; ++e)
      *reinterpret_cast<float4*>(out + e * H + h) = make_float4(acc[e][0], acc[e][1], acc[e][2], acc[e][3]);
  }
}

// In place: dx += dlogits @ Wr ; returns partial [nchunks, E*H] for a column reduction into dWr.
at::Tensor router_input_weight_grad(const at::Tensor& x, const at::Tensor& wr, const at::Tensor& dlogits,
                                    at::Tensor& dx, const std::vector<int64_t>& peer_rows,
                                    const std::vector<int64_t>& xchg) {
  const Xchg xc = xchg_from(xchg);
  const int peer_lo = peer_rows.size() == 2 ? static_cast<int>(peer_rows[0]) : 0;
  const int peer_hi = peer_rows.size() == 2 ? static_cast<int>(peer_rows[1]) : 0;
  const at::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(x.size(-1));
  const int T = static_cast<int>(x.numel() / H);
  const int E = static_cast<int>(wr.size(0));
  TORCH_CHECK(H % 1024 == 0 || H == 256 || H == 512, "router grad: H");
  // token chunk per block: enough blocks to fill the GPU at small T, few
  // enough partial rows for the column reduction at large T
  const int chunk = std::max(16, std::min(kWgChunk, T / 256));
  const int nchunks = std::max(1, (T + chunk - 1) / chunk);
  auto partial = at::empty({nchunks, E * H}, x.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(wr.data_ptr());
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const int smem = E * H * 2;
  const int blocks = std::max(1, std::min((T + 7) / 8, 148 * 2));
#define SB_R(NV, EV)                                                                                 \
  {                                                                                                  \
    auto kern = router_dgrad_kernel<NV, EV>;                                                         \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                  \
    kern<<<blocks, 256, smem, stream>>>(wp, dlogits.data_ptr<float>(), dxp, T, peer_lo, peer_hi, xc); \
    if (T > 0) router_wgrad_kernel<EV><<<nchunks, 256, 0, stream>>>(xp, dlogits.data_ptr<float>(), T, H, partial.data_ptr<float>(), chunk); \
  }
  if (H == 1024 && E == 16) SB_R(4, 16)
  else if (H == 1024 && E == 8) SB_R(4, 8)
  else if (H == 256 && E == 8) SB_R(1, 8)
  else if (H == 256 && E == 16) SB_R(1, 16)
  else if (H == 512 && E == 8) SB_R(2, 8)
  else TORCH_CHECK(false, "router_input_weight_grad: unsupported (H, E)");
#undef SB_R
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return partial;
}

// ---------------------------------------------------------------------------
// Stable bucket sort.
//   keys[n] in [0, nbins) (keys outside [lo, hi) are ignored: pos = -1)
//   pass 1: rank within chunk (number of earlier equal keys in the chunk);
//           the last occurrence writes the chunk count.
//   pass 2: per bin, exclusive scan over chunks; bin totals.
//   pass 3: bin offsets (exclusive scan of padded totals), single block.
//   pass 4: pos = bin_off[key] + chunk_off[chunk][key] + rank.
// ---------------------------------------------------------------------------
__global__ void sort_rank_kernel(const int* __restrict__ keys, int n, int lo, int hi, int* __restrict__ rank,
                                 int* __restrict__ chunk_counts, int nbins) {
  __shared__ int sk[kChunk];
  const int c = blockIdx.x;
  const int i = c * kChunk + threadIdx.x;
  int key = -1;
  if (i < n) {
    key = keys[i];
    if (key < lo || key >= hi) key = -1;
    else key -= lo;
  }
  sk[threadIdx.x] = key;
  __syncthreads();
  if (i >= n || key < 0) {
    if (i < n) rank[i] = -1;
    return;
  }
  int r = 0;
  bool last = true;
  for (int j = 0; j < kChunk; ++j) {
    const int kj = sk[j];
    if (kj == key) {
      if (j < static_cast<int>(threadIdx.x)) ++r;
      else if (j > static_cast<int>(threadIdx.x)) last = false;
    }
  }
  rank[i] = r;
  if (last) chunk_counts[static_cast<long>(c) * nbins + key] = r + 1;
}

// One CTA per bin: exclusive scan of the bin's column of chunk counts, in
// tiles of 256 chunks (warp shuffles + 8 warp totals), carried across tiles.
__global__ void __launch_bounds__(256)
sort_chunk_scan_kernel(int* __restrict__ chunk_counts, int nchunks, int nbins, int* __restrict__ bin_totals) {
  __shared__ int warp_tot[8];
  const int b = blockIdx.x;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int carry = 0;
  for (int base = 0; base < nchunks; base += 256) {
    const int c = base + threadIdx.x;
    const long o = static_cast<long>(c) * nbins + b;
    const int v = c < nchunks ? chunk_counts[o] : 0;
    int x = v;   // inclusive scan within the warp
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    int before = 0, tile = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const int t = warp_tot[w];
      if (w < warp) before += t;
      tile += t;
    }
    if (c < nchunks) chunk_counts[o] = carry + before + x - v;
    carry += tile;
    __syncthreads();   // warp_tot is rewritten by the next tile
  }
  if (threadIdx.x == 0) bin_totals[b] = carry;
}

// Single block exclusive scan of padded bin totals -> offs[nbins+1].
// Also records the padded total in offs[nbins].
__global__ void sort_bin_scan_kernel(const int* __restrict__ bin_totals, int nbins, int pad,
                                     int* __restrict__ offs, int* __restrict__ counts_out) {
  __shared__ int part[1024];
  const int per = (nbins + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int s = 0;
  for (int b = b0; b < min(nbins, b0 + per); ++b) {
    int v = bin_totals[b];
    if (counts_out) counts_out[b] = v;
    if (pad > 1) v = (v + pad - 1) / pad * pad;
    s += v;
  }
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < static_cast<int>(blockDim.x); ++i) {
      const int v = part[i];
      part[i] = run;
      run += v;
    }
    offs[nbins] = run;
  }
  __syncthreads();
  int run = part[threadIdx.x];
  for (int b = b0; b < min(nbins, b0 + per); ++b) {
    offs[b] = run;
    int v = bin_totals[b];
    if (pad > 1) v = (v + pad - 1) / pad * pad;
    run += v;
  }
}

__global__ void sort_pos_kernel(const int* __restrict__ keys, int n, int lo, const int* __restrict__ rank,
                                const int* __restrict__ chunk_off, const int* __restrict__ offs, int nbins,
                                int* __restrict__ pos, int* __restrict__ row_src, int src_div) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rank[i];
  if (r < 0) {
    pos[i] = -1;
    return;
  }
  const int key = keys[i] - lo;
  const int c = i / kChunk;
  const int p = offs[key] + chunk_off[static_cast<long>(c) * nbins + key] + r;
  pos[i] = p;
  if (row_src) row_src[p] = i / src_div;
}

// Returns (pos[n], offs[nbins+1], counts[nbins], row_src[cap]).  row_src maps
// each sorted slot to (input index / src_div), -1 for padding.  cap is the
// host-side capacity bound n + nbins * (pad - 1).
std::vector<at::Tensor> bucket_sort(const at::Tensor& keys, int64_t lo, int64_t hi, int64_t pad, int64_t src_div) {
  TORCH_CHECK(keys.scalar_type() == at::kInt && keys.is_contiguous(), "bucket_sort: int32 keys");
  const at::cuda::CUDAGuard guard(keys.device());
  const int n = static_cast<int>(keys.numel());
  const int nbins = static_cast<int>(hi - lo);
  const int nchunks = std::max(1, (n + kChunk - 1) / kChunk);
  auto opts = keys.options();
  auto rank = at::empty({n}, opts);
  auto chunk = at::zeros({nchunks, nbins}, opts);
  auto totals = at::empty({nbins}, opts);
  auto offs = at::empty({nbins + 1}, opts);
  auto counts = at::empty({nbins}, opts);
  auto pos = at::empty({n}, opts);
  const int64_t cap = n + static_cast<int64_t>(nbins) * std::max<int64_t>(0, pad - 1);
  auto row_src = at::full({cap}, -1, opts);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (n > 0) {
    sort_rank_kernel<<<nchunks, kChunk, 0, stream>>>(keys.data_ptr<int>(), n, (int)lo, (int)hi, rank.data_ptr<int>(),
                                                     chunk.data_ptr<int>(), nbins);
  }
  if (nbins > 0)
    sort_chunk_scan_kernel<<<nbins, 256, 0, stream>>>(chunk.data_ptr<int>(), nchunks, nbins, totals.data_ptr<int>());
  sort_bin_scan_kernel<<<1, 1024, 0, stream>>>(totals.data_ptr<int>(), nbins, (int)pad, offs.data_ptr<int>(),
                                               counts.data_ptr<int>());
  if (n > 0) {
    sort_pos_kernel<<<(n + 255) / 256, 256, 0, stream>>>(keys.data_ptr<int>(), n, (int)lo, rank.data_ptr<int>(),
                                                         chunk.data_ptr<int>(), offs.data_ptr<int>(), nbins,
                                                         pos.data_ptr<int>(), row_src.data_ptr<int>(), (int)src_div);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {pos, offs, counts, row_src};
}

// ---------------------------------------------------------------------------
// Row gather / scatter helpers (one warp per output row, 16-byte vectors).
// ---------------------------------------------------------------------------
// out[r] = src[row_src[r]] (row_src < 0 or r >= *total -> zeros)
__global__ void gather_rows_kernel(const bf16x8* __restrict__ src, const int* __restrict__ row_src,
                                   const int* __restrict__ total, int cap, int vecs, bf16x8* __restrict__ out,
                                   int src_rows) {
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  const int lim = total ? min(cap, *total) : cap;
  for (int r = warp; r < lim; r += nwarps) {
    int s = row_src[r];
    if (s >= 0 && !SB_IN_RANGE(s, src_rows)) s = -1;
    for (int v = lane; v < vecs; v += 32) {
      bf16x8 val;
      if (s >= 0) val = src[static_cast<long>(s) * vecs + v];
      else val.w[0] = val.w[1] = val.w[2] = val.w[3] = 0u;
      out[static_cast<long>(r) * vecs + v] = val;
    }
  }
}

void gather_rows(const at::Tensor& src, const at::Tensor& row_src, const c10::optional<at::Tensor>& total,
                 at::Tensor& out) {
  const at::cuda::CUDAGuard guard(src.device());
  const int H = static_cast<int>(src.size(-1));
  TORCH_CHECK(H % 8 == 0, "gather_rows: H % 8");
  const int cap = static_cast<int>(out.size(0));
  const int blocks = std::max(1, std::min((cap + 7) / 8, 148 * 8));
  gather_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16x8*>(src.data_ptr()), row_src.data_ptr<int>(),
      total.has_value() ? total->data_ptr<int>() : nullptr, cap, H / 8, reinterpret_cast<bf16x8*>(out.data_ptr()),
      static_cast<int>(src.size(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[t] = sum_j w[t,j] * y[pos[t,j]]   (pos < 0 skipped);  optional residual add
template <int NV>
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos,
                               const float* __restrict__ w, int T, int k, __nv_bfloat16* __restrict__ out,
                               int peer_lo, int peer_hi, int own_off, Xchg xc, int y_rows) {
  // Tensor-parallel form: token rows in [peer_lo, peer_hi) go to the peer's
  // receive buffer (xc.peer_out, row t - peer_lo) over NVLink, the others to
  // out at row t - own_off; then the kernel signals.  The expert combine's
  // partial sums thus leave in the same pass that computes them.
  constexpr int H = NV * 256;
  __nv_bfloat16* opeer = reinterpret_cast<__nv_bfloat16*>(xc.peer_out);
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  for (int t = warp; t < T; t += nwarps) {
    float acc[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int p = pos[static_cast<long>(t) * k + j];
      if (p < 0 || !SB_IN_RANGE(p, y_rows)) continue;
      const float wj = w[static_cast<long>(t) * k + j];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float v[8];
        bf16x8_to_float(reinterpret_cast<const bf16x8*>(y + static_cast<long>(p) * H)[i * 32 + lane], v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[i][q] += wj * v[q];
      }
    }
    __nv_bfloat16* dst = (opeer != nullptr && t >= peer_lo && t < peer_hi)
                             ? opeer + static_cast<long>(t - peer_lo) * H
                             : out + static_cast<long>(t - own_off) * H;
#pragma unroll
    for (int i = 0; i < NV; ++i) reinterpret_cast<bf16x8*>(dst)[i * 32 + lane] = float_to_bf16x8(acc[i]);
  }
  xchg_signal(xc);
}

// Backward of combine:
//   dy[r]  = w_r * dout[src(r)]   (zeros for padding rows)
//   dw[t,j] = <dout[t], y[pos[t,j]]>
template <int NV>
__global__ void combine_bwd_rows_kernel(const __nv_bfloat16* __restrict__ dout, const int* __restrict__ row_src,
                                        const int* __restrict__ slot_of_row, const float* __restrict__ w,
                                        const int* __restrict__ total, int cap, __nv_bfloat16* __restrict__ dy,
                                        int dout_rows, int n_slots) {
  constexpr int H = NV * 256;
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  const int lim = min(cap, *total);
  for (int r = warp; r < lim; r += nwarps) {
    int t = row_src[r];
    if (t >= 0 && !(SB_IN_RANGE(t, dout_rows) && SB_IN_RANGE(slot_of_row[r], n_slots))) t = -1;
    const float wr = t >= 0 ? w[slot_of_row[r]] : 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float v[8];
      if (t >= 0) {
        bf16x8_to_float(reinterpret_cast<const bf16x8*>(dout + static_cast<long>(t) * H)[i * 32 + lane], v);
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] *= wr;
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = 0.f;
      }
      reinterpret_cast<bf16x8*>(dy + static_cast<long>(r) * H)[i * 32 + lane] = float_to_bf16x8(v);
    }
  }
}

template <int NV>
__global__ void combine_bwd_weights_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                           const int* __restrict__ pos, int T, int k, float* __restrict__ dw,
                                           int y_rows) {
  constexpr int H = NV * 256;
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  for (int t = warp; t < T; t += nwarps) {
    float d[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i)
      bf16x8_to_float(reinterpret_cast<const bf16x8*>(dout + static_cast<long>(t) * H)[i * 32 + lane], d[i]);
    for (int j = 0; j < k; ++j) {
      const int p = pos[static_cast<long>(t) * k + j];
      float s = 0.f;
      if (p >= 0 && SB_IN_RANGE(p, y_rows)) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float v[8];
          bf16x8_to_float(reinterpret_cast<const bf16x8*>(y + static_cast<long>(p) * H)[i * 32 + lane], v);
#pragma unroll
          for (int q = 0; q < 8; ++q) s += d[i][q] * v[q];
        }
      }
      s = warp_sum(s);
      if (lane == 0) dw[static_cast<long>(t) * k + j] = s;
    }
  }
}

// dx[t] (+)= sum_j dperm[pos[t,j]]
template <int NV>
__global__ void scatter_back_kernel(const __nv_bfloat16* __restrict__ dperm, const int* __restrict__ pos, int T,
                                    int k, __nv_bfloat16* __restrict__ dx, int accumulate, int perm_rows) {
  constexpr int H = NV * 256;
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  for (int t = warp; t < T; t += nwarps) {
    float acc[NV][8];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (accumulate) bf16x8_to_float(reinterpret_cast<const bf16x8*>(dx + static_cast<long>(t) * H)[i * 32 + lane], acc[i]);
      else {
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[i][q] = 0.f;
      }
    }
    for (int j = 0; j < k; ++j) {
      const int p = pos[static_cast<long>(t) * k + j];
      if (p < 0 || !SB_IN_RANGE(p, perm_rows)) continue;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float v[8];
        bf16x8_to_float(reinterpret_cast<const bf16x8*>(dperm + static_cast<long>(p) * H)[i * 32 + lane], v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[i][q] += v[q];
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i)
      reinterpret_cast<bf16x8*>(dx + static_cast<long>(t) * H)[i * 32 + lane] = float_to_bf16x8(acc[i]);
  }
}

static int warp_blocks(int rows) { return std::max(1, std::min((rows + 7) / 8, 148 * 8)); }

#define SB_H_DISPATCH(H, MACRO)   \
  switch (H) {                    \
    case 256: MACRO(1); break;    \
    case 512: MACRO(2); break;    \
    case 1024: MACRO(4); break;   \
    default: TORCH_CHECK(false, "moe: hidden size must be 256/512/1024"); \
  }

// split (optional) = [peer_lo, peer_hi, own_off]: rows in [peer_lo, peer_hi)
// go to xchg's peer_out, the rest to out (allocated [T - (peer_hi - peer_lo), H]
// when not given) at row t - own_off.
at::Tensor combine(const at::Tensor& y, const at::Tensor& pos, const at::Tensor& w, int64_t T,
                   const c10::optional<at::Tensor>& out_opt, const std::vector<int64_t>& split,
                   const std::vector<int64_t>& xchg) {
  const at::cuda::CUDAGuard guard(y.device());
  const int H = static_cast<int>(y.size(-1));
  const int k = static_cast<int>(pos.size(-1));
  const Xchg xc = xchg_from(xchg);
  TORCH_CHECK(split.empty() || (split.size() == 3 && xc.peer_out != nullptr), "combine: split needs a peer buffer");
  const int peer_lo = split.empty() ? 0 : static_cast<int>(split[0]);
  const int peer_hi = split.empty() ? 0 : static_cast<int>(split[1]);
  const int own_off = split.empty() ? 0 : static_cast<int>(split[2]);
  const int64_t own_rows = T - (peer_hi - peer_lo);
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({own_rows, H}, y.options());
  TORCH_CHECK(out.is_contiguous() && out.numel() == own_rows * H, "combine: out size");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto yp = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
#define SB_L(NV) combine_kernel<NV><<<warp_blocks((int)T), 256, 0, stream>>>(yp, pos.data_ptr<int>(), w.data_ptr<float>(), (int)T, k, op, peer_lo, peer_hi, own_off, xc, static_cast<int>(y.size(0)))
  SB_H_DISPATCH(H, SB_L)
#undef SB_L
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Returns (dy [cap, H], dw [T, k]).
std::vector<at::Tensor> combine_bwd(const at::Tensor& dout, const at::Tensor& y, const at::Tensor& pos,
                                    const at::Tensor& w, const at::Tensor& row_src, const at::Tensor& slot_of_row,
                                    const at::Tensor& total) {
  const at::cuda::CUDAGuard guard(y.device());
  const int H = static_cast<int>(y.size(-1));
  const int T = static_cast<int>(pos.size(0)), k = static_cast<int>(pos.size(1));
  const int cap = static_cast<int>(y.size(0));
  auto dy = at::empty_like(y);
  auto dw = at::empty({T, k}, w.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto dp = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  auto yp = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  auto dyp = reinterpret_cast<__nv_bfloat16*>(dy.data_ptr());
#define SB_L(NV)                                                                                                   \
  combine_bwd_rows_kernel<NV><<<warp_blocks(cap), 256, 0, stream>>>(dp, row_src.data_ptr<int>(),                  \
      slot_of_row.data_ptr<int>(), w.data_ptr<float>(), total.data_ptr<int>(), cap, dyp,                       \
      static_cast<int>(dout.size(0)), static_cast<int>(w.numel()));                          \
  combine_bwd_weights_kernel<NV><<<warp_blocks(T), 256, 0, stream>>>(dp, yp, pos.data_ptr<int>(), T, k, dw.data_ptr<float>(), cap)
  SB_H_DISPATCH(H, SB_L)
#undef SB_L
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dy, dw};
}

void scatter_back(const at::Tensor& dperm, const at::Tensor& pos, at::Tensor& dx, bool accumulate) {
  const at::cuda::CUDAGuard guard(dperm.device());
  const int H = static_cast<int>(dperm.size(-1));
  const int T = static_cast<int>(pos.size(0)), k = static_cast<int>(pos.size(1));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto pp = reinterpret_cast<const __nv_bfloat16*>(dperm.data_ptr());
  auto xp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
#define SB_L(NV) scatter_back_kernel<NV><<<warp_blocks(T), 256, 0, stream>>>(pp, pos.data_ptr<int>(), T, k, xp, accumulate ? 1 : 0, static_cast<int>(dperm.size(0)))
  SB_H_DISPATCH(H, SB_L)
#undef SB_L
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// slot_of_row[r] = index i (= t*k + j) of the (token, choice) pair stored in row r.
__global__ void invert_pos_kernel(const int* __restrict__ pos, int n, int* __restrict__ slot_of_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int p = pos[i];
  if (p >= 0) slot_of_row[p] = i;
}

at::Tensor invert_pos(const at::Tensor& pos, int64_t cap) {
  const at::cuda::CUDAGuard guard(pos.device());
  auto out = at::full({cap}, -1, pos.options());
  const int n = static_cast<int>(pos.numel());
  if (n > 0)
    invert_pos_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(pos.data_ptr<int>(), n,
                                                                                   out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// ---------------------------------------------------------------------------
// Embedding: forward gather and deterministic backward (sorted segments).
// ---------------------------------------------------------------------------
// One warp per vocabulary row with at least one token: sums its tokens' rows
// (already in token order) and adds into dW (fp32).
__global__ void embedding_segment_sum_kernel(const __nv_bfloat16* __restrict__ dout, const int* __restrict__ row_src,
                                             const int* __restrict__ offs, int V, int H,
                                             float* __restrict__ dW) {
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  for (int v = warp; v < V; v += nwarps) {
    const int b = offs[v], e = offs[v + 1];
    if (b == e) continue;
    for (int c = lane * 8; c < H; c += 256) {
      float acc[8];
      float4* dst = reinterpret_cast<float4*>(dW + static_cast<long>(v) * H + c);
      float4 o0 = dst[0], o1 = dst[1];
      acc[0] = o0.x; acc[1] = o0.y; acc[2] = o0.z; acc[3] = o0.w;
      acc[4] = o1.x; acc[5] = o1.y; acc[6] = o1.z; acc[7] = o1.w;
      for (int s = b; s < e; ++s) {
        float f[8];
        bf16x8_to_float(*reinterpret_cast<const bf16x8*>(dout + static_cast<long>(row_src[s]) * H + c), f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += f[q];
      }
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// dW (fp32 [V, H]) += scatter of dout rows by ids, deterministic.
void embedding_bwd(const at::Tensor& dout, const at::Tensor& ids, at::Tensor& dW, int64_t vocab_lo) {
  const at::cuda::CUDAGuard guard(dout.device());
  TORCH_CHECK(dW.scalar_type() == at::kFloat && dW.is_contiguous(), "embedding_bwd: fp32 dW");
  const int V = static_cast<int>(dW.size(0)), H = static_cast<int>(dW.size(1));
  TORCH_CHECK(H % 256 == 0, "embedding_bwd: H % 256");
  auto r = bucket_sort(ids, vocab_lo, vocab_lo + V, 1, 1);
  const at::Tensor& offs = r[1];
  const at::Tensor& row_src = r[3];
  const int blocks = std::max(1, std::min((V + 7) / 8, 148 * 8));
  embedding_segment_sum_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), row_src.data_ptr<int>(), offs.data_ptr<int>(), V, H,
      dW.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[t] = W[ids[t] - lo] if in range else 0
__global__ void embedding_fwd_kernel(const bf16x8* __restrict__ W, const int* __restrict__ ids, int T, int lo, int V,
                                     int vecs, bf16x8* __restrict__ out) {
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nwarps = gridDim.x * (blockDim.x / 32);
  for (int t = warp; t < T; t += nwarps) {
    const int id = ids[t] - lo;
    const bool ok = id >= 0 && id < V;
    for (int v = lane; v < vecs; v += 32) {
      bf16x8 val;
      if (ok) val = W[static_cast<long>(id) * vecs + v];
      else val.w[0] = val.w[1] = val.w[2] = val.w[3] = 0u;
      out[static_cast<long>(t) * vecs + v] = val;
    }
  }
}

at::Tensor embedding_fwd(const at::Tensor& W, const at::Tensor& ids, int64_t vocab_lo) {
  const at::cuda::CUDAGuard guard(W.device());
  const int H = static_cast<int>(W.size(1));
  const int T = static_cast<int>(ids.numel());
  auto out = at::empty({T, H}, W.options());
  embedding_fwd_kernel<<<warp_blocks(T), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16x8*>(W.data_ptr()), ids.data_ptr<int>(), T, (int)vocab_lo, (int)W.size(0), H / 8,
      reinterpret_cast<bf16x8*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// ---------------------------------------------------------------------------
// SwiGLU on interleaved gate/up blocks of 16 (layout produced by the GEMM
// epilogue): h[:, 32b + i] = gate_{16b+i}, h[:, 32b + 16 + i] = up_{16b+i}.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ h, long rows, int F, __nv_bfloat16* __restrict__ a) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;  // over rows * F/16 blocks of 16
  const int nb = F / 16;
  if (i >= rows * nb) return;
  const long r = i / nb;
  const int b = static_cast<int>(i % nb);
  const __nv_bfloat16* src = h + r * 2 * F + b * 32;
  float g[16], u[16], o[16];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[0], g);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[1], g + 8);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[2], u);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[3], u + 8);
#pragma unroll
  for (int q = 0; q < 16; ++q) o[q] = silu(g[q]) * u[q];
  bf16x8* dst = reinterpret_cast<bf16x8*>(a + r * F + b * 16);
  dst[0] = float_to_bf16x8(o);
  dst[1] = float_to_bf16x8(o + 8);
}

// dh = [dg | du] interleaved, from h and da.  Rows with row_valid == 0 (padding) get 0.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ da,
                                  long rows, int F, __nv_bfloat16* __restrict__ dh) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nb = F / 16;
  if (i >= rows * nb) return;
  const long r = i / nb;
  const int b = static_cast<int>(i % nb);
  const __nv_bfloat16* src = h + r * 2 * F + b * 32;
  float g[16], u[16], d[16], dg[16], du[16];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[0], g);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[1], g + 8);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[2], u);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(src)[3], u + 8);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(da + r * F + b * 16)[0], d);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(da + r * F + b * 16)[1], d + 8);
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const float sg = __fdividef(1.f, 1.f + __expf(-g[q]));
    const float s = g[q] * sg;
    du[q] = d[q] * s;
    dg[q] = d[q] * u[q] * sg * (1.f + g[q] * (1.f - sg));
  }
  bf16x8* dst = reinterpret_cast<bf16x8*>(dh + r * 2 * F + b * 32);
  dst[0] = float_to_bf16x8(dg);
  dst[1] = float_to_bf16x8(dg + 8);
  dst[2] = float_to_bf16x8(du);
  dst[3] = float_to_bf16x8(du + 8);
}

at::Tensor swiglu_fwd(const at::Tensor& h) {
  const at::cuda::CUDAGuard guard(h.device());
  const int F = static_cast<int>(h.size(-1) / 2);
  TORCH_CHECK(F % 16 == 0, "swiglu: F % 16");
  const long rows = h.numel() / h.size(-1);
  auto a = at::empty({rows, F}, h.options());
  const long n = rows * (F / 16);
  if (n > 0)
    swiglu_fwd_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), rows, F, reinterpret_cast<__nv_bfloat16*>(a.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return a;
}

at::Tensor swiglu_bwd(const at::Tensor& h, const at::Tensor& da) {
  const at::cuda::CUDAGuard guard(h.device());
  const int F = static_cast<int>(h.size(-1) / 2);
  const long rows = h.numel() / h.size(-1);
  auto dh = at::empty_like(h);
  const long n = rows * (F / 16);
  if (n > 0)
    swiglu_bwd_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()),
        rows, F, reinterpret_cast<__nv_bfloat16*>(dh.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dh;
}

}  // namespace moe
}  // namespace sb
