// RMSNorm (forward / backward, with fused residual add) and rotary embedding
// for sm_100a.  One warp owns one row; rows are 128-bit vectorised.  Weight
// gradients are reduced deterministically: per-block partials in a fixed row
// order, then a column reduction over blocks in block order.
//
// Parity: HF Qwen2 RMSNorm (x * rsqrt(mean(x^2) + eps) * w, fp32 statistics)
// and HF rotate-half RoPE, as used by the model the reference trains
// (shift_full/train.py:209-216 loads it; the model code itself is external).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "xchg.h"

namespace sb {
namespace norm {

constexpr int kWarps = 8;

// NV = H / 256: number of 8-element vectors per lane.
// Tensor-parallel forms: delta2 (a partial sum another GPU wrote into this
// GPU's memory; waited for through xc) is added with delta, and y_peer (in
// xc.peer_out) receives a second copy of y in a peer's gather buffer; the
// kernel then signals through xc.  This fuses the sequence-parallel
// all-gather into the norm that produces its input, and the reduce-scatter's
// reduction into the norm that consumes it.
template <int NV, bool kAdd>
__global__ void __launch_bounds__(kWarps * 32, 3)
rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                   const __nv_bfloat16* __restrict__ delta2, const __nv_bfloat16* __restrict__ w,
                   __nv_bfloat16* __restrict__ h_out, __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out,
                   int rows, float eps, Xchg xc, int* status) {
  constexpr int H = NV * 256;
  if (!xchg_wait_cta(xc, status)) return;
  __nv_bfloat16* y_peer = reinterpret_cast<__nv_bfloat16*>(xc.peer_out);
  const int lane = threadIdx.x % 32;
  const int warp = blockIdx.x * kWarps + threadIdx.x / 32;
  const int nwarps = gridDim.x * kWarps;
  float wv[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) bf16x8_to_float(reinterpret_cast<const bf16x8*>(w)[i * 32 + lane], wv[i]);
  for (int r = warp; r < rows; r += nwarps) {
    const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + static_cast<long>(r) * H);
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      bf16x8_to_float(xr[i * 32 + lane], v[i]);
      if (kAdd) {
        float d[8];
        bf16x8_to_float(reinterpret_cast<const bf16x8*>(delta + static_cast<long>(r) * H)[i * 32 + lane], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += d[j];
        if (delta2 != nullptr) {
          bf16x8_to_float(reinterpret_cast<const bf16x8*>(delta2 + static_cast<long>(r) * H)[i * 32 + lane], d);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] += d[j];
        }
        bf16x8 hv = float_to_bf16x8(v[i]);
        reinterpret_cast<bf16x8*>(h_out + static_cast<long>(r) * H)[i * 32 + lane] = hv;
        bf16x8_to_float(hv, v[i]);  // normalise the rounded residual stream
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / H + eps);
    if (lane == 0) rstd_out[r] = rs;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rs * wv[i][j];
      const bf16x8 ov = float_to_bf16x8(o);
      reinterpret_cast<bf16x8*>(y + static_cast<long>(r) * H)[i * 32 + lane] = ov;
      if (y_peer != nullptr) reinterpret_cast<bf16x8*>(y_peer + static_cast<long>(r) * H)[i * 32 + lane] = ov;
    }
  }
  xchg_signal(xc);
}

// dx = rstd * (dy*w - xhat * mean(dy*w*xhat)) (+ dres);  partial dw per block.
// Tensor-parallel forms as in the forward: dy2 (a peer-written partial,
// waited for through xc) is added to dy, and dx is also written to
// xc.peer_out (a peer's gather buffer), then the kernel signals.
//
// A row's inputs stay in registers as packed bf16 (x, dy, dy2, dres all
// loaded up front, so one memory latency per row), the fp32 values are
// recomputed in the second pass, and each thread's dw partial sums live in
// its own slots of the CTA's reduction buffer in shared memory, and the
// weight is re-read from L1: at H = 1024 that keeps the kernel under 128
// registers, two CTAs (16 warps) per SM instead of one.
template <int NV, bool kRes, bool kDy2>
__global__ void __launch_bounds__(kWarps * 32, 2)
rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ dy2,
                   const __nv_bfloat16* __restrict__ x, const float* __restrict__ rstd,
                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_partial, int rows, Xchg xc, int* status) {
  constexpr int H = NV * 256;
  __shared__ float red[kWarps][H];
  const bool go = xchg_wait_cta(xc, status);   // uniform per CTA
  __nv_bfloat16* dx_peer = reinterpret_cast<__nv_bfloat16*>(xc.peer_out);
  const int lane = threadIdx.x % 32;
  const int wib = threadIdx.x / 32;
  const int warp = blockIdx.x * kWarps + wib;
  const int nwarps = gridDim.x * kWarps;
  // this thread's dw partials: red[wib][(i * 32 + lane) * 8 + j], touched by no other thread until the end
  float4* dwacc = reinterpret_cast<float4*>(&red[wib][lane * 8]);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    dwacc[i * 64] = make_float4(0.f, 0.f, 0.f, 0.f);
    dwacc[i * 64 + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r = go ? warp : rows; r < rows; r += nwarps) {
    const float rs = rstd[r];
    const long ro = static_cast<long>(r) * H;
    bf16x8 xp[NV], dp[NV], d2p[kDy2 ? NV : 1], rp[kRes ? NV : 1];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      xp[i] = reinterpret_cast<const bf16x8*>(x + ro)[i * 32 + lane];
      dp[i] = reinterpret_cast<const bf16x8*>(dy + ro)[i * 32 + lane];
      if constexpr (kDy2) d2p[i] = reinterpret_cast<const bf16x8*>(dy2 + ro)[i * 32 + lane];
      if constexpr (kRes) rp[i] = reinterpret_cast<const bf16x8*>(dres + ro)[i * 32 + lane];
    }
    // the fp32 values of chunk i: xhat, dy (+ dy2), g = dy * w
    auto chunk = [&](int i, float* xh, float* dv, float* g) {
      float wv[8];
      bf16x8_to_float(xp[i], xh);
      bf16x8_to_float(dp[i], dv);
      bf16x8_to_float(ld_nc_bf16x8(reinterpret_cast<const bf16x8*>(w) + i * 32 + lane), wv);
      if constexpr (kDy2) {
        float d2[8];
        bf16x8_to_float(d2p[i], d2);
#pragma unroll
        for (int j = 0; j < 8; ++j) dv[j] += d2[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[j] *= rs;
        g[j] = dv[j] * wv[j];
      }
    };
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float xh[8], dv[8], g[8];
      chunk(i, xh, dv, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += g[j] * xh[j];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float4 a = dwacc[i * 64 + u];
        a.x += dv[4 * u] * xh[4 * u];
        a.y += dv[4 * u + 1] * xh[4 * u + 1];
        a.z += dv[4 * u + 2] * xh[4 * u + 2];
        a.w += dv[4 * u + 3] * xh[4 * u + 3];
        dwacc[i * 64 + u] = a;
      }
    }
    dot = warp_sum(dot) / H;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float xh[8], dv[8], g[8], o[8], rr[8];
      chunk(i, xh, dv, g);
      if constexpr (kRes) bf16x8_to_float(rp[i], rr);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rs * (g[j] - xh[j] * dot) + (kRes ? rr[j] : 0.f);
      const bf16x8 ov = float_to_bf16x8(o);
      reinterpret_cast<bf16x8*>(dx + ro)[i * 32 + lane] = ov;
      if (dx_peer != nullptr) reinterpret_cast<bf16x8*>(dx_peer + ro)[i * 32 + lane] = ov;
    }
  }
  xchg_signal(xc);
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += red[k][c];
    dw_partial[static_cast<long>(blockIdx.x) * H + c] = s;
  }
}

// out[c] (+)= sum_b partial[b, c], deterministic: a CTA owns 32 columns;
// warp w sums rows w, w+8, ... (lane = column, coalesced), then warp 0 adds
// the 8 warp sums in warp order.  256 threads per CTA.
__global__ void __launch_bounds__(256)
column_reduce_kernel(const float* __restrict__ partial, int nblocks, int cols, float* __restrict__ out_f32,
                     __nv_bfloat16* __restrict__ out_bf16, int accumulate) {
  __shared__ float red[8][32];
  const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < cols) {
#pragma unroll 4
    for (int b = w; b < nblocks; b += 8) s += partial[static_cast<long>(b) * cols + c];
  }
  red[w][lane] = s;
  __syncthreads();
  if (w != 0 || c >= cols) return;
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += red[k][lane];
  if (out_f32) out_f32[c] = accumulate ? out_f32[c] + t : t;
  if (out_bf16) out_bf16[c] = __float2bfloat16(accumulate ? __bfloat162float(out_bf16[c]) + t : t);
}

// Grid of a row-per-warp norm kernel: every row gets a warp, capped at the
// CTAs that are resident at once (per_sm per SM), which then loop over rows.
static int blocks_for(int rows, int per_sm) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return std::max(1, std::min((rows + kWarps - 1) / kWarps, sms * per_sm));
}

#define SB_NORM_DISPATCH(H, MACRO) \
  switch (H) {                     \
    case 256: MACRO(1); break;     \
    case 512: MACRO(2); break;     \
    case 1024: MACRO(4); break;    \
    default: TORCH_CHECK(false, "rmsnorm: hidden size must be 256/512/1024"); \
  }

// Returns (y, rstd) ; if delta is given also h = x + delta (written to h_out).
// Tensor-parallel options: delta2 (second partial added with delta), y_out
// (write y there instead of a new tensor), xchg (see xchg.h; peer_out gets a
// copy of y), status (the launch's status word).
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& delta,
                                    const at::Tensor& w, double eps, const c10::optional<at::Tensor>& delta2,
                                    const c10::optional<at::Tensor>& y_out, const std::vector<int64_t>& xchg,
                                    const c10::optional<at::Tensor>& status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "rmsnorm: bf16 contiguous x");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16, "rmsnorm: bf16 weight");
  const at::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / H);
  at::Tensor y;
  if (y_out.has_value()) {
    TORCH_CHECK(y_out->is_contiguous() && y_out->numel() == x.numel() && y_out->scalar_type() == at::kBFloat16,
                "rmsnorm: y_out must be a contiguous bf16 tensor of x's size");
    y = *y_out;
  } else {
    y = at::empty_like(x);
  }
  const Xchg xc = xchg_from(xchg);
  TORCH_CHECK(!delta2.has_value() || (delta.has_value() && delta2->is_contiguous() && delta2->numel() == x.numel()),
              "rmsnorm: delta2 needs delta and x's size");
  TORCH_CHECK(xc.wait_flag == nullptr || status.has_value(), "rmsnorm: a wait needs a status word");
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  auto d2p = delta2.has_value() ? reinterpret_cast<const __nv_bfloat16*>(delta2->data_ptr()) : nullptr;
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor h;
  const bool add = delta.has_value();
  if (add) {
    TORCH_CHECK(delta->is_contiguous() && delta->sizes() == x.sizes(), "rmsnorm: delta shape");
    h = at::empty_like(x);
  }
  TORCH_CHECK(aligned16(x.data_ptr()) && aligned16(w.data_ptr()) && aligned16(y.data_ptr()) &&
                  (!add || (aligned16(delta->data_ptr()) && aligned16(h.data_ptr()))) &&
                  (d2p == nullptr || aligned16(d2p)) && (xc.peer_out == nullptr || aligned16(xc.peer_out)),
              "rmsnorm: every row buffer must be 16-byte aligned");
  const int blocks = blocks_for(rows, 3);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto dp = add ? reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()) : nullptr;
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto hp = add ? reinterpret_cast<__nv_bfloat16*>(h.data_ptr()) : nullptr;
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
#define SB_LAUNCH(NV)                                                                                       \
  if (add) rmsnorm_fwd_kernel<NV, true><<<blocks, kWarps * 32, 0, stream>>>(xp, dp, d2p, wp, hp, yp, rstd.data_ptr<float>(), rows, (float)eps, xc, st); \
  else rmsnorm_fwd_kernel<NV, false><<<blocks, kWarps * 32, 0, stream>>>(xp, dp, d2p, wp, hp, yp, rstd.data_ptr<float>(), rows, (float)eps, xc, st);
  SB_NORM_DISPATCH(H, SB_LAUNCH)
#undef SB_LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (add) return {y, rstd, h};
  return {y, rstd};
}

// Returns dx; accumulates dw into dw_out (fp32 or bf16 tensor of shape [H]).
// Tensor-parallel options as in rmsnorm_fwd: dy2 (second partial of dy),
// dx_out, xchg (peer_out gets a copy of dx), status.
at::Tensor rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& w,
                       const c10::optional<at::Tensor>& dres, at::Tensor& dw_out, bool accumulate,
                       const c10::optional<at::Tensor>& dy2, const c10::optional<at::Tensor>& dx_out,
                       const std::vector<int64_t>& xchg, const c10::optional<at::Tensor>& status) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous(), "rmsnorm_bwd: contiguous inputs");
  const at::cuda::CUDAGuard guard(x.device());
  const int H = static_cast<int>(x.size(-1));
  const int rows = static_cast<int>(x.numel() / H);
  at::Tensor dx;
  if (dx_out.has_value()) {
    TORCH_CHECK(dx_out->is_contiguous() && dx_out->numel() == x.numel() && dx_out->scalar_type() == at::kBFloat16,
                "rmsnorm_bwd: dx_out must be a contiguous bf16 tensor of x's size");
    dx = *dx_out;
  } else {
    dx = at::empty_like(x);
  }
  const Xchg xc = xchg_from(xchg);
  TORCH_CHECK(!dy2.has_value() || (dy2->is_contiguous() && dy2->numel() == x.numel()), "rmsnorm_bwd: dy2 size");
  TORCH_CHECK(xc.wait_flag == nullptr || status.has_value(), "rmsnorm_bwd: a wait needs a status word");
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  auto dy2p = dy2.has_value() ? reinterpret_cast<const __nv_bfloat16*>(dy2->data_ptr()) : nullptr;
  TORCH_CHECK(aligned16(dy.data_ptr()) && aligned16(x.data_ptr()) && aligned16(w.data_ptr()) &&
                  aligned16(dx.data_ptr()) && (!dres.has_value() || aligned16(dres->data_ptr())) &&
                  (dy2p == nullptr || aligned16(dy2p)) && (xc.peer_out == nullptr || aligned16(xc.peer_out)),
              "rmsnorm_bwd: every row buffer must be 16-byte aligned");
  const int blocks = blocks_for(rows, 2);
  auto partial = at::empty({blocks, H}, x.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool res = dres.has_value();
  auto dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto rp = res ? reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr()) : nullptr;
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
#define SB_BWD(NV, R, D2) \
  rmsnorm_bwd_kernel<NV, R, D2><<<blocks, kWarps * 32, 0, stream>>>(dyp, dy2p, xp, rstd.data_ptr<float>(), wp, rp, dxp, partial.data_ptr<float>(), rows, xc, st)
#define SB_LAUNCH(NV)                  \
  if (res && dy2p) SB_BWD(NV, true, true);      \
  else if (res) SB_BWD(NV, true, false);        \
  else if (dy2p) SB_BWD(NV, false, true);       \
  else SB_BWD(NV, false, false);
  SB_NORM_DISPATCH(H, SB_LAUNCH)
#undef SB_LAUNCH
#undef SB_BWD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  float* of = dw_out.scalar_type() == at::kFloat ? dw_out.data_ptr<float>() : nullptr;
  __nv_bfloat16* ob = dw_out.scalar_type() == at::kBFloat16 ? reinterpret_cast<__nv_bfloat16*>(dw_out.data_ptr()) : nullptr;
  column_reduce_kernel<<<(H + 31) / 32, 256, 0, stream>>>(partial.data_ptr<float>(), blocks, H, of, ob, accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dx;
}

void column_reduce(const at::Tensor& partial, at::Tensor& out, bool accumulate) {
  const at::cuda::CUDAGuard guard(partial.device());
  const int cols = static_cast<int>(partial.size(1));
  const int nb = static_cast<int>(partial.size(0));
  float* of = out.scalar_type() == at::kFloat ? out.data_ptr<float>() : nullptr;
  __nv_bfloat16* ob = out.scalar_type() == at::kBFloat16 ? reinterpret_cast<__nv_bfloat16*>(out.data_ptr()) : nullptr;
  column_reduce_kernel<<<(cols + 31) / 32, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      partial.data_ptr<float>(), nb, cols, of, ob, accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// RoPE on the fused QKV activation [T, (Hq + 2*Hkv) * D] in place.
// q heads [0, Hq), k heads [Hq, Hq+Hkv); v untouched.  Position of row t is
// pos0 + (t % S).  cos/sin tables are [max_pos, D/2] fp32.
// sign = +1 forward rotation, -1 inverse (backward).
// ---------------------------------------------------------------------------
template <int D>
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int T, int S, int n_rot_heads, int row_stride,
                            int pos0, float sign) {
  // General form for any row stride / base offset: every access is a single
  // element (2-byte bf16, 4-byte fp32), so no alignment beyond the element's
  // own is assumed.  One thread rotates the pair (x1[i], x2[i]).
  constexpr int HALF = D / 2;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long per_row = static_cast<long>(n_rot_heads) * HALF;
  if (idx >= per_row * T) return;
  const int t = static_cast<int>(idx / per_row);
  const int rem = static_cast<int>(idx % per_row);
  const int head = rem / HALF;
  const int i = rem % HALF;
  const int pos = pos0 + (t % S);
  __nv_bfloat16* base = qkv + static_cast<long>(t) * row_stride + head * D;
  const float c = cos_t[static_cast<long>(pos) * HALF + i];
  const float s = sin_t[static_cast<long>(pos) * HALF + i] * sign;
  const float a = __bfloat162float(base[i]);
  const float b = __bfloat162float(base[HALF + i]);
  base[i] = __float2bfloat16(a * c - b * s);
  base[HALF + i] = __float2bfloat16(b * c + a * s);
}

// The same rotation with 16-byte accesses: thread (x, y) of a block rotates
// eight pairs (x1[i..i+7], x2[i..i+7]) of one head in row blockIdx.x * R + y,
// with x = head * (D / 16) + i / 8.  No division; the row pointer and stride
// must be 16-byte aligned (checked by the launcher).
template <int D>
__global__ void __launch_bounds__(512)
rope_vec_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                int T, int S, int row_stride, int pos0, float sign) {
  constexpr int HALF = D / 2;
  const int t = blockIdx.x * blockDim.y + threadIdx.y;
  if (t >= T) return;
  const int head = threadIdx.x / (HALF / 8);
  const int i = (threadIdx.x % (HALF / 8)) * 8;
  const int pos = pos0 + (t % S);
  __nv_bfloat16* base = qkv + static_cast<long>(t) * row_stride + head * D;
  const float4* cp = reinterpret_cast<const float4*>(cos_t + static_cast<long>(pos) * HALF + i);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + static_cast<long>(pos) * HALF + i);
  const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
  const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {s0.x * sign, s0.y * sign, s0.z * sign, s0.w * sign,
                       s1.x * sign, s1.y * sign, s1.z * sign, s1.w * sign};
  float a[8], b[8], oa[8], ob[8];
  bf16x8_to_float(*reinterpret_cast<const bf16x8*>(base + i), a);
  bf16x8_to_float(*reinterpret_cast<const bf16x8*>(base + HALF + i), b);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    oa[k] = a[k] * c[k] - b[k] * sn[k];
    ob[k] = b[k] * c[k] + a[k] * sn[k];
  }
  *reinterpret_cast<bf16x8*>(base + i) = float_to_bf16x8(oa);
  *reinterpret_cast<bf16x8*>(base + HALF + i) = float_to_bf16x8(ob);
}

void rope_(at::Tensor& qkv, const at::Tensor& cos_t, const at::Tensor& sin_t, int64_t S, int64_t n_rot_heads,
           int64_t head_dim, int64_t pos0, bool inverse) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1, "rope: bf16 qkv");
  TORCH_CHECK(head_dim == 64 || head_dim == 128, "rope: head_dim 64 or 128");
  const at::cuda::CUDAGuard guard(qkv.device());
  const int T = static_cast<int>(qkv.numel() / qkv.size(-1));
  const int row_stride = static_cast<int>(qkv.dim() >= 2 ? qkv.stride(-2) : qkv.size(-1));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto p = reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr());
  const float sign = inverse ? -1.f : 1.f;
  const int per_row = static_cast<int>(n_rot_heads * head_dim / 16);   // threads of one row
  if (T == 0) return;
  const bool aligned = reinterpret_cast<uintptr_t>(p) % 16 == 0 && row_stride % 8 == 0 &&
                       reinterpret_cast<uintptr_t>(cos_t.data_ptr()) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(sin_t.data_ptr()) % 16 == 0;
  if (aligned && per_row <= 512) {
    const int R = std::max(1, 256 / per_row);                           // rows per block
    const dim3 block(per_row, R);
    const int blocks = (T + R - 1) / R;
    if (head_dim == 64)
      rope_vec_kernel<64><<<blocks, block, 0, stream>>>(p, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T,
                                                        (int)S, row_stride, (int)pos0, sign);
    else
      rope_vec_kernel<128><<<blocks, block, 0, stream>>>(p, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T,
                                                         (int)S, row_stride, (int)pos0, sign);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const long work = static_cast<long>(T) * n_rot_heads * (head_dim / 2);
  const int threads = 256;
  const int blocks = static_cast<int>((work + threads - 1) / threads);
  if (head_dim == 64)
    rope_kernel<64><<<blocks, threads, 0, stream>>>(p, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T, (int)S,
                                                    (int)n_rot_heads, row_stride, (int)pos0, sign);
  else
    rope_kernel<128><<<blocks, threads, 0, stream>>>(p, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T, (int)S,
                                                     (int)n_rot_heads, row_stride, (int)pos0, sign);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace norm
}  // namespace sb
