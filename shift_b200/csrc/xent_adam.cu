// Fused cross-entropy (forward + gradient in one pass over the logits) and
// the fused AdamW step over flat fp32 master buffers, for sm_100a.
//
// AdamW follows torch.optim.AdamW's single-tensor arithmetic order (the
// optimizer the reference builds at shift_full/train.py:223: betas (0.9, 0.999),
// eps 1e-8, weight decay 0.01) but keeps fp32 master weights and moments and
// writes the bf16 compute copy of the parameters in the same pass.  Inputs and
// outputs may be different buffers (ping-pong), so an uncommitted step leaves
// the previous state untouched.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace sb {
namespace xent {

// One block per row.  loss[r] = logsumexp(z) - z[label]; dz = (softmax - onehot) * scale
// written over the logits (bf16) in place.  Rows with label < 0 get loss 0, dz 0.
// The row is staged as bf16 in shared memory (each thread only reads back the
// vectors it stored, so no barrier is needed for it) and exp(z - max) is
// evaluated twice (row sum, then gradient) instead of being kept in fp32
// registers: three CTAs per SM overlap one row's reductions with the other
// rows' loads and stores.  Max and sum run in four independent chains.
template <int VPT>  // bf16x8 vectors per thread
__global__ void __launch_bounds__(256, 3)
xent_kernel(__nv_bfloat16* __restrict__ logits, const int* __restrict__ labels, int V, float scale,
            float* __restrict__ loss, int label_lo) {
  extern __shared__ bf16x8 srow[];   // V / 8 vectors
  const long r = blockIdx.x;
  __nv_bfloat16* row = logits + r * V;
  const int label = labels[r];
  const int vecs = V / 8;
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < vecs) srow[v] = reinterpret_cast<const bf16x8*>(row)[v];
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < vecs) {
      float z[8];
      bf16x8_to_float(srow[v], z);
#pragma unroll
      for (int j = 0; j < 8; ++j) m4[j & 3] = fmaxf(m4[j & 3], z[j]);
    }
  }
  float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
  __shared__ float red[32];
  __shared__ float bcast;
  mx = warp_max(mx);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) bcast = v;
  }
  __syncthreads();
  mx = bcast;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < vecs) {
      float z[8];
      bf16x8_to_float(srow[v], z);
#pragma unroll
      for (int j = 0; j < 8; ++j) s4[j & 3] += __expf(z[j] - mx);
    }
  }
  float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  s = warp_sum(s);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) bcast = v;
  }
  __syncthreads();
  const float sum = bcast;
  const float inv = 1.f / sum;
  const int lab = label - label_lo;
  const bool valid = label >= 0 && lab >= 0 && lab < V;
  if (threadIdx.x == 0) {
    if (valid) {
      const float zl = __bfloat162float(row[lab]);
      loss[r] = (logf(sum) + mx - zl);
    } else {
      loss[r] = 0.f;
    }
  }
  __syncthreads();  // row[lab] read above before it is overwritten
  const float sc = label >= 0 ? scale : 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < vecs) {
      float z[8], g[8];
      bf16x8_to_float(srow[v], z);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = v * 8 + j;
        g[j] = (__expf(z[j] - mx) * inv - ((valid && col == lab) ? 1.f : 0.f)) * sc;
      }
      reinterpret_cast<bf16x8*>(row)[v] = float_to_bf16x8(g);
    }
  }
}

// Returns per-row loss (fp32); logits are overwritten by dlogits * scale.
at::Tensor xent_fwd_bwd(at::Tensor& logits, const at::Tensor& labels, double scale, int64_t label_lo) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous(), "xent: bf16 contiguous logits");
  TORCH_CHECK(labels.scalar_type() == at::kInt, "xent: int32 labels");
  const at::cuda::CUDAGuard guard(logits.device());
  const int V = static_cast<int>(logits.size(-1));
  const long rows = logits.numel() / V;
  TORCH_CHECK(V % 8 == 0, "xent: V % 8");
  TORCH_CHECK(aligned16(logits.data_ptr()), "xent: logits must be 16-byte aligned");
  auto loss = at::empty({rows}, logits.options().dtype(at::kFloat));
  const int vecs = V / 8;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto lp = reinterpret_cast<__nv_bfloat16*>(logits.data_ptr());
  if (rows == 0) return loss;
  const size_t smem = static_cast<size_t>(V) * sizeof(__nv_bfloat16);
#define SB_XENT(VPT)                                                                                  \
  do {                                                                                                \
    C10_CUDA_CHECK(cudaFuncSetAttribute(xent_kernel<VPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                        256 * 8 * VPT * static_cast<int>(sizeof(__nv_bfloat16))));    \
    xent_kernel<VPT><<<rows, 256, smem, stream>>>(lp, labels.data_ptr<int>(), V, (float)scale,         \
                                                  loss.data_ptr<float>(), (int)label_lo);             \
  } while (0)
  if (vecs <= 256 * 2) SB_XENT(2);
  else if (vecs <= 256 * 8) SB_XENT(8);
  else if (vecs <= 256 * 16) SB_XENT(16);
  else TORCH_CHECK(false, "xent: vocabulary too large for one block (max 32768)");
#undef SB_XENT
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return loss;
}

}  // namespace xent

namespace adam {

struct AdamArgs {
  float lr, beta1, beta2, eps, wd;
  float bc1, bc2_sqrt;   // 1 - beta1^t, sqrt(1 - beta2^t)
  float grad_scale;
};

// master/m/v fp32 (in), grads bf16 list of up to 8 sources summed in order then
// scaled, results written to out_* (may alias the inputs).  Also writes bf16
// params and accumulates a non-finite flag.
struct GradSources {
  const __nv_bfloat16* p[8];
};

__global__ void adamw_kernel(const float* __restrict__ master, const float* __restrict__ m_in,
                             const float* __restrict__ v_in, const GradSources grads, int n_grads, float* __restrict__ master_out, float* __restrict__ m_out,
                             float* __restrict__ v_out, __nv_bfloat16* __restrict__ param_out, long n, AdamArgs a,
                             int* __restrict__ nonfinite, const int* __restrict__ sdev) {
  if (sdev != nullptr) {   // per-step scalars from device memory (graph-replayable)
    a.lr = __int_as_float(sdev[1]);
    a.bc1 = __int_as_float(sdev[2]);
    a.bc2_sqrt = __int_as_float(sdev[3]);
  }
  const long i0 = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x * 4;
  bool bad = false;
  for (long i = i0; i < n; i += stride) {
    if (i + 4 <= n) {
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < n_grads; ++s) {
        const uint2 raw = *reinterpret_cast<const uint2*>(grads.p[s] + i);
        const float2 a0 = unpack_bf16x2(raw.x), a1 = unpack_bf16x2(raw.y);
        g[0] += a0.x; g[1] += a0.y; g[2] += a1.x; g[3] += a1.y;
      }
      const float4 p4 = *reinterpret_cast<const float4*>(master + i);
      const float4 m4 = *reinterpret_cast<const float4*>(m_in + i);
      const float4 v4 = *reinterpret_cast<const float4*>(v_in + i);
      float p[4] = {p4.x, p4.y, p4.z, p4.w}, m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float gq = g[q] * a.grad_scale;
        bad |= !isfinite(gq);
        p[q] = p[q] * (1.f - a.lr * a.wd);
        m[q] = m[q] + (gq - m[q]) * (1.f - a.beta1);
        v[q] = v[q] * a.beta2 + (1.f - a.beta2) * gq * gq;
        const float denom = sqrtf(v[q]) / a.bc2_sqrt + a.eps;
        p[q] = p[q] - (a.lr / a.bc1) * (m[q] / denom);
      }
      *reinterpret_cast<float4*>(master_out + i) = make_float4(p[0], p[1], p[2], p[3]);
      *reinterpret_cast<float4*>(m_out + i) = make_float4(m[0], m[1], m[2], m[3]);
      *reinterpret_cast<float4*>(v_out + i) = make_float4(v[0], v[1], v[2], v[3]);
      uint2 pb;
      pb.x = pack_bf16x2(p[0], p[1]);
      pb.y = pack_bf16x2(p[2], p[3]);
      *reinterpret_cast<uint2*>(param_out + i) = pb;
    } else {
      for (long j = i; j < n; ++j) {
        float g = 0.f;
        for (int s = 0; s < n_grads; ++s) g += __bfloat162float(grads.p[s][j]);
        g *= a.grad_scale;
        bad |= !isfinite(g);
        float p = master[j] * (1.f - a.lr * a.wd);
        float m = m_in[j] + (g - m_in[j]) * (1.f - a.beta1);
        float v = v_in[j] * a.beta2 + (1.f - a.beta2) * g * g;
        const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
        p = p - (a.lr / a.bc1) * (m / denom);
        master_out[j] = p;
        m_out[j] = m;
        v_out[j] = v;
        param_out[j] = __float2bfloat16(p);
      }
    }
  }
  if (bad && nonfinite) atomicOr(nonfinite, 1);
}

// grads: list of bf16 tensors (same numel) whose sum is the gradient.
void adamw_step(const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, const std::vector<at::Tensor>& grads,
                at::Tensor& master_out, at::Tensor& m_out, at::Tensor& v_out, at::Tensor& param_out, double lr,
                double beta1, double beta2, double eps, double wd, int64_t step, double grad_scale,
                const c10::optional<at::Tensor>& nonfinite, const c10::optional<at::Tensor>& step_dev) {
  TORCH_CHECK(grads.size() >= 1 && grads.size() <= 8, "adamw: 1..8 gradient sources");
  if (step_dev.has_value())
    TORCH_CHECK(step_dev->is_cuda() && step_dev->scalar_type() == at::kInt && step_dev->numel() >= 4 &&
                    step_dev->device() == master.device(),
                "adamw: step_dev int32[>=4] on the parameter's device");
  const at::cuda::CUDAGuard guard(master.device());
  const long n = master.numel();
  for (auto& g : grads) TORCH_CHECK(g.numel() == n && g.scalar_type() == at::kBFloat16, "adamw: bf16 grads of equal size");
  AdamArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.grad_scale = static_cast<float>(grad_scale);
  GradSources src{};
  for (size_t i = 0; i < grads.size(); ++i) src.p[i] = reinterpret_cast<const __nv_bfloat16*>(grads[i].data_ptr());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const long blocks = std::min<long>((n / 4 + threads - 1) / threads + 1, 148 * 16);
  adamw_kernel<<<blocks, threads, 0, stream>>>(
      master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      src, static_cast<int>(grads.size()),
      master_out.data_ptr<float>(), m_out.data_ptr<float>(), v_out.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(param_out.data_ptr()), n, a,
      nonfinite.has_value() ? nonfinite->data_ptr<int>() : nullptr,
      step_dev.has_value() ? step_dev->data_ptr<int>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Non-finite check of a bf16 buffer: flag |= any(!isfinite).
__global__ void nonfinite_kernel(const __nv_bfloat16* __restrict__ x, long n, int* __restrict__ flag) {
  const long i0 = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool bad = false;
  for (long i = i0 * 8; i < n; i += static_cast<long>(gridDim.x) * blockDim.x * 8) {
    if (i + 8 <= n) {
      float f[8];
      bf16x8_to_float(*reinterpret_cast<const bf16x8*>(x + i), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) bad |= !isfinite(f[j]);
    } else {
      for (long j = i; j < n; ++j) bad |= !isfinite(__bfloat162float(x[j]));
    }
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x % 32) == 0) atomicOr(flag, 1);
}

void nonfinite_check(const at::Tensor& x, at::Tensor& flag) {
  const at::cuda::CUDAGuard guard(x.device());
  const long n = x.numel();
  if (n == 0) return;
  const long blocks = std::min<long>((n / 8 + 255) / 256 + 1, 148 * 8);
  nonfinite_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), n, flag.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace adam
}  // namespace sb
