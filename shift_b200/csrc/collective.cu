// Peer-memory collectives for one NVLink/NVSwitch box (sm_100a).
//
// Symmetric buffers are plain cudaMalloc allocations exported with CUDA IPC;
// peers map them once per membership (a "reconfigure" re-maps handles, it
// does not rebuild a communicator).  Synchronisation uses system-scope
// release/acquire flags in those buffers, and every wait is bounded: on
// expiry the kernel records kTimeoutPeer in the status word and returns.
//
// K1  fused_reduce_adamw: the cross-replica gradient reduction fused with
//     the bf16->fp32 cast, the participant normalisation and the AdamW step.
//     Each CTA waits (bounded) until every participant has published the
//     bucket for this step, then streams the participants' bf16 gradients
//     straight from their HBM over NVLink (P2P loads, summed in a fixed
//     replica order so all replicas compute bit-identical updates), applies
//     AdamW to the fp32 master/moments and writes the next-generation state
//     and bf16 parameters.  Replaces the reference's per-bucket
//     manager.allreduce + optimizer.step (shift_full/train.py:420-474,574).
// K10 peer_copy: SM-driven copy of a peer's state range into local buffers
//     (live state transfer for heal / handoff).
// Plus reduce-scatter / all-gather helpers for tensor parallelism.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "xchg.h"

namespace sb {
namespace coll {

constexpr int kMaxSrc = 8;

struct SrcPtrs {
  const __nv_bfloat16* p[kMaxSrc];
};
struct FlagPtrs {
  const int* p[kMaxSrc];
};

struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale;
};

// Wait (one thread per CTA) until every peer flag >= target.
__device__ bool cta_wait_flags(const FlagPtrs& f, int n, int target, int* status, uint64_t timeout_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int i = 0; i < n; ++i) {
      if (f.p[i] == nullptr) continue;
      if (!wait_flag_ge(f.p[i], target, status, timeout_ns)) {
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

// Per-step scalars live in device memory so that a captured CUDA graph replays
// correctly every step: sdev[0] = step tag (int), sdev[1..3] = lr, 1 - beta1^t,
// sqrt(1 - beta2^t) (float bits).
SB_DEVICE void load_step(const int* sdev, int& tag, AdamHyper& a) {
  tag = sdev[0];
  a.lr = __int_as_float(sdev[1]);
  a.bc1 = __int_as_float(sdev[2]);
  a.bc2_sqrt = __int_as_float(sdev[3]);
}

// NS: compile-time bound on the number of sources (registers scale with it).
// With one source (the two-phase form's local reduced buffer, or a replica
// alone) loads go through L2 only; with several, the sources are peers'
// memory and are read as volatile (never from a stale cache line).
template <int NS>
__global__ void __launch_bounds__(256, NS <= 2 ? 3 : 2)
fused_reduce_adamw_kernel(SrcPtrs src, int n_src, FlagPtrs flags, int n_flags, const int* __restrict__ sdev,
                          const float* __restrict__ master, const float* __restrict__ m_in,
                          const float* __restrict__ v_in, float* __restrict__ master_out, float* __restrict__ m_out,
                          float* __restrict__ v_out, __nv_bfloat16* __restrict__ param_out, long n, AdamHyper a,
                          int* __restrict__ nonfinite, int* __restrict__ status, uint64_t timeout_ns) {
  int target;
  load_step(sdev, target, a);
  if (n_flags > 0 && !cta_wait_flags(flags, n_flags, target, status, timeout_ns)) return;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x * 8;
  bool bad = false;
  for (long i = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += stride) {
    if (i + 8 <= n) {
      float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // issue all peer loads first (they travel over NVLink), then reduce in order
      bf16x8 raw[NS];
#pragma unroll
      for (int s = 0; s < NS; ++s)
        if (s < n_src) {
          const uint4 u = NS == 1 ? __ldcg(reinterpret_cast<const uint4*>(src.p[s] + i))
                                  : __ldcv(reinterpret_cast<const uint4*>(src.p[s] + i));
          raw[s].w[0] = u.x; raw[s].w[1] = u.y; raw[s].w[2] = u.z; raw[s].w[3] = u.w;
        }
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        if (s < n_src) {
          float f[8];
          bf16x8_to_float(raw[s], f);
#pragma unroll
          for (int q = 0; q < 8; ++q) g[q] += f[q];
        }
      }
      float p[8], m[8], v[8];
      *reinterpret_cast<float4*>(p) = *reinterpret_cast<const float4*>(master + i);
      *reinterpret_cast<float4*>(p + 4) = *reinterpret_cast<const float4*>(master + i + 4);
      *reinterpret_cast<float4*>(m) = *reinterpret_cast<const float4*>(m_in + i);
      *reinterpret_cast<float4*>(m + 4) = *reinterpret_cast<const float4*>(m_in + i + 4);
      *reinterpret_cast<float4*>(v) = *reinterpret_cast<const float4*>(v_in + i);
      *reinterpret_cast<float4*>(v + 4) = *reinterpret_cast<const float4*>(v_in + i + 4);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float gq = g[q] * a.grad_scale;
        bad |= !isfinite(gq);
        p[q] = p[q] * (1.f - a.lr * a.wd);
        m[q] = m[q] + (gq - m[q]) * (1.f - a.beta1);
        v[q] = v[q] * a.beta2 + (1.f - a.beta2) * gq * gq;
        const float denom = sqrtf(v[q]) / a.bc2_sqrt + a.eps;
        p[q] = p[q] - (a.lr / a.bc1) * (m[q] / denom);
      }
      *reinterpret_cast<float4*>(master_out + i) = *reinterpret_cast<float4*>(p);
      *reinterpret_cast<float4*>(master_out + i + 4) = *reinterpret_cast<float4*>(p + 4);
      *reinterpret_cast<float4*>(m_out + i) = *reinterpret_cast<float4*>(m);
      *reinterpret_cast<float4*>(m_out + i + 4) = *reinterpret_cast<float4*>(m + 4);
      *reinterpret_cast<float4*>(v_out + i) = *reinterpret_cast<float4*>(v);
      *reinterpret_cast<float4*>(v_out + i + 4) = *reinterpret_cast<float4*>(v + 4);
      *reinterpret_cast<bf16x8*>(param_out + i) = float_to_bf16x8(p);
    } else {
      for (long j = i; j < n; ++j) {
        float g = 0.f;
        for (int s = 0; s < n_src; ++s) g += __bfloat162float(src.p[s][j]);
        g *= a.grad_scale;
        bad |= !isfinite(g);
        float p = master[j] * (1.f - a.lr * a.wd);
        const float m = m_in[j] + (g - m_in[j]) * (1.f - a.beta1);
        const float v = v_in[j] * a.beta2 + (1.f - a.beta2) * g * g;
        p = p - (a.lr / a.bc1) * (m / (sqrtf(v) / a.bc2_sqrt + a.eps));
        master_out[j] = p;
        m_out[j] = m;
        v_out[j] = v;
        param_out[j] = __float2bfloat16(p);
      }
    }
  }
  if (bad && nonfinite) atomicOr(nonfinite, 1);
}

// ---------------------------------------------------------------------------
// K1, two-phase form (reduce-scatter + all-gather over peer memory, then a
// local AdamW).  Phase A: the CTA waits for every source's ready flag, sums
// this rank's slice of the bucket over all sources in fixed source order
// (fp32), scales it, rounds to bf16 and stores the reduced slice into every
// member's reduced-gradient buffer (P2P stores).  Phase B: after every
// member's slice has landed (slice flags), AdamW reads the reduced gradient
// from local HBM.  Per rank the NVLink traffic is ~(R-1)/R of the bucket in
// each direction instead of (R-1) full buckets read.
// ---------------------------------------------------------------------------
struct DstPtrs {
  __nv_bfloat16* p[kMaxSrc];
};

template <int NS>
__global__ void __launch_bounds__(256)
reduce_slice_scatter_kernel(SrcPtrs src, int n_src, DstPtrs dst, int n_dst, long lo, long hi, FlagPtrs flags,
                            int n_flags, const int* __restrict__ sdev, float scale, int* __restrict__ status,
                            uint64_t timeout_ns) {
  const int target = sdev[0];
  if (n_flags > 0 && !cta_wait_flags(flags, n_flags, target, status, timeout_ns)) return;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x * 8;
  for (long i = lo + (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < hi; i += stride) {
    if (i + 8 <= hi) {
      bf16x8 raw[NS];
#pragma unroll
      for (int s = 0; s < NS; ++s)
        if (s < n_src) {
          const uint4 u = __ldcv(reinterpret_cast<const uint4*>(src.p[s] + i));
          raw[s].w[0] = u.x; raw[s].w[1] = u.y; raw[s].w[2] = u.z; raw[s].w[3] = u.w;
        }
      float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < NS; ++s)
        if (s < n_src) {
          float f[8];
          bf16x8_to_float(raw[s], f);
#pragma unroll
          for (int q = 0; q < 8; ++q) g[q] += f[q];
        }
#pragma unroll
      for (int q = 0; q < 8; ++q) g[q] *= scale;
      const bf16x8 out = float_to_bf16x8(g);
#pragma unroll
      for (int d = 0; d < kMaxSrc; ++d)
        if (d < n_dst) *reinterpret_cast<bf16x8*>(dst.p[d] + i) = out;
    } else {
      for (long j = i; j < hi; ++j) {
        float g = 0.f;
        for (int s = 0; s < n_src; ++s) g += __bfloat162float(src.p[s][j]);
        const __nv_bfloat16 o = __float2bfloat16(g * scale);
        for (int d = 0; d < n_dst; ++d) dst.p[d][j] = o;
      }
    }
  }
  // publish the remote stores (one cumulative system fence per CTA)
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
}

// ---------------------------------------------------------------------------
// flag = step tag + delta
__global__ void flag_set_kernel(int* flag, const int* __restrict__ sdev, int delta) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    __threadfence_system();
    st_release_sys(flag, sdev[0] + delta);
  }
}

// wait until every flag >= step tag + delta
__global__ void flag_wait_kernel(FlagPtrs f, int n, const int* __restrict__ sdev, int delta, int* status,
                                 uint64_t timeout_ns) {
  const int target = sdev[0] + delta;
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    for (int i = 0; i < n; ++i) {
      if (f.p[i] == nullptr) continue;
      if (!wait_flag_ge(f.p[i], target, status, timeout_ns)) break;
    }
  }
}

// out[i] = src[i] for a peer (or local) range, 16-byte vectors.  K10.
__global__ void peer_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long n16) {
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride) dst[i] = src[i];
}

// Copy with tensor-parallel exchange: dst (local, optional) and xc.peer_out
// (a peer's gather buffer, optional) both receive src; optional wait before
// and signal after.  Used where the producer of a gathered operand is not a
// kernel of ours (e.g. a pipeline receive).  Sizes in 16-byte units.
__global__ void xcopy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long n16, Xchg xc,
                             int* status) {
  if (!xchg_wait_cta(xc, status)) return;
  uint4* peer = reinterpret_cast<uint4*>(xc.peer_out);
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = src[i];
    if (dst != nullptr) dst[i] = v;
    if (peer != nullptr) peer[i] = v;
  }
  xchg_signal(xc);
}


// ---------------------------------------------------------------------------
// Deterministic 64-bit fingerprint of a byte range (FNV-1a over 32-bit words):
// thread t of block b hashes words [chunk*(b*T+t), +chunk); the block folds its
// threads' hashes in thread order, the host folds block hashes in block order.
// Equal bytes give equal fingerprints; used for exact-state audits on GPU.
// ---------------------------------------------------------------------------
constexpr unsigned long long kFnvOffset = 1469598103934665603ull;
constexpr unsigned long long kFnvPrime = 1099511628211ull;

__device__ __forceinline__ unsigned long long fnv_word(unsigned long long h, uint32_t w) {
  return (h ^ w) * kFnvPrime;
}

__global__ void fingerprint_kernel(const uint32_t* __restrict__ words, long n, long chunk,
                                   unsigned long long* __restrict__ out) {
  __shared__ unsigned long long th[256];
  const long t = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  unsigned long long h = kFnvOffset;
  const long b0 = t * chunk, b1 = min(n, b0 + chunk);
  for (long i = b0; i < b1; ++i) h = fnv_word(h, words[i]);
  th[threadIdx.x] = h;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = kFnvOffset;
    for (int i = 0; i < static_cast<int>(blockDim.x); ++i) {
      s = fnv_word(s, static_cast<uint32_t>(th[i]));
      s = fnv_word(s, static_cast<uint32_t>(th[i] >> 32));
    }
    out[blockIdx.x] = s;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int sm_count() {
  int dev, n;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Symmetric (IPC-exportable) allocation owned by the caller's tensor.
at::Tensor sym_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(ptr, {nbytes}, [](void* p) { cudaFree(p); }, opts);
}

// 64-byte IPC handle of the allocation that starts at t.data_ptr().
at::Tensor ipc_handle(const at::Tensor& t) {
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, t.data_ptr()));
  auto out = at::empty({static_cast<long>(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

// Map a peer allocation on the current device; unmapped when the tensor dies.
at::Tensor ipc_open(const at::Tensor& handle, int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.numel() == static_cast<long>(sizeof(h)), "ipc_open: bad handle size");
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(ptr, {nbytes}, [](void* p) { cudaIpcCloseMemHandle(p); }, opts);
}

static FlagPtrs make_flags(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(ptrs.size() <= static_cast<size_t>(kMaxSrc), "at most 8 peer flags");
  FlagPtrs f{};
  for (size_t i = 0; i < ptrs.size(); ++i) f.p[i] = reinterpret_cast<const int*>(ptrs[i]);
  return f;
}

void check_step_dev(const at::Tensor& step_dev, const at::Tensor& like) {
  TORCH_CHECK(step_dev.is_cuda() && step_dev.scalar_type() == at::kInt && step_dev.numel() >= 4 &&
                  step_dev.device() == like.device(),
              "step_dev: int32[>=4] on the parameter's device");
}

// K1.  grad_ptrs: device addresses (local or IPC-mapped) of the bucket's
// gradient in each participant, in replica order.  flag_ptrs: addresses of
// the participants' ready flags for this bucket; target: the step tag.
void fused_reduce_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& flag_ptrs,
                        const at::Tensor& step_dev, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v,
                        at::Tensor& master_out, at::Tensor& m_out, at::Tensor& v_out, at::Tensor& param_out,
                        double beta1, double beta2, double eps, double wd, double grad_scale,
                        const at::Tensor& nonfinite, const at::Tensor& status, double timeout_s,
                        int64_t blocks_per_sm) {
  check_step_dev(step_dev, master);
  TORCH_CHECK(!grad_ptrs.empty() && grad_ptrs.size() <= static_cast<size_t>(kMaxSrc), "1..8 gradient sources");
  const at::cuda::CUDAGuard guard(master.device());
  SrcPtrs src{};
  for (size_t i = 0; i < grad_ptrs.size(); ++i) src.p[i] = reinterpret_cast<const __nv_bfloat16*>(grad_ptrs[i]);
  FlagPtrs f = make_flags(flag_ptrs);
  AdamHyper a;
  a.lr = 0.f;  // lr and bias corrections come from step_dev
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = 1.f;
  a.bc2_sqrt = 1.f;
  a.grad_scale = static_cast<float>(grad_scale);
  const long n = master.numel();
  if (n == 0) return;
  // blocks_per_sm <= 0: the whole GPU (8 per SM, grid-stride).  A small value
  // (1) leaves room on every SM for the compute kernels the reduction runs
  // beside during backward: its blocks co-reside with them instead of
  // holding every SM until the bucket is done.
  const long per_sm = blocks_per_sm > 0 ? blocks_per_sm : 8;
  const long blocks = std::min<long>((n / 8 + 255) / 256 + 1, static_cast<long>(sm_count()) * per_sm);
  const int ns = static_cast<int>(grad_ptrs.size());
#define SB_K1(NS)                                                                                              \
  fused_reduce_adamw_kernel<NS><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(                          \
      src, ns, f, static_cast<int>(flag_ptrs.size()), step_dev.data_ptr<int>(), master.data_ptr<float>(),       \
      m.data_ptr<float>(), v.data_ptr<float>(), master_out.data_ptr<float>(), m_out.data_ptr<float>(),          \
      v_out.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(param_out.data_ptr()), n, a,                     \
      nonfinite.data_ptr<int>(), status.data_ptr<int>(), static_cast<uint64_t>(timeout_s * 1e9))
  if (ns == 1) SB_K1(1);
  else if (ns == 2) SB_K1(2);
  else if (ns <= 4) SB_K1(4);
  else SB_K1(8);
#undef SB_K1
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Phase A of the two-phase K1 (see reduce_slice_scatter_kernel).  Ranges are
// element offsets relative to the given base pointers.
void reduce_slice_scatter(const std::vector<int64_t>& src_ptrs, const std::vector<int64_t>& dst_ptrs, int64_t lo,
                          int64_t hi, const std::vector<int64_t>& flag_ptrs, const at::Tensor& step_dev,
                          double scale, const at::Tensor& status, double timeout_s, int64_t blocks_per_sm) {
  TORCH_CHECK(!src_ptrs.empty() && src_ptrs.size() <= static_cast<size_t>(kMaxSrc), "1..8 sources");
  TORCH_CHECK(!dst_ptrs.empty() && dst_ptrs.size() <= static_cast<size_t>(kMaxSrc), "1..8 destinations");
  if (hi <= lo) return;
  SrcPtrs s{};
  for (size_t i = 0; i < src_ptrs.size(); ++i) s.p[i] = reinterpret_cast<const __nv_bfloat16*>(src_ptrs[i]);
  DstPtrs d{};
  for (size_t i = 0; i < dst_ptrs.size(); ++i) d.p[i] = reinterpret_cast<__nv_bfloat16*>(dst_ptrs[i]);
  const long n = hi - lo;
  const long per_sm = blocks_per_sm > 0 ? blocks_per_sm : 4;
  const long blocks = std::max<long>(1, std::min<long>((n / 8 + 255) / 256 + 1, static_cast<long>(sm_count()) * per_sm));
  const int ns = static_cast<int>(src_ptrs.size());
#define SB_RS(NS)                                                                                           \
  reduce_slice_scatter_kernel<NS><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(                     \
      s, ns, d, static_cast<int>(dst_ptrs.size()), lo, hi, make_flags(flag_ptrs),                           \
      static_cast<int>(flag_ptrs.size()), step_dev.data_ptr<int>(), static_cast<float>(scale),              \
      status.data_ptr<int>(), static_cast<uint64_t>(timeout_s * 1e9))
  if (ns <= 2) SB_RS(2);
  else if (ns <= 4) SB_RS(4);
  else SB_RS(8);
#undef SB_RS
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// flag := step_dev[0] + delta (release, system scope)
void flag_set(int64_t flag_ptr, const at::Tensor& step_dev, int64_t delta) {
  flag_set_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<int*>(flag_ptr),
                                                                   step_dev.data_ptr<int>(), static_cast<int>(delta));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// bounded wait until every flag >= step_dev[0] + delta
void flag_wait(const std::vector<int64_t>& flag_ptrs, const at::Tensor& step_dev, int64_t delta,
               const at::Tensor& status, double timeout_s) {
  if (flag_ptrs.empty()) return;
  flag_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_flags(flag_ptrs), static_cast<int>(flag_ptrs.size()), step_dev.data_ptr<int>(), static_cast<int>(delta),
      status.data_ptr<int>(), static_cast<uint64_t>(timeout_s * 1e9));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_copy(int64_t src_ptr, int64_t dst_ptr, int64_t nbytes) {
  TORCH_CHECK(nbytes % 16 == 0 && src_ptr % 16 == 0 && dst_ptr % 16 == 0, "peer_copy: 16-byte aligned ranges");
  const long n16 = nbytes / 16;
  if (n16 == 0) return;
  const long blocks = std::min<long>((n16 + 255) / 256, static_cast<long>(sm_count()) * 4);
  peer_copy_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const uint4*>(src_ptr),
                                                                          reinterpret_cast<uint4*>(dst_ptr), n16);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst_ptr may be 0 (only the peer copy); see xcopy_kernel.
void xcopy(int64_t src_ptr, int64_t dst_ptr, int64_t nbytes, const std::vector<int64_t>& xchg,
           const at::Tensor& status) {
  const Xchg xc = xchg_from(xchg);
  TORCH_CHECK(nbytes % 16 == 0 && src_ptr % 16 == 0 && dst_ptr % 16 == 0, "xcopy: 16-byte aligned ranges");
  const long n16 = nbytes / 16;
  const long blocks = std::max<long>(1, std::min<long>((n16 + 255) / 256, static_cast<long>(sm_count()) * 2));
  xcopy_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(src_ptr), reinterpret_cast<uint4*>(dst_ptr), n16, xc, status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fingerprint of a contiguous tensor's bytes (size must be a multiple of 4).
std::string fingerprint(const at::Tensor& t) {
  TORCH_CHECK(t.is_contiguous() && t.is_cuda(), "fingerprint: contiguous CUDA tensor");
  const long nbytes = t.numel() * t.element_size();
  TORCH_CHECK(nbytes % 4 == 0, "fingerprint: byte size must be a multiple of 4");
  const at::cuda::CUDAGuard guard(t.device());
  const long n = nbytes / 4;
  const int threads = 256;
  const long total_threads = 148L * 4 * threads;
  const long chunk = std::max<long>(1, (n + total_threads - 1) / total_threads);
  const long blocks = std::max<long>(1, (n + chunk * threads - 1) / (chunk * threads));
  auto part = at::empty({blocks}, t.options().dtype(at::kLong));
  if (n > 0)
    fingerprint_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const uint32_t*>(t.data_ptr()), n, chunk,
        reinterpret_cast<unsigned long long*>(part.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  auto host = part.cpu();
  unsigned long long s = kFnvOffset;
  const auto* hp = reinterpret_cast<const unsigned long long*>(host.data_ptr());
  for (long i = 0; i < blocks; ++i) {
    s = (s ^ static_cast<uint32_t>(hp[i])) * kFnvPrime;
    s = (s ^ static_cast<uint32_t>(hp[i] >> 32)) * kFnvPrime;
  }
  s = (s ^ static_cast<uint32_t>(nbytes)) * kFnvPrime;
  char buf[32];
  std::snprintf(buf, sizeof(buf), "%016llx", s);
  return std::string(buf);
}


}  // namespace coll
}  // namespace sb
