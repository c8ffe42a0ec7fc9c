// Allocation-free RMSNorm backward (see noalloc.h).  No counterpart in the
// reference.  The two-phase reduction of the weight gradient keeps its
// per-block partial sums in a fixed file-scope device array instead of a
// per-call buffer, so the entry point never calls cudaMalloc, cudaFree or any
// allocating library routine.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "noalloc.h"

namespace sb {
namespace noalloc {

constexpr int kWarps = 8;
constexpr int kMaxBlocks = 256;
constexpr int kMaxDevices = 64;

// Shared scratch: one row of `hidden` fp32 partial sums per thread block.
static __device__ __align__(256) float g_rmsnorm_scratch[SB_NOALLOC_SCRATCH_FLOATS];

template <int NV, bool kRes>
__global__ void __launch_bounds__(kWarps * 32)
bwd_partial_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                   const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ w,
                   const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                   float* __restrict__ partial, int rows) {
  constexpr int H = NV * 256;
  __shared__ float red[kWarps][H];
  const int lane = threadIdx.x % 32;
  const int wib = threadIdx.x / 32;
  const int warp = blockIdx.x * kWarps + wib;
  const int nwarps = gridDim.x * kWarps;
  float wv[NV][8], acc[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    bf16x8_to_float(reinterpret_cast<const bf16x8*>(w)[i * 32 + lane], wv[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  }
  for (int r = warp; r < rows; r += nwarps) {
    const float rs = rstd[r];
    float xh[NV][8], g[NV][8];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float dv[8];
      bf16x8_to_float(reinterpret_cast<const bf16x8*>(x + static_cast<long>(r) * H)[i * 32 + lane], xh[i]);
      bf16x8_to_float(reinterpret_cast<const bf16x8*>(dy + static_cast<long>(r) * H)[i * 32 + lane], dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[i][j] *= rs;
        g[i][j] = dv[j] * wv[i][j];
        dot += g[i][j] * xh[i][j];
        acc[i][j] += dv[j] * xh[i][j];
      }
    }
    dot = warp_sum(dot) / H;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float o[8], rr[8];
      if (kRes) bf16x8_to_float(reinterpret_cast<const bf16x8*>(dres + static_cast<long>(r) * H)[i * 32 + lane], rr);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rs * (g[i][j] - xh[i][j] * dot) + (kRes ? rr[j] : 0.f);
      reinterpret_cast<bf16x8*>(dx + static_cast<long>(r) * H)[i * 32 + lane] = float_to_bf16x8(o);
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) red[wib][(i * 32 + lane) * 8 + j] = acc[i][j];
  __syncthreads();
  // every block writes its full row of partials (no element is left stale)
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += red[k][c];
    partial[static_cast<long>(blockIdx.x) * H + c] = s;
  }
}

__global__ void reduce_kernel(const float* __restrict__ partial, int nblocks, int cols, float* __restrict__ dw) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += partial[static_cast<long>(b) * cols + c];
  dw[c] = s;
}

// Per-device address of the scratch array, looked up once with that device current.
static std::mutex g_mu;
static float* g_ptr[kMaxDevices] = {};

static float* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_rmsnorm_scratch) != cudaSuccess) return nullptr;
    g_ptr[dev] = static_cast<float*>(p);
  }
  return g_ptr[dev];
}

template <int NV>
static cudaError_t launch(const void* dy, const void* x, const float* rstd, const void* w, const void* dres, void* dx,
                          float* dw, int rows, int blocks, float* scratch, cudaStream_t s) {
  constexpr int H = NV * 256;
  auto* dyp = static_cast<const __nv_bfloat16*>(dy);
  auto* xp = static_cast<const __nv_bfloat16*>(x);
  auto* wp = static_cast<const __nv_bfloat16*>(w);
  auto* rp = static_cast<const __nv_bfloat16*>(dres);
  auto* dxp = static_cast<__nv_bfloat16*>(dx);
  if (dres) bwd_partial_kernel<NV, true><<<blocks, kWarps * 32, 0, s>>>(dyp, xp, rstd, wp, rp, dxp, scratch, rows);
  else bwd_partial_kernel<NV, false><<<blocks, kWarps * 32, 0, s>>>(dyp, xp, rstd, wp, rp, dxp, scratch, rows);
  reduce_kernel<<<(H + 255) / 256, 256, 0, s>>>(scratch, blocks, H, dw);
  return cudaGetLastError();
}

}  // namespace noalloc
}  // namespace sb

extern "C" __attribute__((visibility("default"))) int sb_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const float* rstd, const void* w, const void* dres, void* dx, float* dw, int rows,
    int hidden, void* stream) {
  using namespace sb::noalloc;
  if (rows < 0 || (hidden != 256 && hidden != 512 && hidden != 1024)) return 1;
  // The kernels move bf16 rows as 16-byte vectors and fp32 values one at a
  // time: refuse, before any launch, a pointer the hardware cannot access
  // that way (a misaligned vector access faults the whole context).
  auto aligned = [](const void* p, uintptr_t a) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  if (!aligned(dy, 16) || !aligned(x, 16) || !aligned(w, 16) || !aligned(dx, 16) ||
      (dres != nullptr && !aligned(dres, 16)) || !aligned(rstd, 4) || !aligned(dw, 4))
    return 4;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int blocks = (rows + kWarps - 1) / kWarps;
  if (blocks > sms) blocks = sms;
  if (blocks > kMaxBlocks) blocks = kMaxBlocks;
  if (blocks < 1) blocks = 1;
  if (static_cast<long>(blocks) * hidden > SB_NOALLOC_SCRATCH_FLOATS) return 1;
  float* scratch = scratch_for_current_device();
  if (scratch == nullptr) return 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (hidden) {
    case 256: e = launch<1>(dy, x, rstd, w, dres, dx, dw, rows, blocks, scratch, s); break;
    case 512: e = launch<2>(dy, x, rstd, w, dres, dx, dw, rows, blocks, scratch, s); break;
    default: e = launch<4>(dy, x, rstd, w, dres, dx, dw, rows, blocks, scratch, s); break;
  }
  return e == cudaSuccess ? 0 : 3;
}
