// Persistent tcgen05 GEMM for sm_100a (dense and grouped / MoE).
//
//   D[m, n] = alpha * sum_k A[m, k] * B[n, k]
//
// Operands are bf16 and staged by TMA into 128-byte-swizzled shared memory;
// the accumulator lives in tensor memory (TMEM) and is read back with
// tcgen05.ld by four epilogue warps.  One elected thread issues every
// tcgen05.mma.  Two TMEM accumulators let the epilogue of tile i overlap the
// main loop of tile i+1.
//
// Warp roles (192 threads):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2..5  epilogue (TMEM lane quarter = warp % 4)
//
// Operand majors:
//   A K-major  : A stored [rows, K] (K contiguous)
//   A MN-major : A stored [K, M]    (M contiguous)      -> D = A^T ...
//   B K-major  : B stored [N, K]
//   B MN-major : B stored [K, N]
//
// Grouping (G >= 1 groups; a dense GEMM is G = 1):
//   kRowGroups : A/D rows are split into segments by offs[0..G]; group g uses
//                B rows [g*N, (g+1)*N) (K-major B) or [g*K, (g+1)*K)
//                (MN-major B).  This is the MoE expert forward / dgrad.
//   kKGroups   : the contraction dim is split into segments by offs[0..G];
//                group g writes D rows [g*M, (g+1)*M).  This is the MoE
//                expert weight gradient.  Segments must be multiples of 64
//                unless G == 1.
//
// All waits are bounded (see common.cuh); on expiry the kernel records a
// status code, drains what it issued, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "gemm_kernel.cuh"
#include "xchg.h"

namespace sb {
namespace gemm {

void dispatch_bn128(bool, bool, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                    const Params&, int, cudaStream_t);
void dispatch_bn192(bool, bool, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                    const Params&, int, cudaStream_t);
void dispatch_bn256(bool, bool, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                    const Params&, int, cudaStream_t);

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "shift_b200: cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// 2D bf16 tensor map over a row-major matrix [rows, cols] with row stride ld
// (elements), box {box_cols, box_rows}; 128-byte swizzle for 64-column
// boxes, 64-byte swizzle for 32-column boxes.
static CUtensorMap make_map(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                            int box_cols = 64) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK(box_cols == 64 || box_cols == 32, "TMA box width");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return m;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// ---------------------------------------------------------------------------
// Split-K for dense weight gradients with few output tiles (e.g. a 1024 x 1024
// weight over 16k tokens is 32 tiles on 148 SMs): the contraction is cut into
// S 64-aligned ranges run as the kernel's k-groups into an fp32 workspace
// [S*M, N], then summed over S in a fixed order (deterministic) into D with
// the requested epilogue.
// ---------------------------------------------------------------------------
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int S, long MN, int epi, void* D) {
  const long i = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= MN) return;
  float4 acc = *reinterpret_cast<const float4*>(ws + i);
  for (int s = 1; s < S; ++s) {
    const float4 v = *reinterpret_cast<const float4*>(ws + static_cast<long>(s) * MN + i);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (epi == kEpiF32 || epi == kEpiAccF32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(D) + i);
    if (epi == kEpiAccF32) {
      const float4 b = *o;
      acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
    }
    *o = acc;
  } else {
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(D) + i);
    if (epi == kEpiAccBF16) {
      const float2 b0 = __bfloat1622float2(o[0]), b1 = __bfloat1622float2(o[1]);
      acc.x += b0.x; acc.y += b0.y; acc.z += b1.x; acc.w += b1.y;
    }
    o[0] = __floats2bfloat162_rn(acc.x, acc.y);
    o[1] = __floats2bfloat162_rn(acc.z, acc.w);
  }
}

// device table of split boundaries, created once per (K, S, device) outside
// graph capture and reused (a capture may not upload host data)
static const at::Tensor* split_offsets(int64_t K, int S, const at::Device& dev) {
  static std::map<std::tuple<int64_t, int, int>, at::Tensor> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(K, S, static_cast<int>(dev.index()));
  auto it = cache.find(key);
  if (it != cache.end()) return &it->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(at::cuda::getCurrentCUDAStream(), &cs);
  if (cs != cudaStreamCaptureStatusNone) return nullptr;
  std::vector<int> o(S + 1);
  for (int s = 0; s <= S; ++s) o[s] = static_cast<int>((K * s / S) / 64 * 64);
  o[S] = static_cast<int>(K);
  auto t = at::tensor(o, at::TensorOptions().dtype(at::kInt)).to(dev);
  return &(cache[key] = t);
}

// Generic entry.  See gemm_sm100.h for argument meaning.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& D2,
          const c10::optional<at::Tensor>& offs, int64_t M, int64_t N, int64_t K, int64_t G, int64_t mode,
          bool a_mn, bool b_mn, int64_t epi, double alpha, int64_t bn, const at::Tensor& status,
          int64_t max_rows_hint, const std::vector<int64_t>& xchg, const std::vector<int64_t>& tp) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  // split-K for a dense k-mode GEMM (weight gradient) that fills few SMs
  if (mode == kKGroups && G == 1 && !offs.has_value() && epi != kEpiSwiGLU && D.is_contiguous() &&
      (xchg.empty() || xchg[2] == 0) && (M * N) % 4 == 0) {
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const int S = static_cast<int>(std::min<int64_t>(num_sms() / std::max<int64_t>(tiles, 1), K / 1024));
    if (S >= 2) {
      const at::Tensor* so = split_offsets(K, S, A.device());
      if (so != nullptr) {
        const at::cuda::CUDAGuard guard(A.device());
        auto ws = at::empty({S * M, N}, A.options().dtype(at::kFloat));
        gemm(A, B, ws, c10::nullopt, *so, M, N, K, S, kKGroups, a_mn, b_mn, kEpiF32, alpha, bn, status,
             max_rows_hint, xchg, tp);
        const long MN = M * N;
        splitk_reduce_kernel<<<static_cast<unsigned>((MN / 4 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
            ws.data_ptr<float>(), S, MN, static_cast<int>(epi), D.data_ptr());
        C10_CUDA_KERNEL_LAUNCH_CHECK();
        return;
      }
    }
  }
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && D.stride(-1) == 1, "gemm: inner dim must be contiguous");
  TORCH_CHECK(G >= 1 && G <= kMaxGroups, "gemm: group count out of range");
  TORCH_CHECK(N % 16 == 0, "gemm: N must be a multiple of 16");
  TORCH_CHECK(bn == 128 || bn == 192 || bn == 256, "gemm: BN must be 128, 192 or 256");
  if (b_mn) TORCH_CHECK(bn % 64 == 0, "gemm: MN-major B needs BN % 64 == 0");
  if (epi == kEpiSwiGLU) {
    TORCH_CHECK(D2.has_value() && N % 32 == 0 && mode == kRowGroups, "gemm: SwiGLU epilogue needs D2, N%32==0");
  }
  if (epi == kEpiSwiGLUBwd) {
    TORCH_CHECK(D2.has_value() && N % 32 == 0 && mode == kRowGroups && D.size(-1) == 2 * N &&
                    D2->size(-1) == 2 * N && D2->stride(-1) == 1,
                "gemm: SwiGLU-backward epilogue needs h [rows, 2N] (D2) and dh [rows, 2N] (D), N % 32 == 0");
  }
  const bool f32_out = (epi == kEpiF32 || epi == kEpiAccF32);
  TORCH_CHECK(D.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm: output dtype does not match epilogue");
  const at::cuda::CUDAGuard guard(A.device());

  // A / B are viewed as 2D row-major matrices
  const int64_t a_rows = A.numel() / A.size(-1), a_cols = A.size(-1), lda = A.dim() >= 2 ? A.stride(-2) : a_cols;
  const int64_t b_rows = B.numel() / B.size(-1), b_cols = B.size(-1), ldb = B.dim() >= 2 ? B.stride(-2) : b_cols;
  CUtensorMap ta = make_map(A.data_ptr(), a_rows, a_cols, lda, a_mn ? 64 : BM);
  CUtensorMap tb = make_map(B.data_ptr(), b_rows, b_cols, ldb, b_mn ? 64 : static_cast<int>(bn));

  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.G = static_cast<int>(G);
  p.mode = static_cast<int>(mode);
  p.epi = static_cast<int>(epi);
  p.offs = offs.has_value() ? offs->data_ptr<int>() : nullptr;
  p.D = D.data_ptr();
  p.ldd = static_cast<int>(D.dim() >= 2 ? D.stride(-2) : D.size(-1));
  p.D2 = D2.has_value() ? D2->data_ptr() : nullptr;
  p.ldd2 = D2.has_value() ? static_cast<int>(D2->dim() >= 2 ? D2->stride(-2) : D2->size(-1)) : 0;
  p.alpha = static_cast<float>(alpha);
  p.status = status.data_ptr<int>();
  // tensor-parallel exchange: xchg (see xchg.h; peer_out = the peer's
  // receive buffer) and tp = [wait_lo, wait_hi, m_rot, peer_lo, peer_hi, d_row_off]
  p.xc = xchg_from(xchg);
  TORCH_CHECK(tp.empty() || tp.size() == 6, "gemm: tp = [wait_lo, wait_hi, m_rot, peer_lo, peer_hi, d_row_off]");
  p.wait_lo = tp.empty() ? 0 : static_cast<int>(tp[0]);
  p.wait_hi = tp.empty() ? 0 : static_cast<int>(tp[1]);
  p.m_rot = tp.empty() ? 0 : static_cast<int>(tp[2]);
  p.peer_lo = tp.empty() ? 0 : static_cast<int>(tp[3]);
  p.peer_hi = tp.empty() ? 0 : static_cast<int>(tp[4]);
  p.d_row_off = tp.empty() ? 0 : static_cast<int>(tp[5]);
  if (p.m_rot != 0) TORCH_CHECK(mode == kRowGroups && G == 1 && p.m_rot > 0, "gemm: m_rot needs a dense row-mode GEMM");
  if (p.xc.peer_out != nullptr) {
    TORCH_CHECK(mode == kRowGroups && p.peer_lo % BM == 0 && p.peer_hi % BM == 0 && epi != kEpiSwiGLU,
                "gemm: peer output rows must be whole 128-row tiles of a row-mode GEMM");
  }
  if (p.xc.wait_flag != nullptr && mode == kKGroups)
    TORCH_CHECK(p.wait_lo % BK == 0 && p.wait_hi % BK == 0, "gemm: k-mode wait range must be 64-aligned");

  // Output through TMA stores (bf16 / SwiGLU epilogues into local memory):
  // D viewed as [d_rows, N] with row stride ldd, D2 as [d_rows, N/2].
  CUtensorMap td, td2;
  std::memset(&td, 0, sizeof(td));
  std::memset(&td2, 0, sizeof(td2));
  p.use_tma_store = 0;
  p.d_rows = 0;
  const int64_t d_rows = D.dim() >= 2 ? D.numel() / D.size(-1) : 1;
  const bool d_dense = D.dim() < 3 || D.is_contiguous();
  if ((epi == kEpiBF16 || epi == kEpiSwiGLU) && d_dense && reinterpret_cast<uintptr_t>(D.data_ptr()) % 16 == 0 &&
      (static_cast<int64_t>(p.ldd) * 2) % 16 == 0 && N % 8 == 0 && d_rows > 0) {
    bool ok = true;
    if (epi == kEpiSwiGLU) {
      ok = reinterpret_cast<uintptr_t>(D2->data_ptr()) % 16 == 0 && (static_cast<int64_t>(p.ldd2) * 2) % 16 == 0 &&
           (N / 2) % 8 == 0;
      if (ok) td2 = make_map(D2->data_ptr(), d_rows, N / 2, p.ldd2, 32, 32);
    }
    if (ok) {
      td = make_map(D.data_ptr(), d_rows, N, p.ldd, 32, 64);
      p.use_tma_store = 1;
      p.d_rows = static_cast<int>(d_rows);
    }
  }

  // Upper bound of tiles for the grid size (the kernel computes the exact count).
  const int64_t tn = (N + bn - 1) / bn;
  int64_t tiles;
  if (mode == kRowGroups) tiles = ((max_rows_hint + BM - 1) / BM + G) * tn;
  else tiles = G * ((M + BM - 1) / BM) * tn;
  const int hint = static_cast<int>(std::min<int64_t>(tiles, 1 << 30));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  if (bn == 256) dispatch_bn256(a_mn, b_mn, ta, tb, td, td2, p, hint, stream);
  else if (bn == 192) dispatch_bn192(a_mn, b_mn, ta, tb, td, td2, p, hint, stream);
  else dispatch_bn128(a_mn, b_mn, ta, tb, td, td2, p, hint, stream);
}

}  // namespace gemm
}  // namespace sb
