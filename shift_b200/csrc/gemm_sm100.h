// Public interface of the sm_100a tcgen05 GEMM (see gemm_sm100.cu).
#pragma once
#include <torch/extension.h>

namespace sb {
namespace gemm {

enum Mode : int { kRowGroups = 0, kKGroups = 1 };
enum Epilogue : int {
  kEpiBF16 = 0,     // D = bf16(alpha * acc)
  kEpiF32 = 1,      // D = alpha * acc (fp32)
  kEpiAccBF16 = 2,  // D = bf16(D + alpha * acc)
  kEpiAccF32 = 3,   // D += alpha * acc (fp32)
  kEpiSwiGLU = 4,   // D = bf16(acc) (interleaved gate/up), D2 = silu(gate) * up
  kEpiSwiGLUBwd = 5,  // acc = dact [rows, F]; D2 = h (interleaved gate/up, input) -> D = dh [rows, 2F]
};

void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& D, const c10::optional<at::Tensor>& D2,
          const c10::optional<at::Tensor>& offs, int64_t M, int64_t N, int64_t K, int64_t G, int64_t mode,
          bool a_mn, bool b_mn, int64_t epi, double alpha, int64_t bn, const at::Tensor& status,
          int64_t max_rows_hint, const std::vector<int64_t>& xchg, const std::vector<int64_t>& tp);

}  // namespace gemm
}  // namespace sb
