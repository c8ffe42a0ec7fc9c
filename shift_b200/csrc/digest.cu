// SHA-256 leaf digests of a device buffer, for state audits that must not
// copy gigabytes of training state to the host.
//
// The buffer is cut into consecutive leaves of `leaf` bytes (the last one may
// be shorter); one thread computes the SHA-256 (FIPS 180-4) of one leaf and
// writes its 32-byte digest.  The host then hashes the concatenated leaf
// digests with SHA-256 (a two-level hash tree), so the audit digest of a 3.5 GB
// shard costs a few milliseconds of GPU time and a 1-2 MB host hash instead of
// a device-to-host copy and a multi-second CPU hash.
//
// The 64 round constants and the 8 initial hash words are passed in by the
// caller (computed exactly from the first 64 primes, as the standard defines
// them) rather than written out here.
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdint>

namespace sb {
namespace digest {

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }
__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// One 64-byte block, big-endian words w[0..15], into state h.
__device__ __forceinline__ void compress(uint32_t h[8], uint32_t w[16], const uint32_t* __restrict__ k) {
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int t = 0; t < 64; ++t) {
    uint32_t wt;
    if (t < 16) {
      wt = w[t];
    } else {
      const uint32_t w15 = w[(t + 1) & 15], w2 = w[(t + 14) & 15];
      const uint32_t s0 = rotr(w15, 7) ^ rotr(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = rotr(w2, 17) ^ rotr(w2, 19) ^ (w2 >> 10);
      wt = w[t & 15] = w[t & 15] + s0 + w[(t + 9) & 15] + s1;
    }
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + k[t] + wt;
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + maj;
    hh = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h[0] += a;
  h[1] += b;
  h[2] += c;
  h[3] += d;
  h[4] += e;
  h[5] += f;
  h[6] += g;
  h[7] += hh;
}

__global__ void __launch_bounds__(128)
sha256_leaves_kernel(const uint8_t* __restrict__ data, int64_t nbytes, int64_t leaf,
                     const uint32_t* __restrict__ consts, uint8_t* __restrict__ out) {
  __shared__ uint32_t k[64 + 8];
  for (int i = threadIdx.x; i < 72; i += blockDim.x) k[i] = consts[i];
  __syncthreads();
  const int64_t nleaves = (nbytes + leaf - 1) / leaf;
  const int64_t li = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (li >= nleaves) return;
  const uint8_t* p = data + li * leaf;
  const int64_t len = nbytes - li * leaf < leaf ? nbytes - li * leaf : leaf;
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = k[64 + i];
  const int64_t full = len / 64;
  const bool aligned = (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  uint32_t w[16];
  for (int64_t blk = 0; blk < full; ++blk) {
    const uint8_t* q = p + blk * 64;
    if (aligned) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 x = reinterpret_cast<const uint4*>(q)[v];
        w[4 * v] = bswap(x.x);
        w[4 * v + 1] = bswap(x.y);
        w[4 * v + 2] = bswap(x.z);
        w[4 * v + 3] = bswap(x.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        w[j] = (uint32_t(q[4 * j]) << 24) | (uint32_t(q[4 * j + 1]) << 16) | (uint32_t(q[4 * j + 2]) << 8) |
               uint32_t(q[4 * j + 3]);
    }
    compress(h, w, k);
  }
  // tail: the remaining bytes, 0x80, zeros, the message length in bits (big-endian 64-bit)
  const int r = static_cast<int>(len - full * 64);
  const uint8_t* q = p + full * 64;
  const uint64_t bits = static_cast<uint64_t>(len) * 8;
  const int nblk = r < 56 ? 1 : 2;
  for (int b = 0; b < nblk; ++b) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      uint32_t word = 0;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int idx = b * 64 + 4 * j + s;
        uint32_t byte;
        if (idx < r) {
          byte = q[idx];
        } else if (idx == r) {
          byte = 0x80;
        } else if (idx >= nblk * 64 - 8) {
          byte = static_cast<uint32_t>(bits >> (8 * (nblk * 64 - 1 - idx))) & 0xff;
        } else {
          byte = 0;
        }
        word = (word << 8) | byte;
      }
      w[j] = word;
    }
    compress(h, w, k);
  }
  uint8_t* o = out + li * 32;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o[4 * i] = h[i] >> 24;
    o[4 * i + 1] = (h[i] >> 16) & 0xff;
    o[4 * i + 2] = (h[i] >> 8) & 0xff;
    o[4 * i + 3] = h[i] & 0xff;
  }
}

// Leaf digests [ceil(nbytes / leaf), 32] (uint8, on the tensor's device) of a
// contiguous tensor's bytes.  consts: uint32[72] = 64 round constants, then
// the 8 initial hash words.
at::Tensor sha256_leaves(const at::Tensor& t, int64_t leaf, const at::Tensor& consts) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "sha256_leaves: contiguous CUDA tensor");
  TORCH_CHECK(consts.is_cuda() && consts.numel() == 72 && consts.scalar_type() == at::kInt, "sha256_leaves: consts");
  TORCH_CHECK(leaf >= 64 && leaf % 64 == 0, "sha256_leaves: leaf must be a positive multiple of 64 bytes");
  const at::cuda::CUDAGuard guard(t.device());
  const int64_t nbytes = t.numel() * t.element_size();
  const int64_t nleaves = nbytes > 0 ? (nbytes + leaf - 1) / leaf : 0;
  auto out = at::empty({nleaves, 32}, t.options().dtype(at::kByte));
  if (nleaves == 0) return out;
  const int threads = 128;
  const int64_t blocks = (nleaves + threads - 1) / threads;
  sha256_leaves_kernel<<<static_cast<unsigned>(blocks), threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint8_t*>(t.data_ptr()), nbytes, leaf,
      reinterpret_cast<const uint32_t*>(consts.data_ptr<int32_t>()), out.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace digest
}  // namespace sb
