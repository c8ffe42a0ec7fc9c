// Shared device helpers for the sm_100a kernels of shift_b200.
//
// Everything here is written for Blackwell (sm_100a) only: mbarrier pipelines,
// TMA tiled loads (never with cluster multicast), tcgen05 MMA / TMEM access, and
// bounded spin-waits.  Every wait in this library is bounded by the global
// nanosecond timer; on expiry the waiting thread records a status code in a
// caller-provided status word and returns false, so that the kernel can wind
// down (drain its own copies, free TMEM) and the host can read the status.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SB_DEVICE __device__ __forceinline__

namespace sb {

// ---------------------------------------------------------------------------
// Status codes written into the per-launch status word (first error wins).
// ---------------------------------------------------------------------------
enum Status : int {
  kOk = 0,
  kTimeoutPipeline = 1,   // an mbarrier wait inside one CTA ran out
  kTimeoutPeer = 2,       // a wait on a flag written by another GPU ran out
  kBadShape = 3,          // a kernel met a size it was not built for
};

// Host-side check for kernels that move 16-byte vectors: the base address
// (and therefore, with a row length that is a multiple of 8 bf16, every row)
// must be 16-byte aligned, or the vector accesses would fault.
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Debug builds (SHIFT_DEBUG_BOUNDS=1 in the environment of `setup.py build_ext`
// adds -DSHIFT_DEBUG_BOUNDS=1) check the row indices that kernels read from
// data -- routing slots, token ids -- before using them as addresses.  A bad
// index is printed with the source line and the access is skipped (the row
// reads as zeros / is not written); nothing traps, so the context survives and
// the run can be inspected.  Release builds compile the check away.
#if defined(SHIFT_DEBUG_BOUNDS) && SHIFT_DEBUG_BOUNDS
#include <cstdio>
#define SB_IN_RANGE(i, n) ::sb::debug_in_range(static_cast<long long>(i), static_cast<long long>(n), __LINE__)
__device__ __noinline__ inline bool debug_in_range(long long i, long long n, int line) {
  if (i >= 0 && i < n) return true;
  printf("shift_b200 bounds check: line %d: index %lld not in [0, %lld)\n", line, i, n);
  return false;
}
#else
#define SB_IN_RANGE(i, n) true
#endif

SB_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

SB_DEVICE void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Default bound for waits that only depend on work inside the same kernel.
constexpr uint64_t kPipelineTimeoutNs = 4000000000ull;  // 4 s

// ---------------------------------------------------------------------------
// Small math helpers
// ---------------------------------------------------------------------------
SB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

SB_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
SB_DEVICE float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// 16-byte vector of 8 bf16 values.
struct alignas(16) bf16x8 {
  uint32_t w[4];
};
SB_DEVICE void bf16x8_to_float(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p = unpack_bf16x2(v.w[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}
SB_DEVICE bf16x8 float_to_bf16x8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
  return v;
}

// ---------------------------------------------------------------------------
// Shared-memory addressing
// ---------------------------------------------------------------------------
// 16-byte read-only load that the compiler may neither hoist out of a loop
// nor merge with another: for small loop-invariant operands (a norm weight)
// that should come from L1 each time instead of occupying registers.
SB_DEVICE bf16x8 ld_nc_bf16x8(const void* p) {
  bf16x8 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "l"(p));
  return v;
}

SB_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
SB_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
SB_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SB_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
SB_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
SB_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000000;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait for the given parity.  Returns false (and records the status) if
// the barrier did not complete within the bound.
SB_DEVICE bool mbar_wait(uint64_t* bar, uint32_t phase, int* status,
                         uint64_t timeout_ns = kPipelineTimeoutNs) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - start > timeout_ns) {
      record_status(status, kTimeoutPipeline);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast).  Loads complete on an mbarrier with tx-bytes.
// ---------------------------------------------------------------------------
SB_DEVICE void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
SB_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// TMA tiled store smem -> global (bulk-group completion).  x must be a
// multiple of 16 bytes; coordinates are never negative here.
SB_DEVICE void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
SB_DEVICE void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N bulk groups still READ their shared-memory source
template <int N>
SB_DEVICE void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N bulk groups are still in flight (writes performed)
template <int N>
SB_DEVICE void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
SB_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
SB_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory at `dst`.  Must be executed by one whole warp.
SB_DEVICE void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
SB_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SB_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
SB_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SB_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T for kind::f16 (bf16/fp16 inputs, fp32 accumulate).
SB_DEVICE void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T (A operand read from tensor memory).
SB_DEVICE void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
SB_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
SB_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SB_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
SB_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 32 bit, 32 consecutive columns per thread.
SB_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 32 bit store, 16 consecutive columns per thread.
SB_DEVICE void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (sm_100 format)
//   smem descriptor: start>>4 [0,14) | LBO>>4 [16,30) | SBO>>4 [32,46) |
//                    version=1 [46,48) | base offset [49,52) | lbo mode [52] |
//                    layout [61,64): 0 none, 2 = 128B swizzle
//   instruction descriptor (kind::f16): D fmt [4,6) | A fmt [7,10) | B fmt [10,13)
//                    | A major [15] | B major [16] | N>>3 [17,23) | M>>4 [24,29)
// ---------------------------------------------------------------------------
SB_DEVICE uint64_t make_sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// bf16 x bf16 -> fp32, M x N tile, majors: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                                   // D = F32
         | (1u << 7)                                 // A = BF16
         | (1u << 10)                                // B = BF16
         | (static_cast<uint32_t>(a_mn_major) << 15) //
         | (static_cast<uint32_t>(b_mn_major) << 16) //
         | (static_cast<uint32_t>(N >> 3) << 17)     //
         | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// System-scope flag helpers for peer-memory signalling.
// ---------------------------------------------------------------------------
SB_DEVICE void st_release_sys(volatile int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
SB_DEVICE int ld_acquire_sys(const volatile int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until *flag >= target.  Returns false on timeout.
SB_DEVICE bool wait_flag_ge(const volatile int* flag, int target, int* status, uint64_t timeout_ns) {
  if (ld_acquire_sys(flag) >= target) return true;
  // a peer wait of this step already ran out (the host clears the word after
  // every step): the step is lost, so do not spend another full bound here --
  // a dead peer would otherwise cost one timeout per bucket / exchange
  const volatile int* st = reinterpret_cast<const volatile int*>(status);
  if (st != nullptr && *st == kTimeoutPeer) return false;
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys(flag) >= target) return true;
    // the same word is also written from the host (a copy-engine write while
    // this kernel spins) when a peer process is seen to have died, so a wait on
    // a dead peer ends within one poll instead of at the bound
    if (st != nullptr && *st == kTimeoutPeer) return false;
    if (globaltimer_ns() - start > timeout_ns) {
      record_status(status, kTimeoutPeer);
      return false;
    }
    __nanosleep(64);
  }
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange hooks shared by the kernels that produce or consume
// data another GPU of the TP group reads or writes (norms, GEMM epilogues,
// MoE combine, push copies).  Every field is optional (null / 0 = unused).
//   wait_flag : before touching peer-produced data, wait until
//               *wait_flag >= sdev[0] + wait_delta (a flag the peer
//               releases at system scope after its kernel finished)
//   sig_flag  : after the kernel's last store, the last CTA to finish sets
//               *sig_flag = sdev[0] + sig_delta (sig_counter counts CTAs
//               and is reset to 0 by that CTA)
//   peer_out  : a kernel-specific destination in a peer's memory
// sdev is the device step block (sdev[0] = step tag), so that a replayed
// CUDA graph signals and waits with the current step's values.
// ---------------------------------------------------------------------------
struct Xchg {
  const int* wait_flag;
  int wait_delta;
  int* sig_flag;
  int* sig_counter;
  int sig_delta;
  const int* sdev;
  void* peer_out;
};

constexpr uint64_t kPeerWaitNs = 10ull * 1000 * 1000 * 1000;   // 10 s

// Thread 0 of every CTA waits; the CTA barrier then orders every thread's
// later loads after the acquire.  Returns false (status recorded) on timeout.
SB_DEVICE bool xchg_wait_cta(const Xchg& x, int* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = 1;
    if (x.wait_flag != nullptr && !wait_flag_ge(x.wait_flag, x.sdev[0] + x.wait_delta, status, kPeerWaitNs))
      s_ok = 0;
  }
  __syncthreads();
  return s_ok != 0;
}

// Called by EVERY thread of every CTA after its last store of the kernel.
// The CTA barrier orders every thread's stores before thread 0's system-scope
// fence (fences are cumulative), so one fence per CTA publishes them all.
SB_DEVICE void xchg_signal(const Xchg& x) {
  if (x.sig_flag == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int prev = atomicAdd(x.sig_counter, 1);
    if (prev == static_cast<int>(gridDim.x * gridDim.y * gridDim.z) - 1) {
      atomicExch(x.sig_counter, 0);
      __threadfence_system();
      st_release_sys(x.sig_flag, x.sdev[0] + x.sig_delta);
    }
  }
}

}  // namespace sb
