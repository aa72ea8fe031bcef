// Dense tensor-core throughput of this GPU for the two MMA kinds the fused
// attention kernel issues (kind::i8 for INT8 QK^T, kind::f8f6f4 for E4M3
// P.V): the measured denominator of the kernel's roofline.
//
// One CTA per SM.  Both operands sit in shared memory (K-major, 128-byte
// swizzle) filled with pseudo-random bytes (E4M3 bytes without NaN
// patterns), so the arithmetic and its power draw resemble real data.  Each
// issuing warp issues ``iters`` rounds of four M=128 x N x K=32 MMAs into
// its tensor-memory accumulator, commits once and waits (bounded).
// Thread 0 records clock64 at the start, after the last issue and after
// completion, so issue cost per instruction and execution rate can be read
// separately from the host-side event time.  With ``a_tmem`` the A operand
// is read from tensor memory instead (the form the attention kernel's P.V
// uses).  ``issuers`` warps (1-4) issue concurrently, each into its own
// accumulator, which shows how much of an MMA's cost is the issuing warp's.
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kPeakA = 128 * 128;   // A: 128 rows x 128 bytes
constexpr int kPeakB = 256 * 128;   // B: up to 256 rows x 128 bytes

__global__ void __launch_bounds__(128, 1)
    tensor_peak_kernel(int kind, int n, int64_t iters, int a_tmem, int issuers, unsigned long long* stamps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + kPeakA + kPeakB);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + kPeakA + kPeakB + 8);
  // pseudo-random operand bytes (a 32-bit LCG per word); E4M3 NaN is S.1111.111, cleared by & 0x77
  for (int i = threadIdx.x; i < (kPeakA + kPeakB) / 4; i += blockDim.x) {
    uint32_t h = static_cast<uint32_t>(i) * 2654435761u + 12345u * (blockIdx.x + 1);
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    reinterpret_cast<uint32_t*>(smem)[i] = kind == 1 ? (h & 0x77777777u) : h;
  }
  if (threadIdx.x == 0) {
    mbar_init(done, issuers);
    fence_barrier_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // operands visible to the MMA
  if (threadIdx.x < 32) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const int warp = threadIdx.x >> 5;
  if (warp < issuers) {
    // ``issuers`` warps issue concurrently, warp w into its own accumulator at
    // column w * ceil(n/32)*32; each loop runs in the whole warp (warp-uniform
    // descriptor arithmetic) and one elected lane issues each MMA
    const uint32_t idesc = kind == 1 ? idesc_make(1, 0, 0, 128, static_cast<uint32_t>(n))    // f32 <- e4m3 x e4m3
                                     : idesc_make(2, 1, 1, 128, static_cast<uint32_t>(n));   // s32 <- s8 x s8
    const uint64_t ad = smem_desc_sw128(smem_u32(smem));
    const uint64_t bd = smem_desc_sw128(smem_u32(smem + kPeakA));
    const uint32_t d = tmem + static_cast<uint32_t>(warp) * ((static_cast<uint32_t>(n) + 31u) & ~31u);
    __syncwarp();
    const unsigned long long t0 = clock64();
    for (int64_t it = 0; it < iters; ++it) {
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          if (a_tmem) {
            // A from tensor memory (columns [448, 480): whatever they hold)
            if (kind == 1) mma_f8_ts(d, tmem + 448 + kk * 8, bd + 2 * kk, idesc, 1u);
            else mma_i8_ts(d, tmem + 448 + kk * 8, bd + 2 * kk, idesc, 1u);
          } else {
            if (kind == 1) mma_f8_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, 1u);
            else mma_i8_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, 1u);
          }
        }
      }
      __syncwarp();
    }
    const unsigned long long t1 = clock64();
    if (elect_one()) mma_commit(done);
    __syncwarp();
    const bool ok = mbar_wait_warp(done, 0, kErrTimeoutMma);
    const unsigned long long t2 = clock64();
    if (stamps && threadIdx.x == 0) {
      stamps[3 * blockIdx.x + 0] = t1 - t0;
      stamps[3 * blockIdx.x + 1] = t2 - t0;
      stamps[3 * blockIdx.x + 2] = ok ? 1ull : 0ull;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int tensor_peak(int kind, int n, int64_t iters, int ctas, int a_tmem, int issuers, unsigned long long* stamps,
                cudaStream_t st) {
  const int smem = kPeakA + kPeakB + 16 + 1024;
  if (cudaFuncSetAttribute(tensor_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return VC_ERR_LAUNCH;
  tensor_peak_kernel<<<ctas, 128, smem, st>>>(kind, n, iters, a_tmem, issuers, stamps);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

cudaError_t tensor_peak_error_word(uint32_t* code, bool clear) { return read_tu_error_word(code, clear); }

}  // namespace vcb
