// Shared device helpers for the sm_100a VC-attention library.
//
// Everything here is hand-written PTX or plain CUDA C++ for sm_100a:
// input element loads, the device error word, mbarriers with bounded waits,
// TMA tile loads (never multicast) and the tcgen05 (tensor memory / UMMA)
// instructions used by the fused attention kernel.
#pragma once
#include <climits>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include "vc_b200.h"

namespace vcb {

// ---------------------------------------------------------------------------
// Device error word.  Kernels never trap: a wait that exceeds its budget or a
// violated device-side invariant ORs a bit in here and the kernel returns.
// Each translation unit has its own copy (the library is built without
// relocatable device code so that ptxas honours setmaxnreg); the units that
// raise errors export a host reader, combined by vc_error_read().
// ---------------------------------------------------------------------------
static __device__ uint32_t g_error_word = 0;

enum : uint32_t {
  kErrTimeoutTma = 1u << 0,
  kErrTimeoutMma = 1u << 1,
  kErrTimeoutSoftmax = 1u << 2,
  kErrTimeoutCorrection = 1u << 3,
  kErrTimeoutProducer = 1u << 4,
  kErrTmemAlloc = 1u << 5,
  kErrBadArgument = 1u << 6,
  kErrBadIndex = 1u << 7,     // a permutation entry outside [0, S): that row read as zeros
  kErrTimeoutSelfTest = 1u << 8,   // vc_selftest_wait_timeout: its wait gave up, as intended
};

__device__ __forceinline__ void raise_error(uint32_t bits) { atomicOr(&g_error_word, bits); }

// Host: copy (and optionally clear) this translation unit's error word on the
// current device.  Synchronous.
static inline cudaError_t read_tu_error_word(uint32_t* code, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_error_word, sizeof(uint32_t));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof(uint32_t));
  }
  return e;
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// ---------------------------------------------------------------------------
// Element loads of the three accepted input types as FP32.
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<VC_DTYPE_F16> { using T = __half; };
template <> struct Elem<VC_DTYPE_BF16> { using T = __nv_bfloat16; };
template <> struct Elem<VC_DTYPE_F32> { using T = float; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// Round an FP32 value to the storage type and back (exact torch elementwise
// semantics for ``a - b`` on half/bfloat16 tensors: FP32 op, one RN rounding).
__device__ __forceinline__ float round_as(float x, float*) { return x; }
__device__ __forceinline__ float round_as(float x, __half*) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float round_as(float x, __nv_bfloat16*) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Load N consecutive elements (N*sizeof(T) is 8, 16 or 32 bytes) as FP32.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  static_assert((N * sizeof(T)) % 8 == 0, "vector loads of 8/16/32 bytes");
  constexpr int kWords = N * sizeof(T) / 4;
  uint32_t w[kWords];
  if constexpr (kWords % 4 == 0) {
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + i);
      w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kWords / 2; ++i) {
      uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + i);
      w[2 * i] = u.x; w[2 * i + 1] = u.y;
    }
  }
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = __uint_as_float(w[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      T lo, hi;
      uint16_t l16 = static_cast<uint16_t>(w[i] & 0xFFFFu), h16 = static_cast<uint16_t>(w[i] >> 16);
      memcpy(&lo, &l16, 2);
      memcpy(&hi, &h16, 2);
      out[2 * i] = to_f32(lo);
      out[2 * i + 1] = to_f32(hi);
    }
  }
}

// E4M3 pair conversion: cvt.rn.satfinite.e4m3x2.f32 packs (hi, lo) into 16 bits,
// ``lo`` in the low byte.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// ---------------------------------------------------------------------------
// Shared-memory addresses and mbarriers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about ``ns`` nanoseconds pass, issuing nothing meanwhile.
__device__ __forceinline__ bool mbar_try_wait_for(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after about two seconds of wall time (far beyond
// any legitimate wait inside one launch), records ``err`` and returns false;
// callers then unwind.  The budget is wall time, so it holds whether the
// hardware honours the suspend hint or returns early.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;
constexpr uint32_t kSuspendHintNs = 100000;
// mbar_wait with an explicit budget (the self-test uses a short one).
__device__ __forceinline__ bool mbar_wait_budget(uint64_t* bar, uint32_t parity, uint32_t err, uint64_t budget_ns) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint32_t hint = budget_ns < kSuspendHintNs ? static_cast<uint32_t>(budget_ns) : kSuspendHintNs;
  for (;;) {
    if (mbar_try_wait_for(a, parity, hint)) return true;
    if (globaltimer_ns() - t0 > budget_ns) break;
  }
  raise_error(err);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t err) {
  return mbar_wait_budget(bar, parity, err, kWaitBudgetNs);
}

// Non-blocking test of a phase (mbarrier.test_wait).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait by polling (no suspension, so no wake-up latency once the
// phase completes; costs issue slots while it waits).  Same 2 s budget.
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, uint32_t err) {
  const uint32_t a = smem_u32(bar);
  if (mbar_test(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(a, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) break;
  }
  raise_error(err);
  return false;
}
__device__ __forceinline__ bool mbar_spin_warp(uint64_t* bar, uint32_t parity, uint32_t err) {
  const bool ok = mbar_spin(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform bounded wait: every lane polls, the warp agrees on the result
// and reconverges (required before .sync.aligned tcgen05 instructions).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint32_t err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), plain CTA-local loads only -- no multicast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Untiled bulk copy global -> shared (CTA-local, no multicast); both addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 16-byte asynchronous copy global -> shared; src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
// The mbarrier's current phase also waits for every cp.async this thread has
// issued so far (pending count +1 now, one arrival when they complete: no net
// change to the expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// N values of type T (16-byte aligned, N*sizeof(T) a multiple of 8) from
// shared memory, widened to FP32.
template <typename T, int N>
__device__ __forceinline__ void load_vec_smem(const T* p, float (&out)[N]) {
  static_assert((N * sizeof(T)) % 8 == 0, "8/16/32-byte vectors");
  constexpr int kWords = N * sizeof(T) / 4;
  uint32_t w[kWords];
  const uint32_t a = smem_u32(p);
  if constexpr (kWords % 4 == 0) {
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i)
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(w[4 * i]), "=r"(w[4 * i + 1]), "=r"(w[4 * i + 2]), "=r"(w[4 * i + 3])
                   : "r"(a + 16 * i));
  } else {
#pragma unroll
    for (int i = 0; i < kWords / 2; ++i)
      asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(w[2 * i]), "=r"(w[2 * i + 1]) : "r"(a + 8 * i));
  }
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = __uint_as_float(w[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      T lo, hi;
      uint16_t l16 = static_cast<uint16_t>(w[i] & 0xFFFFu), h16 = static_cast<uint16_t>(w[i] >> 16);
      memcpy(&lo, &l16, 2);
      memcpy(&hi, &h16, 2);
      out[2 * i] = to_f32(lo);
      out[2 * i + 1] = to_f32(hi);
    }
  }
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, commit, loads/stores, fences.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc], kind::i8 (s32 accumulate).
__device__ __forceinline__ void mma_i8_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f8f6f4 (f32 accumulate).
__device__ __forceinline__ void mma_f8_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (f16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// True in exactly one active lane of a converged warp (elect.sync).  MMA
// issue loops run in the whole warp, so descriptor arithmetic stays
// warp-uniform, and elect one lane per instruction.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 rx;\n .reg .pred px;\n elect.sync rx|px, 0xffffffff;\n selp.b32 %0, 1, 0, px;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::i8 (s32 accumulate).
__device__ __forceinline__ void mma_i8_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f8f6f4 (f32 accumulate).
__device__ __forceinline__ void mma_f8_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16 (f16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on ``bar`` once all previously issued tcgen05 ops of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// wait::ld that also ties register r to the wait, so no use of r is scheduled before it
__device__ __forceinline__ void tmem_wait_ld_reg(uint32_t& r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r) :: "memory");
}
// the same for 32 registers (a second wait::ld with nothing outstanding returns at once)
__device__ __forceinline__ void tmem_wait_ld_tie32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :: "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// UMMA shared-memory matrix descriptor (sm_100 format): K-major operand,
// 128-byte swizzle, rows of 128 bytes grouped by 8 (1024-byte stride).
//   [0,14) start>>4 | [16,30) LBO>>4 | [32,46) SBO>>4 | [46,48) version=1
//   [49,52) base offset | [61,64) layout (2 = 128B swizzle)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                 // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B
  return d;
}

// Same for rows of 64 bytes (64-byte swizzle, 512-byte stride per 8 rows).
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;                 // SWIZZLE_64B
  return d;
}

// K-major operand without swizzle: 8-row x 16-byte core matrices, ``lbo``
// bytes between core matrices along K, ``sbo`` bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version for sm_100
  return d;                                             // layout 0: no swizzle
}

// Packed FP32 pairs (sm_100 f32x2 arithmetic): each half is rounded on its
// own, exactly as the scalar .rn instruction would round it.
__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pk2f(float lo, float hi) { return pk2(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ void up2(uint64_t v, uint32_t& lo, uint32_t& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// UMMA instruction descriptor: dense, K-major A and B, M=128.
//   [4,6) D format (1=f32, 2=s32) | [7,10) A fmt | [10,13) B fmt
//   [17,23) N>>3 | [24,29) M>>4
__host__ __device__ constexpr uint32_t idesc_make(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, uint32_t m, uint32_t n) {
  return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace vcb
