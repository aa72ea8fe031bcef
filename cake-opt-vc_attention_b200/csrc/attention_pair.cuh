// Paired-tile fused attention kernel (ExpCast, channel-scaled V, no block
// means).  Included by attention.cu after attention_fast.cuh (shares helpers).
//
// One CTA owns TWO 128-row Q tiles (x = 0, 1) of the same (batch, head) and
// streams the head's K/V tiles once for both:
//
//   warps 0-3   softmax for Q tile 0 (thread t = row t, whole 128-key rows)
//   warps 4-7   softmax for Q tile 1
//   warp 8      TMA producer (Q tiles once, then the K/V ring)
//   warp 9      tensor-memory allocator + single-thread MMA issuer
//   warps 10-11 idle (complete the third warpgroup for setmaxnreg)
//
// The two softmax warpgroups work on different rows and never synchronise
// with each other, so while one waits for its next scores the other computes:
// per K tile the tensor core runs PV_0(j-1), QK_0(j), PV_1(j-1), QK_1(j).
//
// Tensor memory (512 columns): S_0 [0,128) S_1 [128,256) (s32 scores; the
// ExpCast bytes P_x are written into S_x[0,32) after the row is read),
// O_0 [256,256+D) O_1 [384,384+D) (FP32 output accumulators for the whole K
// loop).  Q tiles are A operands from shared memory.  The ExpCast denominator
// is the exact FP32 sum of the decoded bytes, accumulated per thread as
// sum(as_float(byte << 20)) * 2^120 (subnormal-exact).
#pragma once

constexpr int kPairThreads = 384;
__device__ __forceinline__ uint32_t pcol_s(int x) { return x ? 128u : 0u; }     // S_x column base
__device__ __forceinline__ uint32_t pcol_o(int x) { return x ? 384u : 256u; }   // O_x column base

struct __align__(8) PairBarriers {
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t q_full, s_full[2], p_full[2], o_done[2];
};

template <int D>
struct PairSmem {
  static constexpr int kQ = 128 * D;
  static constexpr int kK = 128 * D;
  static constexpr int kV = D * 128;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + 2 * kQ;
  static constexpr int kOffV = kOffK + kStages * kK;
  static constexpr int kOffBar = kOffV + kStages * kV;
  static constexpr int kOffSlot = kOffBar + int(sizeof(PairBarriers));
  static constexpr int kBytes = kOffSlot + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  if constexpr (D == 128) return smem_desc_sw128(saddr);
  else return smem_desc_sw64(saddr);
}

template <int D, typename OutT>
__global__ void __launch_bounds__(kPairThreads, 1)
    vc_attention_pair_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                             const __grid_constant__ CUtensorMap tmv, Params p) {
  using L = PairSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBarriers* bar = reinterpret_cast<PairBarriers*>(smem + L::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA -> (head, pair of Q tiles); units outside [unit_begin, unit_end) are
  // computed but not stored.
  const int64_t pairs = (p.qtiles + 1) >> 1;
  const int64_t cta = p.pair_begin + blockIdx.x;
  const int64_t hb = cta / pairs;
  const int64_t qt0 = (cta - hb * pairs) * 2;
  const int T = static_cast<int>(p.ktiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
    }
    mbar_init(&bar->q_full, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bar->s_full[x], 1);
      mbar_init(&bar->p_full[x], 128);
      mbar_init(&bar->o_done[x], 1);
    }
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    setmaxnreg_dec<56>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- producer
      mbar_expect_tx(&bar->q_full, 2 * L::kQ);
      tma_load_3d(smem + L::kOffQ, &tmq, &bar->q_full, 0, static_cast<int>(qt0 * 128), static_cast<int>(hb));
      tma_load_3d(smem + L::kOffQ + L::kQ, &tmq, &bar->q_full, 0, static_cast<int>(qt0 * 128 + 128),
                  static_cast<int>(hb));
      for (int j = 0; j < T; ++j) {
        const int s = j % kStages;
        const uint32_t ph = ((j / kStages) & 1) ^ 1;
        if (j >= kStages && !mbar_wait(&bar->k_empty[s], ph, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->k_full[s], L::kK);
        tma_load_3d(smem + L::kOffK + s * L::kK, &tmk, &bar->k_full[s], 0, j * 128, static_cast<int>(hb));
        if (j >= kStages && !mbar_wait(&bar->v_empty[s], ph, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->v_full[s], L::kV);
        tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(hb));
      }
    } else if (warp == 9 && lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_qk = idesc_make(2, 1, 1, 128, 128);  // s32 <- s8 x s8
      constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 128, D);    // f32 <- e4m3 x e4m3
      bool ok = mbar_wait(&bar->q_full, 0, kErrTimeoutMma);
      const uint32_t qaddr = smem_u32(smem + L::kOffQ);
      auto pv = [&](int x, int i) -> bool {
        if (!mbar_wait(&bar->p_full[x], i & 1, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t vaddr = smem_u32(smem + L::kOffV + (i % kStages) * L::kV);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ts(tmem + pcol_o(x), tmem + pcol_s(x) + kk * 8, smem_desc_sw128(vaddr + kk * 32), idesc_pv,
                    (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar->o_done[x]);
        return true;
      };
      auto qk = [&](int x, int j) {
        const uint32_t kaddr = smem_u32(smem + L::kOffK + (j % kStages) * L::kK);
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk)
          mma_i8_ss(tmem + pcol_s(x), kmajor_desc<D>(qaddr + x * L::kQ + kk * 32), kmajor_desc<D>(kaddr + kk * 32),
                    idesc_qk, kk > 0);
        mma_commit(&bar->s_full[x]);
      };
      for (int j = 0; ok && j < T; ++j) {
        const int s = j % kStages;
        ok = mbar_wait(&bar->k_full[s], (j / kStages) & 1, kErrTimeoutMma);
        if (ok && j >= 1) ok = mbar_wait(&bar->v_full[(j - 1) % kStages], ((j - 1) / kStages) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        for (int x = 0; ok && x < 2; ++x) {
          if (j >= 1) ok = pv(x, j - 1);
          if (ok) qk(x, j);
        }
        if (!ok) break;
        mma_commit(&bar->k_empty[s]);
        if (j >= 1) mma_commit(&bar->v_empty[(j - 1) % kStages]);
      }
      if (ok && T >= 1) {
        ok = mbar_wait(&bar->v_full[(T - 1) % kStages], ((T - 1) / kStages) & 1, kErrTimeoutMma);
        for (int x = 0; ok && x < 2; ++x) ok = pv(x, T - 1);
        if (ok) mma_commit(&bar->v_empty[(T - 1) % kStages]);
      }
    }
  } else {
    setmaxnreg_inc<224>();
    // ------------------------------------------------------------ softmax of Q tile x
    const int x = warp >> 2;
    const int quarter = warp & 3;
    const int t = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t qtile = qt0 + x;
    const int64_t row = qtile * 128 + t;
    const int64_t unit = hb * p.qtiles + qtile;
    const bool row_valid = row < p.Sq;
    const bool store = row_valid && qtile < p.qtiles && unit >= p.unit_begin && unit < p.unit_end;
    const float qscale = row_valid ? p.qs[hb * p.nqs + (row >> 4) * 8 + (row & 7)] : 0.f;
    const float scale = p.sm_scale;
    const uint32_t scol = tmem + lane_base + pcol_s(x);
    const uint32_t ocol = tmem + lane_base + pcol_o(x);
    float m = -5000000.0f, denom = 0.f;
    bool ok = true;
    float4 ksv_next = __ldg(reinterpret_cast<const float4*>(p.ks + hb * p.nks));
    const uint64_t bias2 = pk2f(kBias, kBias), mag2 = pk2f(kMag, kMag);
    for (int j = 0; j < T; ++j) {
      const float4 ksv = ksv_next;
      if (j + 1 < T) ksv_next = __ldg(reinterpret_cast<const float4*>(p.ks + hb * p.nks + (j + 1) * 4));
      ok = mbar_wait_warp(&bar->s_full[x], j & 1, kErrTimeoutSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t raw[128];
      tmem_ld32(scol + 0, *reinterpret_cast<uint32_t(*)[32]>(raw + 0));
      tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(raw + 32));
      tmem_ld32(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(raw + 64));
      tmem_ld32(scol + 96, *reinterpret_cast<uint32_t(*)[32]>(raw + 96));
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 128; ++c) raw[c] += kBiasBits;
      if (j == T - 1) {
        const int valid = static_cast<int>(p.Sk - int64_t(j) * 128);
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= valid) raw[c] = 0xFF800000u;   // -inf: excluded from the max, encodes to 0
      }
      const float ksg[4] = {ksv.x, ksv.y, ksv.z, ksv.w};
      float f1[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) f1[g] = __fmul_rn(scale, __fmul_rn(qscale, ksg[g]));
      float lmax = -__int_as_float(0x7f800000);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float mx = max3f(__uint_as_float(raw[2 * g]), __uint_as_float(raw[2 * g + 1]), __uint_as_float(raw[2 * g + 8]));
        mx = fmaxf(mx, __uint_as_float(raw[2 * g + 9]));
#pragma unroll
        for (int k = 2; k < 16; ++k)
          mx = max3f(mx, __uint_as_float(raw[8 * k + 2 * g]), __uint_as_float(raw[8 * k + 2 * g + 1]));
        if (mx > 0.f) lmax = fmaxf(lmax, __fmul_rn(__fsub_rn(mx, kBias), f1[g]));
      }
      const float mn = fmaxf(m, lmax);
      const float alpha = expf(m - mn);
      m = mn;
      uint32_t pw[32];
      uint64_t acc = pk2f(0.f, 0.f);
      float gain[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) gain[g] = __fmul_rn(f1[g], kExpA) * (1.0f / 128.0f);
      const float cb = __fmaf_rn(-mn, kExpA, kExpB) * (1.0f / 128.0f);
      const bool safe = !p.exact_expcast && fabsf(mn) <= 128.f && scale >= 1.1754943508222875e-38f &&
                        isfinite(gain[0]) && isfinite(gain[1]) && isfinite(gain[2]) && isfinite(gain[3]);
      if (__all_sync(0xffffffffu, safe)) {
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          uint32_t hw[2];
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int c = 4 * w + 2 * q2;
            const int g = (c >> 1) & 3;
            uint32_t a, bb;
            up2(f2_sub(pk2(raw[c], raw[c + 1]), bias2), a, bb);
            const float va = fma_sat(__uint_as_float(a), gain[g], cb);
            const float vb = fma_sat(__uint_as_float(bb), gain[g], cb);
            uint32_t wa, wb;
            up2(f2_add(pk2f(va, vb), mag2), wa, wb);
            acc = f2_add(acc, pk2(wa << 20, wb << 20));
            hw[q2] = __byte_perm(wa, wb, 0x0040);
          }
          pw[w] = __byte_perm(hw[0], hw[1], 0x5410);
        }
      } else {
        const uint64_t m2 = pk2f(mn, mn);
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          uint32_t hw[2];
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int c = 4 * w + 2 * q2;
            const int g = (c >> 1) & 3;
            const uint64_t sh = f2_sub(f2_mul(f2_sub(pk2(raw[c], raw[c + 1]), bias2), pk2f(f1[g], f1[g])), m2);
            uint32_t a, bb;
            up2(sh, a, bb);
            const float va = fma_sat(__uint_as_float(a), kExpA128, kExpB128);
            const float vb = fma_sat(__uint_as_float(bb), kExpA128, kExpB128);
            uint32_t wa, wb;
            up2(f2_add(pk2f(va, vb), mag2), wa, wb);
            acc = f2_add(acc, pk2(wa << 20, wb << 20));
            hw[q2] = __byte_perm(wa, wb, 0x0040);
          }
          pw[w] = __byte_perm(hw[0], hw[1], 0x5410);
        }
      }
      uint32_t alo, ahi;
      up2(acc, alo, ahi);
      const float mass = __fmul_rn(__fadd_rn(__uint_as_float(alo), __uint_as_float(ahi)), 1.329227995784916e+36f);
      denom = __fadd_rn(__fmul_rn(denom, alpha), mass);
      // rescale this warp's lanes of O_x between PV_x(j-1) and PV_x(j) if any max grew
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        ok = mbar_wait_warp(&bar->o_done[x], (j - 1) & 1, kErrTimeoutSoftmax);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          tmem_ld32(ocol + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__fmul_rn(__uint_as_float(o[i]), alpha));
          tmem_st32(ocol + cc * 32, o);
        }
      }
      tmem_st32(scol, pw);            // P_x(j) into S_x[0,32)
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[x]);
    }
    if (ok) ok = mbar_wait_warp(&bar->o_done[x], (T - 1) & 1, kErrTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      OutT* orow = reinterpret_cast<OutT*>(p.out) + (hb / p.H) * p.osb + (hb % p.H) * p.osh + row * p.oss;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        tmem_ld32(ocol + cc * 32, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int c0 = cc * 32 + c8 * 8;
            const float4 vsa = __ldg(reinterpret_cast<const float4*>(p.vs + hb * D + c0));
            const float4 vsb = __ldg(reinterpret_cast<const float4*>(p.vs + hb * D + c0 + 4));
            const float vsv[8] = {vsa.x, vsa.y, vsa.z, vsa.w, vsb.x, vsb.y, vsb.z, vsb.w};
            float ov[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) ov[i] = __fmul_rn(__fdiv_rn(__uint_as_float(o[c8 * 8 + i]), denom), vsv[i]);
            constexpr int kWords = 8 * int(sizeof(OutT)) / 16;
            uint4 u[kWords];
            OutT* h = reinterpret_cast<OutT*>(u);
#pragma unroll
            for (int i = 0; i < 8; ++i) h[i] = to_out<OutT>(ov[i]);
#pragma unroll
            for (int w = 0; w < kWords; ++w) reinterpret_cast<uint4*>(orow + c0)[w] = u[w];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
