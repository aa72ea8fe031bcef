// Fast fused attention kernel (ExpCast, channel-scaled V, no block means).
// Included by attention.cu (shares its Params, helpers and constants).
//
// Warp roles (320 threads):
//   warps 0-3   softmax half 0: keys 0..63 of every tile, row t = thread t
//   warps 4-7   softmax half 1: keys 64..127, row t = thread t-128 (same
//               TMEM lanes as warp-4); the two halves exchange their partial
//               row maxima through shared memory (64-thread named barrier)
//   warp 8      TMA producer: K [128 x D] and V^T [D x 128] tiles into a ring
//   warp 9      tensor-memory allocator + single-thread MMA issuer
//
// Tensor memory (512 columns):
//   S0 [0,128) S1 [128,256)   s32 scores Q.K^T of tiles j%2; after the row has
//                             been read, its ExpCast bytes P are written into
//                             the first 32 columns (A operand of P.V)
//   O  [256,256+D+16)         FP32 output accumulator for the whole K loop;
//                             column D accumulates P.1 (the denominator)
//   Q  [480,480+D/4)          int8 Q tile (A operand of Q.K^T)
// V tiles carry 16 extra K-major rows in shared memory: row D is E4M3 1.0
// (0x38), rows D+1.. are 0, so the P.V MMA (N = D+16) also produces the FP32
// sum of the decoded probabilities -- the ExpCast denominator -- with no
// per-score ALU work.  Out-of-range keys of the last tile encode to byte 0.
//
// Ordering: the tensor core executes MMAs in issue order, so QK(j) (issued
// after PV(j-2)) cannot overwrite P(j-2) before it is consumed.  A warp whose
// rows' maximum grew scales its lanes of O after PV(j-1) completes and before
// it releases P(j); PV(j) then accumulates on the rescaled O.
//
// Per-score arithmetic (no conversion-unit instructions):
//   float(raw) = as_float(raw + 0x4B400000) - 1.5*2^23    (exact, |raw| < 2^22)
//   logit      = RN(float(raw) * RN(scale * RN(qs*ks)))   (packed f32x2)
//   v          = sat(fma(RN(logit - m'), A/128, B/128))    (= clamp(u,0,128)/128)
//   byte       = low byte of as_int(v + 1.5*2^16)          (RNE to 1/128)
#pragma once

constexpr int kFastThreads = 320;
constexpr uint32_t kFColS0 = 0, kFColS1 = 128, kFColO = 256, kFColQ = 480;

struct __align__(8) FastBarriers {
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t q_ready, s_full[2], p_full[2], o_done;
};

template <int D>
struct FastSmem {
  static constexpr int kK = 128 * D;            // K stage bytes
  static constexpr int kV = (D + 16) * 128;      // V stage bytes incl. the ones/zero rows
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kStages * kK;
  static constexpr int kOffX = kOffV + kStages * kV;    // float [2 tiles][2 halves][128 rows] max exchange
  static constexpr int kOffBar = kOffX + 4 * 128 * 4;
  static constexpr int kOffSlot = kOffBar + int(sizeof(FastBarriers));
  static constexpr int kBytes = kOffSlot + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pk2f(float lo, float hi) { return pk2(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ void up2(uint64_t v, uint32_t& lo, uint32_t& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float r;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr uint32_t kBiasBits = 0x4B400000u;   // 1.5 * 2^23
constexpr float kBias = 12582912.0f;
constexpr float kMag = 98304.0f;              // 1.5 * 2^16
constexpr float kExpA128 = 11.541560173034668f / 128.0f;
constexpr float kExpB128 = 119.6500015258789f / 128.0f;

template <int D, typename OutT>
__global__ void __launch_bounds__(kFastThreads, 1)
    vc_attention_fast_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                             Params p) {
  using L = FastSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FastBarriers* bar = reinterpret_cast<FastBarriers*>(smem + L::kOffBar);
  float* xch = reinterpret_cast<float*>(smem + L::kOffX);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = p.unit_begin + blockIdx.x;
  const int64_t bh = unit / p.qtiles;
  const int64_t qt = unit - bh * p.qtiles;
  const int T = static_cast<int>(p.ktiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
    }
    mbar_init(&bar->q_ready, 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->s_full[b], 1);
      mbar_init(&bar->p_full[b], 256);
    }
    mbar_init(&bar->o_done, 1);
    fence_barrier_init();
  }
  // ones row (E4M3 1.0) and zero rows below each V stage's D rows
  for (int i = threadIdx.x; i < kStages * 16 * 128 / 16; i += kFastThreads) {
    const int s = i / (16 * 128 / 16), r = (i / 8) % 16, c = i % 8;
    const uint32_t fill = r == 0 ? 0x38383838u : 0u;
    *reinterpret_cast<uint4*>(smem + L::kOffV + s * L::kV + (D + r) * 128 + c * 16) = make_uint4(fill, fill, fill, fill);
  }
  fence_proxy_async_smem();
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int j = 0; j < T; ++j) {
        const int s = j % kStages;
        const uint32_t ph = ((j / kStages) & 1) ^ 1;
        if (j >= kStages && !mbar_wait(&bar->k_empty[s], ph, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->k_full[s], L::kK);
        tma_load_3d(smem + L::kOffK + s * L::kK, &tmk, &bar->k_full[s], 0, j * 128, static_cast<int>(bh));
        if (j >= kStages && !mbar_wait(&bar->v_empty[s], ph, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->v_full[s], D * 128);
        tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(bh));
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_make(2, 1, 1, 128, 128);    // s32 <- s8 x s8
      constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 128, D + 16); // f32 <- e4m3 x e4m3
      bool ok = mbar_wait(&bar->q_ready, 0, kErrTimeoutMma);
      tc_fence_after();
      auto issue_pv = [&](int i) -> bool {
        const int s = i % kStages;
        if (!mbar_wait(&bar->v_full[s], (i / kStages) & 1, kErrTimeoutMma)) return false;
        if (!mbar_wait(&bar->p_full[i & 1], (i >> 1) & 1, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t vaddr = smem_u32(smem + L::kOffV + s * L::kV);
        const uint32_t pcol = (i & 1) ? kFColS1 : kFColS0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ts(tmem + kFColO, tmem + pcol + kk * 8, smem_desc_sw128(vaddr + kk * 32), idesc_pv,
                    (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar->v_empty[s]);
        mma_commit(&bar->o_done);
        return true;
      };
      for (int j = 0; ok && j < T; ++j) {
        const int s = j % kStages;
        ok = mbar_wait(&bar->k_full[s], (j / kStages) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kaddr = smem_u32(smem + L::kOffK + s * L::kK);
        const uint32_t scol = (j & 1) ? kFColS1 : kFColS0;
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          uint64_t desc;
          if constexpr (D == 128) desc = smem_desc_sw128(kaddr + kk * 32);
          else desc = smem_desc_sw64(kaddr + kk * 32);
          mma_i8_ts(tmem + scol, tmem + kFColQ + kk * 8, desc, idesc_qk, kk > 0);
        }
        mma_commit(&bar->k_empty[s]);
        mma_commit(&bar->s_full[j & 1]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && T >= 1) issue_pv(T - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax halves
    const int half = warp >> 2;                 // 0: keys 0..63, 1: keys 64..127
    const int quarter = warp & 3;
    const int t = threadIdx.x & 127;            // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t row = qt * 128 + t;
    const bool row_valid = row < p.Sq;
    if (half == 0) {
      uint32_t qw[32];
      const int8_t* qrow = p.q8 + (bh * p.Sq + row) * D;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        uint4 u = row_valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + i) : make_uint4(0, 0, 0, 0);
        qw[4 * i] = u.x; qw[4 * i + 1] = u.y; qw[4 * i + 2] = u.z; qw[4 * i + 3] = u.w;
      }
      if constexpr (D == 128) tmem_st32(tmem + lane_base + kFColQ, qw);
      else tmem_st16(tmem + lane_base + kFColQ, qw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->q_ready);
    }
    const float qscale = row_valid ? p.qs[bh * p.nqs + (row >> 4) * 8 + (row & 7)] : 0.f;
    const float scale = p.sm_scale;
    const int key0 = half * 64;
    float m = -5000000.0f;
    bool ok = true;
    float4 ksv_next = __ldg(reinterpret_cast<const float4*>(p.ks + bh * p.nks));
    for (int j = 0; j < T; ++j) {
      const int b = j & 1;
      const uint32_t sbase = b ? kFColS1 : kFColS0;
      const float4 ksv = ksv_next;
      if (j + 1 < T) ksv_next = __ldg(reinterpret_cast<const float4*>(p.ks + bh * p.nks + (j + 1) * 4));
      ok = mbar_wait_warp(&bar->s_full[b], (j >> 1) & 1, kErrTimeoutSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t raw[64];
      tmem_ld32(tmem + lane_base + sbase + key0, *reinterpret_cast<uint32_t(*)[32]>(raw + 0));
      tmem_ld32(tmem + lane_base + sbase + key0 + 32, *reinterpret_cast<uint32_t(*)[32]>(raw + 32));
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 64; ++c) raw[c] += kBiasBits;
      if (j == T - 1) {
        const int valid = static_cast<int>(p.Sk - int64_t(j) * 128) - key0;
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= valid) raw[c] = 0xFF800000u;   // -inf: excluded from the max, encodes to 0
      }
      const float ksg[4] = {ksv.x, ksv.y, ksv.z, ksv.w};
      float f1[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) f1[g] = __fmul_rn(scale, __fmul_rn(qscale, ksg[g]));
      // partial max over this half's keys, per column group g = (c>>1)&3
      float lmax = -__int_as_float(0x7f800000);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float mx = max3f(__uint_as_float(raw[2 * g]), __uint_as_float(raw[2 * g + 1]), __uint_as_float(raw[2 * g + 8]));
        mx = fmaxf(mx, __uint_as_float(raw[2 * g + 9]));
#pragma unroll
        for (int k = 2; k < 8; ++k)
          mx = max3f(mx, __uint_as_float(raw[8 * k + 2 * g]), __uint_as_float(raw[8 * k + 2 * g + 1]));
        if (mx > 0.f) lmax = fmaxf(lmax, __fmul_rn(__fsub_rn(mx, kBias), f1[g]));
      }
      // exchange with the other half of the row (same TMEM lanes)
      tc_fence_before();
      xch[(b * 2 + half) * 128 + t] = lmax;
      named_bar(1 + quarter, 64);
      tc_fence_after();
      const float mn = fmaxf(m, fmaxf(lmax, xch[(b * 2 + (half ^ 1)) * 128 + t]));
      const float alpha = expf(m - mn);
      m = mn;
      // ExpCast bytes for this half's 64 keys (16 words).  Default: the
      // reference's folded affine encoder (csrc/vc/vc_math.cuh:17-71, 96-106)
      //   u = fma(float(raw), RN(f1*A), fma(-m', A, B))
      // used while |m'| <= 128 and the gain is finite; otherwise (and when
      // the exact mode is requested) the unfused RN(RN(raw*f1) - m') form.
      const uint64_t bias2 = pk2f(kBias, kBias), mag2 = pk2f(kMag, kMag);
      uint32_t pw[16];
      float gain[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) gain[g] = __fmul_rn(f1[g], kExpA) * (1.0f / 128.0f);
      const float cb = __fmaf_rn(-mn, kExpA, kExpB) * (1.0f / 128.0f);
      const bool safe = !p.exact_expcast && fabsf(mn) <= 128.f && scale >= 1.1754943508222875e-38f &&
                        isfinite(gain[0]) && isfinite(gain[1]) && isfinite(gain[2]) && isfinite(gain[3]);
      if (__all_sync(0xffffffffu, safe)) {
#pragma unroll
        for (int w = 0; w < 16; ++w) {
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
            hw[q2] = __byte_perm(wa, wb, 0x0040);
          }
          pw[w] = __byte_perm(hw[0], hw[1], 0x5410);
        }
      } else {
        const uint64_t m2 = pk2f(mn, mn);
#pragma unroll
        for (int w = 0; w < 16; ++w) {
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
            hw[q2] = __byte_perm(wa, wb, 0x0040);
          }
          pw[w] = __byte_perm(hw[0], hw[1], 0x5410);
        }
      }
      // rescale this warp's share of O (after PV(j-1), before PV(j)) if any max grew
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        ok = mbar_wait_warp(&bar->o_done, (j - 1) & 1, kErrTimeoutSoftmax);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ocol = tmem + lane_base + kFColO + half * (D / 2);
#pragma unroll
        for (int cc = 0; cc < D / 64; ++cc) {
          uint32_t o[32];
          tmem_ld32(ocol + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__fmul_rn(__uint_as_float(o[i]), alpha));
          tmem_st32(ocol + cc * 32, o);
        }
        if (half == 1) {   // the denominator column
          uint32_t o[16];
          tmem_ld16(tmem + lane_base + kFColO + D, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__fmul_rn(__uint_as_float(o[i]), alpha));
          tmem_st16(tmem + lane_base + kFColO + D, o);
        }
        tmem_wait_st();
      }
      // P bytes into the first 32 columns of this S buffer (keys 4c..4c+3 per column)
      tmem_st16(tmem + lane_base + sbase + half * 16, pw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[b]);
    }
    // epilogue: this half's output channels, O / denominator * channel scale
    if (ok) ok = mbar_wait_warp(&bar->o_done, (T - 1) & 1, kErrTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      uint32_t dn[16];
      tmem_ld16(tmem + lane_base + kFColO + D, dn);
      tmem_wait_ld();
      const float denom = __uint_as_float(dn[0]);
      OutT* orow = reinterpret_cast<OutT*>(p.out) + (bh / p.H) * p.osb + (bh % p.H) * p.osh + row * p.oss;
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c0 = half * (D / 2) + cc * 32;
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kFColO + c0, o);
        tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const float4 vsa = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c0 + c8 * 8));
            const float4 vsb = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c0 + c8 * 8 + 4));
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
            for (int w = 0; w < kWords; ++w) reinterpret_cast<uint4*>(orow + c0 + c8 * 8)[w] = u[w];
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
