// Fused VC attention for sm_100a (B200).
//
// One CTA owns a 128-row Q tile of one (batch, head) and streams all K/V
// tiles of 128 tokens:
//
//   warp 8      TMA producer: K tile [128 x D] int8 and V^T tile [D x 128]
//               E4M3 into a ring of shared-memory stages (128B/64B swizzle)
//   warp 9      tensor-memory allocator and single-thread MMA issuer:
//                 S[j%2]  = Q . K_j^T   tcgen05.mma kind::i8, A = Q in TMEM
//                 O       = P_j . V_j   tcgen05.mma kind::f8f6f4, A = P in TMEM
//   warps 0-3   softmax: thread t owns row t (TMEM lane t) -- the whole
//               128-key row is thread-local, so row max / mass need no
//               cross-thread reduction.  Dequantises S with the Sage
//               per-thread scales, updates the running max, encodes
//               ExpCast bytes straight into the P tensor-memory buffer and
//               computes the FP32 mass of the decoded bytes.
//   warps 4-7   correction/epilogue: thread 128+t owns row t; keeps the FP32
//               output history in registers (two-level accumulation:
//               out = out*alpha + P.V [+ mass*mean]) and writes bf16/fp16.
//
// Tensor memory (512 columns): Q [0,32) | P0 [32,64) | P1 [64,96) |
// S0 [128,256) | S1 [256,384) | O [384,384+D).
//
// Arithmetic follows the decoded-payload contract of the reference
// (third_party/sageattention_local/sageattention_local/vc_reference.py:20-91,
// csrc/vc/vc_math.cuh:269-479, csrc/vc/vc_sm90.cu:284-604):
//   logits = RN(raw * RN(scale * RN(qs*ks)))         (last tile: RN(RN(raw*qs*ks)*scale))
//   m'     = max(m, max logits) from m = -5e6;  alpha = exp(m - m')
//   code   = cvt.rni.sat(fma(RN(logit - m'), 8 log2 e, 119.65)) clamped to [0,120]
//   mass   = sum of decoded E4M3 codes (exact in FP32)
//   out    = out*alpha + P.V (+ mass*mean [* block scale]);  out/denom [* channel scale]
// All device waits are bounded; on timeout the kernel records an error bit
// and unwinds instead of hanging.
#include <cuda.h>
#include <cstdlib>
#include <cstring>
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kThreads = 320;
constexpr int kStages = 3;
constexpr uint32_t kColQ = 0, kColP0 = 32, kColP1 = 64, kColS0 = 128, kColS1 = 256, kColO = 384;
constexpr float kExpA = 11.541560173034668f;
constexpr float kExpB = 119.6500015258789f;

struct Params {
  const int8_t* q8;
  const float* qs;
  const float* ks;
  const float* vs;
  const __half* means;
  void* out;
  int64_t H, Sq, Sk;
  int64_t osb, osh, oss;
  int64_t nqs, nks, ktiles, qtiles;
  int64_t kq_tiles;   // E4M3 block Q/K: K tiles per K scale
  int64_t unit_begin, unit_end;   // units (b*H+h)*qtiles + q_tile to compute
  int64_t pair_begin, qpairs;     // paired-tile kernel: first pair (b*H+h)*qpairs + q_tile/2, pairs per head
  float sm_scale;
  int exact_expcast;   // 1: unfused RN(RN(raw*f)-m) encoder instead of the folded affine one
  float ctl_offset;    // FP8-P control: P = e4m3(exp2(logit - max + offset)); 8.807 Sage, 8 the Config contract
};

struct __align__(8) Barriers {
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t q_ready, s_full[2], s_free[2], p_full[2], p_free[2], o_full, o_free, st_full[2], st_free[2];
};

template <int D>
struct Smem {
  static constexpr int kK = 128 * D;   // bytes per K stage
  static constexpr int kV = D * 128;   // bytes per V stage
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kStages * kK;
  static constexpr int kOffStats = kOffV + kStages * kV;          // float2 [2][128]
  static constexpr int kOffBar = kOffStats + 2 * 128 * 8;
  static constexpr int kOffSlot = kOffBar + int(sizeof(Barriers));
  static constexpr int kBytes = kOffSlot + 16;
  static constexpr int kAlloc = kBytes + 1024;                     // room for 1024B alignment
};

__device__ __forceinline__ float decode_e4m3_code(uint32_t c) {
  // codes 0..120 only (non-negative ExpCast bytes)
  return c < 8u ? static_cast<float>(c) * 0.001953125f : __uint_as_float((c << 20) + 0x3C000000u);
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float x);
template <>
__device__ __forceinline__ __half to_out<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ float to_out<float>(float x) { return x; }

// QF8: E4M3 block Q/K (the Config contract's Hadamard path): QK^T is
// kind::f8f6f4 into FP32, the Q scale is one per 128-row tile and the K scale
// one per kq_tiles K tiles; logits are raw * RN(scale * RN(qs * ks)) on every tile.
template <int D, typename OutT, bool EXPCAST, bool BLOCK_VALUES, bool VS_PER_BLOCK, bool QF8 = false>
__global__ void __launch_bounds__(kThreads, 1)
    vc_attention_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Params p) {
  using L = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bar = reinterpret_cast<Barriers*>(smem + L::kOffBar);
  float2* stats = reinterpret_cast<float2*>(smem + L::kOffStats);
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
      mbar_init(&bar->s_free[b], 128);
      mbar_init(&bar->p_full[b], 128);
      mbar_init(&bar->p_free[b], 1);
      mbar_init(&bar->st_full[b], 128);
      mbar_init(&bar->st_free[b], 128);
    }
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->o_free, 128);
    fence_barrier_init();
  }
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
        mbar_expect_tx(&bar->v_full[s], L::kV);
        tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(bh));
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = QF8 ? idesc_make(1, 0, 0, 128, 128)     // f32 <- e4m3 x e4m3
                                        : idesc_make(2, 1, 1, 128, 128);    // s32 <- s8 x s8
      constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 128, D);    // f32 <- e4m3 x e4m3
      bool ok = mbar_wait(&bar->q_ready, 0, kErrTimeoutMma);
      tc_fence_after();
      auto issue_pv = [&](int i) -> bool {
        const int s = i % kStages;
        if (!mbar_wait(&bar->v_full[s], (i / kStages) & 1, kErrTimeoutMma)) return false;
        if (!mbar_wait(&bar->p_full[i & 1], (i >> 1) & 1, kErrTimeoutMma)) return false;
        if (i >= 1 && !mbar_wait(&bar->o_free, (i - 1) & 1, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t vaddr = smem_u32(smem + L::kOffV + s * L::kV);
        const uint32_t pcol = (i & 1) ? kColP1 : kColP0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ts(tmem + kColO, tmem + pcol + kk * 8, smem_desc_sw128(vaddr + kk * 32), idesc_pv, kk > 0);
        mma_commit(&bar->v_empty[s]);
        mma_commit(&bar->p_free[i & 1]);
        mma_commit(&bar->o_full);
        return true;
      };
      for (int j = 0; ok && j < T; ++j) {
        const int s = j % kStages;
        ok = mbar_wait(&bar->k_full[s], (j / kStages) & 1, kErrTimeoutMma);
        if (ok && j >= 2) ok = mbar_wait(&bar->s_free[j & 1], ((j - 2) >> 1) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kaddr = smem_u32(smem + L::kOffK + s * L::kK);
        const uint32_t scol = (j & 1) ? kColS1 : kColS0;
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          uint64_t desc;
          if constexpr (D == 128) desc = smem_desc_sw128(kaddr + kk * 32);
          else desc = smem_desc_sw64(kaddr + kk * 32);
          if constexpr (QF8) mma_f8_ts(tmem + scol, tmem + kColQ + kk * 8, desc, idesc_qk, kk > 0);
          else mma_i8_ts(tmem + scol, tmem + kColQ + kk * 8, desc, idesc_qk, kk > 0);
        }
        mma_commit(&bar->k_empty[s]);
        mma_commit(&bar->s_full[j & 1]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && T >= 1) issue_pv(T - 1);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ softmax
    const int t = threadIdx.x;  // row within tile
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t row = qt * 128 + t;
    const bool row_valid = row < p.Sq;
    {
      uint32_t qw[32];
      const int8_t* qrow = p.q8 + (bh * p.Sq + row) * D;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        uint4 u = row_valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + i) : make_uint4(0, 0, 0, 0);
        qw[4 * i] = u.x; qw[4 * i + 1] = u.y; qw[4 * i + 2] = u.z; qw[4 * i + 3] = u.w;
      }
      if constexpr (D == 128) {
        tmem_st32(tmem + lane_base + kColQ, qw);
      } else {
        tmem_st16(tmem + lane_base + kColQ, qw);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->q_ready);
    }
    const float qscale =
        row_valid ? (QF8 ? p.qs[bh * p.nqs + qt] : p.qs[bh * p.nqs + (row >> 4) * 8 + (row & 7)]) : 0.f;
    const float scale = EXPCAST ? p.sm_scale : __fmul_rn(p.sm_scale, 1.4426950408889634f);
    float m = -5000000.0f;
    for (int j = 0; j < T; ++j) {
      const int b = j & 1;
      if (!mbar_wait_warp(&bar->s_full[b], (j >> 1) & 1, kErrTimeoutSoftmax)) break;
      tc_fence_after();
      uint32_t raw[128];
      const uint32_t scol = tmem + lane_base + (b ? kColS1 : kColS0);
      tmem_ld32(scol + 0, *reinterpret_cast<uint32_t(*)[32]>(raw + 0));
      tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(raw + 32));
      tmem_ld32(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(raw + 64));
      tmem_ld32(scol + 96, *reinterpret_cast<uint32_t(*)[32]>(raw + 96));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bar->s_free[b]);

      float4 ksv;
      if constexpr (QF8) {
        const float kv = __ldg(p.ks + bh * p.nks + j / p.kq_tiles);
        ksv = make_float4(kv, kv, kv, kv);
      } else {
        ksv = __ldg(reinterpret_cast<const float4*>(p.ks + bh * p.nks + j * 4));
      }
      const float ksg[4] = {ksv.x, ksv.y, ksv.z, ksv.w};
      const int valid = j == T - 1 ? static_cast<int>(p.Sk - int64_t(j) * 128) : 128;
      // INT8: the reference's last-tile order (raw * qs * ks) * scale; E4M3 blocks: one order on every tile
      const bool last = j == T - 1 && !QF8;
      // per-column-group logit multipliers (a group shares one K scale)
      float f1[4], f2[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const float dq = __fmul_rn(qscale, ksg[g]);
        f1[g] = last ? dq : __fmul_rn(scale, dq);   // first multiply
        f2[g] = scale;                              // second multiply (last tile only)
      }
      auto rawf = [&](int c) -> float {
        return QF8 ? __uint_as_float(raw[c]) : __int2float_rn(static_cast<int>(raw[c]));
      };
      auto logit = [&](int c) -> float {
        const float x = rawf(c);
        const int g = (c >> 1) & 3;
        return last ? __fmul_rn(__fmul_rn(x, f1[g]), f2[g]) : __fmul_rn(x, f1[g]);
      };
      float alpha, mass = 0.f;
      uint32_t pw[32];
      if constexpr (EXPCAST) {
        float lmax = -__int_as_float(0x7f800000);
        if constexpr (QF8) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < valid) lmax = fmaxf(lmax, logit(c));
        } else {
          int gm[4] = {INT_MIN, INT_MIN, INT_MIN, INT_MIN};
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < valid) gm[(c >> 1) & 3] = max(gm[(c >> 1) & 3], static_cast<int>(raw[c]));
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (gm[g] == INT_MIN) continue;
            const float x = __int2float_rn(gm[g]);
            lmax = fmaxf(lmax, last ? __fmul_rn(__fmul_rn(x, f1[g]), f2[g]) : __fmul_rn(x, f1[g]));
          }
        }
        const float mn = fmaxf(m, lmax);
        alpha = expf(m - mn);
        m = mn;
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          uint32_t word = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = 4 * w + e;
            uint32_t code = 0;
            if (c < valid) {
              const float u = __fmaf_rn(__fsub_rn(logit(c), m), kExpA, kExpB);
              uint32_t cv;
              asm("cvt.rni.sat.u8.f32 %0, %1;" : "=r"(cv) : "f"(u));
              code = min(cv, 120u);
            }
            mass = __fadd_rn(mass, decode_e4m3_code(code));
            word |= code << (8 * e);
          }
          pw[w] = word;
        }
      } else {
        // FP8 probability control (vc_reference.py:56-64): the row maximum is
        // taken over fma(logit, 1, -offset); P = e4m3(exp2(logit - m')), the
        // denominator uses the unrounded exp2 values.  offset 8.807 is Sage's;
        // 8 gives the Config contract's P8 = e4m3(256 exp(s - max)) with the
        // exact exp row sums (src/vc_attention/core.py:357-360).
        const float off = p.ctl_offset;
        float lmax = -__int_as_float(0x7f800000);
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          if (c >= valid) continue;
          const int g = (c >> 1) & 3;
          const float x = rawf(c);
          const float base = last ? __fmul_rn(x, f1[g]) : x;
          const float fac = last ? f2[g] : f1[g];
          lmax = fmaxf(lmax, __fmaf_rn(base, fac, -off));
        }
        const float mn = fmaxf(m, lmax);
        alpha = exp2f(m - mn);
        m = mn;
#pragma unroll
        for (int w = 0; w < 32; ++w) {
          float pv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = 4 * w + e;
            pv[e] = 0.f;
            if (c < valid) {
              const int g = (c >> 1) & 3;
              const float x = rawf(c);
              const float base = last ? __fmul_rn(x, f1[g]) : x;
              const float fac = last ? f2[g] : f1[g];
              pv[e] = exp2f(__fmaf_rn(base, fac, -m));
            }
            mass = __fadd_rn(mass, pv[e]);
          }
          pw[w] = uint32_t(e4m3x2(pv[0], pv[1])) | (uint32_t(e4m3x2(pv[2], pv[3])) << 16);
        }
      }
      if (j >= 2 && !mbar_wait_warp(&bar->p_free[b], ((j - 2) >> 1) & 1, kErrTimeoutSoftmax)) break;
      tc_fence_after();
      tmem_st32(tmem + lane_base + (b ? kColP1 : kColP0), pw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[b]);
      if (j >= 2 && !mbar_wait_warp(&bar->st_free[b], ((j - 2) >> 1) & 1, kErrTimeoutSoftmax)) break;
      stats[b * 128 + t] = make_float2(alpha, mass);
      mbar_arrive(&bar->st_full[b]);
    }
  } else {
    // ------------------------------------------------------------ correction
    const int t = threadIdx.x - 128;
    const uint32_t lane_base = static_cast<uint32_t>((warp - 4) * 32) << 16;
    const int64_t row = qt * 128 + t;
    float acc[D];
#pragma unroll
    for (int c = 0; c < D; ++c) acc[c] = 0.f;
    float denom = 0.f;
    bool ok = true;
    for (int j = 0; j < T; ++j) {
      const int b = j & 1;
      ok = mbar_wait_warp(&bar->st_full[b], (j >> 1) & 1, kErrTimeoutCorrection);
      if (!ok) break;
      const float2 st = stats[b * 128 + t];
      mbar_arrive(&bar->st_free[b]);
      const float alpha = st.x, mass = st.y;
      denom = __fadd_rn(__fmul_rn(denom, alpha), mass);
      ok = mbar_wait_warp(&bar->o_full, j & 1, kErrTimeoutCorrection);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t pr[32];
        tmem_ld32(tmem + lane_base + kColO + cc * 32, pr);
        tmem_wait_ld();
        float mean[32], bscale[32];
        if constexpr (BLOCK_VALUES) {
          const __half* mp = p.means + (bh * p.ktiles + j) * D + cc * 32;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(mp) + i);
            const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __half22float2(h2[k]);
              mean[8 * i + 2 * k] = f.x;
              mean[8 * i + 2 * k + 1] = f.y;
            }
          }
          if constexpr (VS_PER_BLOCK) {
            const float* sp = p.vs + (bh * p.ktiles + j) * D + cc * 32;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 f = __ldg(reinterpret_cast<const float4*>(sp) + i);
              bscale[4 * i] = f.x; bscale[4 * i + 1] = f.y; bscale[4 * i + 2] = f.z; bscale[4 * i + 3] = f.w;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float contrib = __uint_as_float(pr[i]);
          if constexpr (BLOCK_VALUES) {
            contrib = __fadd_rn(contrib, __fmul_rn(mass, mean[i]));
            if constexpr (VS_PER_BLOCK) contrib = __fmul_rn(contrib, bscale[i]);
          }
          acc[cc * 32 + i] = __fadd_rn(__fmul_rn(acc[cc * 32 + i], alpha), contrib);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar->o_free);
    }
    if (ok && row < p.Sq) {
      OutT* orow = reinterpret_cast<OutT*>(p.out) + (bh / p.H) * p.osb + (bh % p.H) * p.osh + row * p.oss;
#pragma unroll
      for (int c8 = 0; c8 < D / 8; ++c8) {
        float o[8];
        float4 vsa = make_float4(1.f, 1.f, 1.f, 1.f), vsb = vsa;
        if constexpr (!VS_PER_BLOCK) {
          vsa = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c8 * 8));
          vsb = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c8 * 8 + 4));
        }
        const float vsv[8] = {vsa.x, vsa.y, vsa.z, vsa.w, vsb.x, vsb.y, vsb.z, vsb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = __fdiv_rn(acc[c8 * 8 + i], denom);
          if constexpr (!VS_PER_BLOCK) o[i] = __fmul_rn(o[i], vsv[i]);
        }
        constexpr int kWords = 8 * int(sizeof(OutT)) / 16;  // 16-byte stores per 8 outputs
        uint4 u[kWords];
        OutT* h = reinterpret_cast<OutT*>(u);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = to_out<OutT>(o[i]);
#pragma unroll
        for (int w = 0; w < kWords; ++w) reinterpret_cast<uint4*>(orow + c8 * 8)[w] = u[w];
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

#include "attention_softmax.cuh"
#include "attention_alt.cuh"
#include "attention_pair.cuh"

// ---------------------------------------------------------------------------
// Host side: tensor maps and dispatch.
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

bool make_map_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1,
                 CUtensorMapSwizzle sw) {
  EncodeFn enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {d0, d0 * d1};  // bytes (uint8 elements)
  const cuuint32_t box[3] = {b0, b1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, typename OutT, bool EXPCAST, bool BV, bool VPB, bool QF8 = false>
int launch_attn(const AttnArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p, int64_t units,
                cudaStream_t st) {
  auto k = vc_attention_kernel<D, OutT, EXPCAST, BV, VPB, QF8>;
  const int smem = Smem<D>::kAlloc;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return VC_ERR_LAUNCH;
  k<<<static_cast<unsigned>(units), kThreads, smem, st>>>(mk, mv, p);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

// VC_B200_KERNEL selects another kernel for ExpCast + channel-scaled V:
// "general" (register accumulation), "alt" (one Q tile per CTA, the two
// softmax groups alternating K tiles) or "pair" (the paired-tile kernel for
// every pair, no alternating-tile tail); the default is the paired-tile
// kernel with the tail rule below.
bool use_general_kernel() {
  const char* e = getenv("VC_B200_KERNEL");
  return e && strcmp(e, "general") == 0;
}
bool use_alt_kernel() {
  const char* e = getenv("VC_B200_KERNEL");
  return e && strcmp(e, "alt") == 0;
}
bool use_pair_only() {
  const char* e = getenv("VC_B200_KERNEL");
  return e && strcmp(e, "pair") == 0;
}

struct Maps {
  CUtensorMap q, k, v;
};

template <int D, typename OutT, bool BV, bool QF8 = false>
int launch_pair(const Maps& m, const Params& p, int64_t pairs, cudaStream_t st) {
  auto k = vc_attention_pair_kernel<D, OutT, BV, QF8>;
  const int smem = PairSmem<D>::kAlloc;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return VC_ERR_LAUNCH;
  k<<<static_cast<unsigned>(pairs), kPairThreads, smem, st>>>(m.q, m.k, m.v, p);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

template <int D, typename OutT, bool BV, bool QF8 = false>
int launch_alt(const Maps& m, const Params& p, int64_t units, cudaStream_t st) {
  auto k = vc_attention_alt_kernel<D, OutT, BV, QF8>;
  const int smem = AltSmem<D>::kAlloc;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return VC_ERR_LAUNCH;
  k<<<static_cast<unsigned>(units), kAltThreads, smem, st>>>(m.k, m.v, p);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

// How a unit range is spread over the two tensor-memory kernels: the paired
// kernel over `pairs` pairs from p.pair_begin, then the alternating-tile kernel
// over tail.unit_begin .. tail.unit_end (tail_units of them, possibly none).
struct Split {
  int64_t pairs = 0;
  Params tail;
  int64_t tail_units = 0;
};

template <int D, typename OutT, bool BV, bool QF8 = false>
int launch_split(const Maps& m, const Params& p, const Split& sp, cudaStream_t st) {
  if (sp.pairs > 0) {
    const int rc = launch_pair<D, OutT, BV, QF8>(m, p, sp.pairs, st);
    if (rc != VC_OK) return rc;
  }
  return sp.tail_units > 0 ? launch_alt<D, OutT, BV, QF8>(m, sp.tail, sp.tail_units, st) : VC_OK;
}

template <int D, typename OutT>
int dispatch_flags(const AttnArgs& a, const Maps& m, const Params& p, int64_t units, const Split& sp,
                   cudaStream_t st) {
  const bool alt = use_alt_kernel();
  if (a.qk_e4m3 && (!a.expcast || a.vs_per_block)) {
    // E4M3 block Q/K with the FP8-P control or per-block V scales (the Config
    // contract's own formats): the register-accumulating kernel
    if (a.expcast) return launch_attn<D, OutT, true, true, true, true>(a, m.k, m.v, p, units, st);
    if (!a.block_values) return launch_attn<D, OutT, false, false, false, true>(a, m.k, m.v, p, units, st);
    if (a.vs_per_block) return launch_attn<D, OutT, false, true, true, true>(a, m.k, m.v, p, units, st);
    return launch_attn<D, OutT, false, true, false, true>(a, m.k, m.v, p, units, st);
  }
  if (a.qk_e4m3) {   // E4M3 block Q/K, ExpCast, channel V scales: the tensor-memory kernels
    if (alt) {
      if (a.block_values) return launch_alt<D, OutT, true, true>(m, p, units, st);
      return launch_alt<D, OutT, false, true>(m, p, units, st);
    }
    if (a.block_values) return launch_split<D, OutT, true, true>(m, p, sp, st);
    return launch_split<D, OutT, false, true>(m, p, sp, st);
  }
  if (a.expcast && !a.vs_per_block && !use_general_kernel() && !alt) {
    if (a.block_values) return launch_split<D, OutT, true>(m, p, sp, st);
    return launch_split<D, OutT, false>(m, p, sp, st);
  }
  if (a.expcast && !a.vs_per_block && alt) {
    if (a.block_values) return launch_alt<D, OutT, true>(m, p, units, st);
    return launch_alt<D, OutT, false>(m, p, units, st);
  }
  const CUtensorMap& mk = m.k;
  const CUtensorMap& mv = m.v;
  if (a.expcast) {
    if (!a.block_values) return launch_attn<D, OutT, true, false, false>(a, mk, mv, p, units, st);
    if (a.vs_per_block) return launch_attn<D, OutT, true, true, true>(a, mk, mv, p, units, st);
    return launch_attn<D, OutT, true, true, false>(a, mk, mv, p, units, st);
  }
  if (!a.block_values) return launch_attn<D, OutT, false, false, false>(a, mk, mv, p, units, st);
  if (a.vs_per_block) return launch_attn<D, OutT, false, true, true>(a, mk, mv, p, units, st);
  return launch_attn<D, OutT, false, true, false>(a, mk, mv, p, units, st);
}

}  // namespace

// Streaming multiprocessors of the current device (cached per device).
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// One paired-tile CTA per SM.  If the last wave of pairs would be at most half
// full, the tiles of those pairs (at most one per SM) run on the
// alternating-tile kernel after the full waves: about 0.6 of a pair period
// instead of one.  The tail pairs are the last ones of the range, so their
// units are the range's last ones too.  sms = 0: pairs only.  Host only.
AttnPlan attention_plan(int64_t qtiles, int64_t ub, int64_t ue, int64_t sms) {
  AttnPlan r;
  if (qtiles <= 0 || ub < 0 || ue <= ub) {
    r.tail_begin = ue;
    return r;
  }
  const int64_t qpairs = (qtiles + 1) / 2;
  const int64_t pb = (ub / qtiles) * qpairs + (ub % qtiles) / 2;
  const int64_t pe = ((ue - 1) / qtiles) * qpairs + ((ue - 1) % qtiles) / 2 + 1;
  const int64_t npairs = pe - pb, tail = sms > 0 ? npairs % sms : 0;
  r.pairs = npairs;
  r.tail_begin = ue;
  r.launches = 1;
  if (tail > 0 && tail <= sms / 2) {
    const int64_t first = pe - tail;   // the first tail pair
    const int64_t ut = (first / qpairs) * qtiles + (first % qpairs) * 2;
    r.pairs = npairs - tail;
    r.tail_begin = ut > ub ? ut : ub;
    r.tail_units = ue - r.tail_begin;
    r.launches = (r.pairs > 0 ? 1 : 0) + 1;
  }
  return r;
}

int attention_fwd(const AttnArgs& a, cudaStream_t st) {
  const int64_t BH = a.B * a.H;
  const int64_t qtiles = (a.Sq + 127) / 128, ktiles = (a.Sk + 127) / 128;
  const int64_t total = BH * qtiles;
  const int64_t ub = a.unit_begin, ue = a.unit_end < 0 ? total : a.unit_end;
  if (ub < 0 || ue > total || ub > ue) {
    set_last_error("vc_attention_fwd: unit range [%lld, %lld) outside [0, %lld)", (long long)ub, (long long)ue,
                   (long long)total);
    return VC_ERR_ARG;
  }
  if (ue == ub) return VC_OK;
  Maps m;
  const CUtensorMapSwizzle swk = a.D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (!make_map_3d(&m.q, a.q8, a.D, a.Sq, BH, a.D, 128, swk) || !make_map_3d(&m.k, a.k8, a.D, a.Sk, BH, a.D, 128, swk) ||
      !make_map_3d(&m.v, a.v8, ktiles * 128, a.D, BH, 128, a.D, CU_TENSOR_MAP_SWIZZLE_128B)) {
    set_last_error("vc_attention_fwd: cuTensorMapEncodeTiled failed");
    return VC_ERR_LAUNCH;
  }
  Params p;
  p.q8 = a.q8;
  p.qs = a.qs;
  p.ks = a.ks;
  p.vs = a.vs;
  p.means = reinterpret_cast<const __half*>(a.means);
  p.out = a.out;
  p.H = a.H;
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.osb = a.osb;
  p.osh = a.osh;
  p.oss = a.oss;
  p.nqs = a.qk_e4m3 ? qtiles : (a.Sq + 63) / 64 * 32;
  p.nks = a.qk_e4m3 ? (a.Sk + a.kqb - 1) / a.kqb : ktiles * 4;
  p.kq_tiles = a.qk_e4m3 ? a.kqb / 128 : 1;
  p.ktiles = ktiles;
  p.qtiles = qtiles;
  p.unit_begin = ub;
  p.unit_end = ue;
  // paired-tile kernel: the pairs (two consecutive Q tiles of one head) that meet [ub, ue)
  p.qpairs = (qtiles + 1) / 2;
  const int64_t pb = (ub / qtiles) * p.qpairs + (ub % qtiles) / 2;
  p.pair_begin = pb;
  p.sm_scale = a.sm_scale;
  p.exact_expcast = a.expcast == 2 ? 1 : 0;
  p.ctl_offset = a.config_control ? 8.0f : 8.807f;
  const int64_t units = ue - ub;
  const AttnPlan plan = attention_plan(qtiles, ub, ue, use_pair_only() ? 0 : sm_count());
  Split sp;
  sp.pairs = plan.pairs;
  if (plan.tail_units > 0) {
    sp.tail = p;
    sp.tail.unit_begin = plan.tail_begin;
    sp.tail_units = plan.tail_units;
  }
  if (a.out_dtype == VC_DTYPE_BF16)
    return a.D == 128 ? dispatch_flags<128, __nv_bfloat16>(a, m, p, units, sp, st)
                      : dispatch_flags<64, __nv_bfloat16>(a, m, p, units, sp, st);
  if (a.out_dtype == VC_DTYPE_F32)
    return a.D == 128 ? dispatch_flags<128, float>(a, m, p, units, sp, st)
                      : dispatch_flags<64, float>(a, m, p, units, sp, st);
  return a.D == 128 ? dispatch_flags<128, __half>(a, m, p, units, sp, st)
                    : dispatch_flags<64, __half>(a, m, p, units, sp, st);
}

cudaError_t attention_error_word(uint32_t* code, bool clear) { return read_tu_error_word(code, clear); }

int attention_resources(int head_dim, int64_t* out4) {
  cudaFuncAttributes fa;
  cudaError_t e = head_dim == 64 ? cudaFuncGetAttributes(&fa, vc_attention_kernel<64, __nv_bfloat16, true, false, false>)
                                 : cudaFuncGetAttributes(&fa, vc_attention_kernel<128, __nv_bfloat16, true, false, false>);
  if (e != cudaSuccess) return VC_ERR_LAUNCH;
  out4[0] = fa.numRegs;
  out4[1] = static_cast<int64_t>(fa.sharedSizeBytes);
  out4[2] = head_dim == 64 ? Smem<64>::kAlloc : Smem<128>::kAlloc;
  out4[3] = kThreads;
  return VC_OK;
}

}  // namespace vcb
