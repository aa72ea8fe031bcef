// Alternating-tile fused attention kernel (ExpCast, channel-scaled V, with or
// without 128-token block means): the default kernel for those modes.  Included by attention.cu
// after attention_softmax.cuh (register-level helpers).
//
// One CTA owns one 128-row Q tile of a (batch, head).  Warp roles (384 thr):
//   warps 0-3   softmax group 0: K tiles j = 0, 2, 4, ...
//   warps 4-7   softmax group 1: K tiles j = 1, 3, 5, ...
//               thread t owns row t (TMEM lane t) of its tile and the whole
//               128-key row; the only cross-group dependency is the running
//               row maximum m_{j-1}, handed over through shared memory with
//               an mbarrier per tile parity and per warp (a warp needs only
//               its own 32 rows, so no warp waits for another warp's skew)
//   warp 8      K producer (TMA, 4-deep ring);  warp 10  V producer (3-deep)
//   warp 9      TMEM allocator + QK^T issuer: preset + QK(j) are issued as
//               soon as K(j) has landed and the scores of tile j-2 have been read
//   warp 11     P.V issuer: PV(j) as soon as P(j) and V(j) are ready
//
// Tensor memory (496 of 512 columns):
//   S0 [0,128) S1 [128,256)   s32 scores of tiles j%2.  Before QK(j) the
//                             QK^T issuer presets S[j%2] to 0x4B400000 (the
//                             bits of 1.5*2^23) with one kind::f16 MMA,
//                             A.B^T = 2048 x 6144 from constant shared-memory
//                             operands, and QK^T accumulates onto it, so the
//                             scores arrive as the bit patterns of
//                             1.5*2^23 + s: floats without an int->float
//                             conversion and without register fills.
//   O  [256,256+D+16)         FP32 accumulator for the whole K loop; column D
//                             accumulates P.1 (the ExpCast denominator) via a
//                             row of E4M3 1.0 appended to every V tile
//   P0 [400,432) P1 [432,464) ExpCast bytes of tiles j%2 (A operand of P.V)
//   Q  [480,480+D/4)          int8 Q tile (A operand of Q.K^T)
// QF8 (E4M3 block Q/K of the Config contract's Hadamard path): Q and K are
// E4M3 bytes in the same layouts, QK^T is kind::f8f6f4 straight into FP32
// (no preset, so the softmax reads plain FP32 scores and skips the bias
// subtraction), and the scale factor of a tile is qs[q tile] * ks[key tile /
// (k_quant_block/128)] for all its columns.
// A group whose rows' maximum grew at tile j scales its lanes of O (and the
// denominator column) after PV(j-1) completes and before it releases P(j).
//
// Block means (V smoothing, channel scales): the payload is E4M3 of
// (V - mean_t)/s, so O needs mass_t * mean_t/s per tile besides P.V.  The
// tile masses come from the denominator column: the group of tile j reads
// column D after PV(j-1) (d_{j-1}), hands d_{j-1} alpha_j -- the column's
// value just before PV(j) -- to the other group through shared memory, and
// takes mass_{j-1} = d_{j-1} - (the value handed over for tile j-1).  The
// difference loses at most an ulp of the running denominator per tile.
// Masses are applied in batches of 8 tiles, one kind::f16 MMA (K = 16) per
// batch: row r of the 128x16 FP16 A operand holds [hi_0, lo_0, ..., hi_7,
// lo_7], the FP16 hi + lo split (exact to ~2^-22) of the batch's 8 masses,
// and channel c of the Dx16 B operand holds [mean_0, mean_0, ..., mean_7,
// mean_7] (written by the V producer warp, two batch buffers).  Until its
// batch is applied a mass waits in FP32 in shared memory at O's scale.
// Everything between PV(j-1) completing and P(j) being released is on the
// critical chain of the kernel, so the mass bookkeeping of tile j (mass_{j-1},
// the pending masses times alpha_j, the handover) runs after P(j) is
// released, while PV(j) executes; only the read of the denominator column
// stays before it.  Batch k is complete after tile 8k+8's bookkeeping, which
// also writes the batch's A operand (its masses are at O's scale for PV(8k+8))
// and arrives on a_full; the P.V issuer issues the batch's MMA right after
// PV(8k+8) and commits pv_done after it, so the next rescale of O follows it.
// After the last tile the group of parity T%2 completes the open batch
// (possibly partial, its unused slots zero) and that MMA precedes o_final.
//
// Barrier phases.  Every parity wait below is unconditional (taken on every
// tile), so a waiter can never be two phases behind its barrier, and no
// barrier can run ahead of its waiter (each next phase needs the waiter's own
// next release).  In particular the group at tile j always waits pv_done[j&1]
// for PV(j-1): that both frees P[j&1] (PV(j-2) precedes PV(j-1)) and orders
// the O rescale after PV(j-1).  A conditional wait on a barrier that advances
// every tile would alias phases and let the rescale race an MMA.
#pragma once

constexpr int kAltThreads = 384;
constexpr int kKS = 4;   // K ring depth
constexpr int kVS = 3;   // V ring depth
constexpr uint32_t kAColS0 = 0, kAColS1 = 128, kAColO = 256, kAColP0 = 400, kAColP1 = 432, kAColQ = 480;
// ExpCast code of an FP32 argument u (already rounded by its FMA): u * 2^-149
// lands on the denormal grid, whose round-to-nearest-even gives the bit
// pattern RNE(u) for 0 <= u < 2^23 and a negative (sign-bit) pattern for
// u < 0; cvt.pack.sat.u8.s32 then clamps to [0, 255] (u <= 120.5 here, as
// s <= m) and packs two codes per instruction.  No conversion-unit work, no
// explicit clamp.
constexpr uint32_t kDenormOne = 1u;   // bits of 2^-149

struct __align__(8) AltBarriers {
  uint64_t k_full[kKS], k_empty[kKS], v_full[kVS], v_empty[kVS];
  uint64_t q_ready, s_full[2], s_free[2], p_full[2], o_final;
  uint64_t pv_done[2];      // PV(i) completes pv_done[(i+1)&1]: the group of tile i+1 waits on it
  uint64_t m_ready[2][4];   // [tile parity][warp of the group]
  uint64_t mean_full[2];                      // block means: batch buffer k%2 of the means operand written
  uint64_t a_full;                            // block means: a batch's A operand written (count 128)
  uint64_t d_ready[2][4];                     // block means: denominator before PV(j) handed over
};

template <int D>
struct AltSmem {
  static constexpr int kK = 128 * D;
  static constexpr int kV = (D + 16) * 128;       // V^T rows + ones row + zero rows
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kKS * kK;
  static constexpr int kOffM = kOffV + kVS * kV;  // float [2][128] running maxima
  // block means: FP16 operands without swizzle, rows of 32 bytes (K = 16),
  // 8-row groups 256 bytes apart, the two K halves 128 bytes apart
  static constexpr int kOffD = kOffM + 2 * 128 * 4;        // float [2][128] denominators before PV(j)
  static constexpr int kOffPend = kOffD + 2 * 128 * 4;     // float4 [2][128]: row t's masses, slot j%8
  static constexpr int kMassA = 128 * 32;                    // 128 x 16 FP16 (mass hi, lo) x 8 tiles
  static constexpr int kOffMassA = kOffPend + 2 * 128 * 16;
  static constexpr int kMean = D * 32;                       // D x 16 FP16 (mean, mean) x 8 tiles
  static constexpr int kOffMean = kOffMassA + kMassA;        // two batch buffers
  // score preset operands: 128 x 16 FP16 each, element 0 of every row set
  // (2048 in A, 6144 in B), so A.B^T = 12582912 = 1.5*2^23 everywhere
  static constexpr int kOffPresetA = kOffMean + 2 * kMean;
  static constexpr int kOffPresetB = kOffPresetA + 128 * 32;
  static constexpr int kOffBar = kOffPresetB + 128 * 32;
  static constexpr int kOffSlot = kOffBar + int(sizeof(AltBarriers));
  static constexpr int kBytes = kOffSlot + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

// Byte offset of (row, first K element) in the no-swizzle 32-byte-row layout.
__device__ __forceinline__ int plain32_offset(int r) { return (r >> 3) * 256 + (r & 7) * 16; }

// Row t of the means MMA's A operand from row t's 8 pending masses: the first
// n as FP16 hi + lo pairs, the rest zero; then made visible to the MMA.
__device__ __forceinline__ void write_mass_operand(uint8_t* a, const float4* pend, int t, int n) {
  const float4 x0 = pend[t], x1 = pend[128 + t];
  const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  uint32_t wd[8];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const __half2 hi = __floats2half2_rn(x[i], x[i + 1]);
    const __half2 lo = __floats2half2_rn(__fsub_rn(x[i], __low2float(hi)), __fsub_rn(x[i + 1], __high2float(hi)));
    const uint32_t h = *reinterpret_cast<const uint32_t*>(&hi), l = *reinterpret_cast<const uint32_t*>(&lo);
    wd[i] = i < n ? __byte_perm(h, l, 0x5410) : 0u;           // [hi_i, lo_i]
    wd[i + 1] = i + 1 < n ? __byte_perm(h, l, 0x7632) : 0u;   // [hi_i+1, lo_i+1]
  }
  *reinterpret_cast<uint4*>(a + plain32_offset(t)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  *reinterpret_cast<uint4*>(a + plain32_offset(t) + 128) = make_uint4(wd[4], wd[5], wd[6], wd[7]);
  fence_proxy_async_smem();
}

template <int D, typename OutT, bool BV, bool QF8>
__global__ void __launch_bounds__(kAltThreads, 1)
    vc_attention_alt_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                            Params p) {
  using L = AltSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AltBarriers* bar = reinterpret_cast<AltBarriers*>(smem + L::kOffBar);
  float* mbuf = reinterpret_cast<float*>(smem + L::kOffM);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = p.unit_begin + blockIdx.x;
  const int64_t bh = unit / p.qtiles;
  const int64_t qt = unit - bh * p.qtiles;
  const int T = static_cast<int>(p.ktiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKS; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
    }
    mbar_init(&bar->q_ready, 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->s_full[b], 1);
      mbar_init(&bar->s_free[b], 128);
      mbar_init(&bar->p_full[b], 128);
      mbar_init(&bar->pv_done[b], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&bar->m_ready[b][q], 32);
    }
    for (int s = 0; s < 2; ++s) mbar_init(&bar->mean_full[s], 32);
    mbar_init(&bar->a_full, 128);
    for (int b = 0; b < 2; ++b)
      for (int q = 0; q < 4; ++q) mbar_init(&bar->d_ready[b][q], 32);
    mbar_init(&bar->o_final, 1);
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < kVS * 16 * 8; i += kAltThreads) {
    const int s = i / (16 * 8), r = (i / 8) % 16, c = i % 8;
    const uint32_t fill = r == 0 ? 0x38383838u : 0u;   // E4M3 1.0 in row D, zeros below
    *reinterpret_cast<uint4*>(smem + L::kOffV + s * L::kV + (D + r) * 128 + c * 16) = make_uint4(fill, fill, fill, fill);
  }
  for (int r = threadIdx.x; r < 128; r += kAltThreads) {
    *reinterpret_cast<uint4*>(smem + L::kOffPresetA + plain32_offset(r)) = make_uint4(0x6800u, 0, 0, 0);   // FP16 2048
    *reinterpret_cast<uint4*>(smem + L::kOffPresetA + plain32_offset(r) + 128) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(smem + L::kOffPresetB + plain32_offset(r)) = make_uint4(0x6E00u, 0, 0, 0);   // FP16 6144
    *reinterpret_cast<uint4*>(smem + L::kOffPresetB + plain32_offset(r) + 128) = make_uint4(0, 0, 0, 0);
  }
  if constexpr (BV) {
    // zero the pending masses and the FP16 operands once
    for (int i = threadIdx.x; i < (2 * 128 * 16 + L::kMassA + 2 * L::kMean) / 16; i += kAltThreads)
      *reinterpret_cast<uint4*>(smem + L::kOffPend + i * 16) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) tma_prefetch_desc(&tmk);
  if (warp == 10 && lane == 0) tma_prefetch_desc(&tmv);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    setmaxnreg_dec<56>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- K producer
      for (int j = 0; j < T; ++j) {
        const int s = j % kKS;
        if (j >= kKS && !mbar_wait(&bar->k_empty[s], ((j / kKS) & 1) ^ 1, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->k_full[s], L::kK);
        tma_load_3d(smem + L::kOffK + s * L::kK, &tmk, &bar->k_full[s], 0, j * 128, static_cast<int>(bh));
      }
    } else if (warp == 10 && !BV && lane == 0) {
      // ---------------------------------------------------------- V producer
      for (int j = 0; j < T; ++j) {
        const int s = j % kVS;
        if (j >= kVS && !mbar_wait(&bar->v_empty[s], ((j / kVS) & 1) ^ 1, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->v_full[s], D * 128);
        tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(bh));
      }
    } else if (warp == 10 && BV) {
      // ------------------------------------- V producer + means operand (warp)
      // lane l writes channels l, l+32, ... of tile j's means into slot j%8
      // of batch buffer (j/8)%2.  Buffer k%2 is written again for batch k+2
      // only after PV(8k+13) has completed (the v_empty wait below), and the
      // MMA of batch k precedes PV(8k+8), so no other release is needed.
      // Tile j+1's means are loaded while the warp waits for tile j+1's V slot.
      const uint16_t* mbase = reinterpret_cast<const uint16_t*>(p.means) + bh * T * D;
      uint32_t mnext[D / 32];
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) mnext[cc] = __ldg(mbase + lane + 32 * cc);
      for (int j = 0; j < T; ++j) {
        const int s = j % kVS;
        if (j >= kVS && !mbar_wait_warp(&bar->v_empty[s], ((j / kVS) & 1) ^ 1, kErrTimeoutProducer)) break;
        if (lane == 0) {
          mbar_expect_tx(&bar->v_full[s], D * 128);
          tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(bh));
        }
        uint32_t mcur[D / 32];
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          mcur[cc] = mnext[cc];
          if (j + 1 < T) mnext[cc] = __ldg(mbase + (j + 1) * D + lane + 32 * cc);
        }
        const int kb = j >> 3, slot = j & 7;
        uint8_t* mop = smem + L::kOffMean + (kb & 1) * L::kMean;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          const int c = lane + 32 * cc;
          const uint32_t m16 = mcur[cc];
          *reinterpret_cast<uint32_t*>(mop + plain32_offset(c) + (slot >> 2) * 128 + (slot & 3) * 4) = m16 | (m16 << 16);
          if (j == T - 1)   // the final batch's unused slots: zeros (their A entries are zero too)
            for (int z = slot + 1; z < 8; ++z)
              *reinterpret_cast<uint32_t*>(mop + plain32_offset(c) + (z >> 2) * 128 + (z & 3) * 4) = 0u;
        }
        if (slot == 7 || j == T - 1) {
          fence_proxy_async_smem();
          mbar_arrive(&bar->mean_full[kb & 1]);
        }
      }
    } else if (warp == 9 && lane == 0) {
      // ------------------------------------------------------- QK^T issuer
      // QK(j) goes as soon as K(j) has landed and the scores of tile j-2 have
      // been read out of S[j%2].
      // s32 <- s8 x s8, or with E4M3 block Q/K f32 <- e4m3 x e4m3
      constexpr uint32_t idesc_qk = QF8 ? idesc_make(1, 0, 0, 128, 128) : idesc_make(2, 1, 1, 128, 128);
      constexpr uint32_t idesc_preset = idesc_make(1, 0, 0, 128, 128); // f32 <- f16 x f16
      const uint64_t adesc_preset = smem_desc_plain(smem_u32(smem + L::kOffPresetA), 128, 256);
      const uint64_t bdesc_preset = smem_desc_plain(smem_u32(smem + L::kOffPresetB), 128, 256);
      const uint64_t kdesc0 = kmajor_desc<D>(smem_u32(smem + L::kOffK));
      constexpr uint64_t kStepK = (L::kK >> 4);                         // descriptor start-address units
      if (mbar_wait(&bar->q_ready, 0, kErrTimeoutMma)) {
        for (int j = 0; j < T; ++j) {
          const int s = j % kKS, b = j & 1;
          if (!mbar_wait(&bar->k_full[s], (j / kKS) & 1, kErrTimeoutMma)) break;
          // completion (j>>1) of s_free[b]: the scores of tile j-2 were read (or the initial release)
          if (!mbar_wait(&bar->s_free[b], (j >> 1) & 1, kErrTimeoutMma)) break;
          tc_fence_after();
          const uint64_t kd = kdesc0 + s * kStepK;
          const uint32_t scol = tmem + (b ? kAColS1 : kAColS0);
          if constexpr (QF8) {
            // FP32 scores straight from the MMA: no preset
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              mma_f8_ts(scol, tmem + kAColQ + kk * 8, kd + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
          } else {
            mma_f16_ss(scol, adesc_preset, bdesc_preset, idesc_preset, 0u);   // S = the bits of 1.5*2^23
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              mma_i8_ts(scol, tmem + kAColQ + kk * 8, kd + 2 * kk, idesc_qk, 1u);   // onto the preset
          }
          mma_commit(&bar->k_empty[s]);
          mma_commit(&bar->s_full[b]);
        }
      }
    } else if (warp == 11 && lane == 0) {
      // ---------------------------------------------------------- P.V issuer
      // PV(j) goes as soon as P(j) and V(j) are ready; P has its own TMEM
      // buffers, so this thread never waits on the QK^T issuer.
      constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 128, D + 16);  // f32 <- e4m3 x e4m3
      constexpr uint32_t idesc_mean = idesc_make(1, 0, 0, 128, D);     // f32 <- f16 x f16
      const uint64_t vdesc0 = smem_desc_sw128(smem_u32(smem + L::kOffV));
      constexpr uint64_t kStepV = (L::kV >> 4);
      const uint64_t massdesc = smem_desc_plain(smem_u32(smem + L::kOffMassA), 128, 256);
      const uint64_t meandesc0 = smem_desc_plain(smem_u32(smem + L::kOffMean), 128, 256);
      constexpr uint64_t kStepMean = (L::kMean >> 4);
      bool ok = true;
      for (int j = 0; j < T && ok; ++j) {
        const int s = j % kVS, b = j & 1;
        ok = mbar_wait(&bar->p_full[b], (j >> 1) & 1, kErrTimeoutMma) &&
             mbar_wait(&bar->v_full[s], (j / kVS) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint64_t vd = vdesc0 + s * kStepV;
        const uint32_t pcol = tmem + (b ? kAColP1 : kAColP0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ts(tmem + kAColO, pcol + kk * 8, vd + 2 * kk, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bar->v_empty[s]);
        if (BV && j >= 8 && (j & 7) == 0) {
          // batch kb, completed by tile j's bookkeeping while PV(j) runs:
          // O += sum over the batch's tiles of (mass alpha...) x mean
          const int kb = (j >> 3) - 1;
          ok = mbar_wait(&bar->a_full, kb & 1, kErrTimeoutMma) &&
               mbar_wait(&bar->mean_full[kb & 1], (kb >> 1) & 1, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          mma_f16_ss(tmem + kAColO, massdesc, meandesc0 + (kb & 1) * kStepMean, idesc_mean, 1u);
        }
        mma_commit(&bar->pv_done[(j + 1) & 1]);
      }
      if constexpr (BV) {
        // the open batch: its A operand comes from the group of parity T%2
        const int kb = (T - 1) >> 3;
        if (ok) ok = mbar_wait(&bar->p_full[T & 1], (T >> 1) & 1, kErrTimeoutMma) &&
                     mbar_wait(&bar->mean_full[kb & 1], (kb >> 1) & 1, kErrTimeoutMma);
        if (ok) {
          tc_fence_after();
          mma_f16_ss(tmem + kAColO, massdesc, meandesc0 + (kb & 1) * kStepMean, idesc_mean, 1u);
        }
      }
      if (ok) mma_commit(&bar->o_final);
    }
  } else {
    setmaxnreg_inc<224>();
    // ------------------------------------------------------------ softmax group w
    const int w = warp >> 2;
    const int quarter = warp & 3;
    const int t = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t row = qt * 128 + t;
    const bool row_valid = row < p.Sq;
    if (w == 0) {
      uint32_t qw[32];
      const int8_t* qrow = p.q8 + (bh * p.Sq + row) * D;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        uint4 u = row_valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + i) : make_uint4(0, 0, 0, 0);
        qw[4 * i] = u.x; qw[4 * i + 1] = u.y; qw[4 * i + 2] = u.z; qw[4 * i + 3] = u.w;
      }
      if constexpr (D == 128) tmem_st32(tmem + lane_base + kAColQ, qw);
      else tmem_st16(tmem + lane_base + kAColQ, qw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->q_ready);
    }
    // INT8: the Sage per-thread Q scale of the row; E4M3 blocks: one scale per 128-row Q tile
    const float qscale = !row_valid ? 0.f : QF8 ? p.qs[bh * p.nqs + qt] : p.qs[bh * p.nqs + (row >> 4) * 8 + (row & 7)];
    const float scale = p.sm_scale;
    const uint64_t bias2 = pk2f(kBias, kBias);
    const uint64_t tiny2 = pk2(kDenormOne, kDenormOne);
    const uint64_t expa2 = pk2f(kExpA, kExpA), expb2 = pk2f(kExpB, kExpB);
    mbar_arrive(&bar->s_free[w]);   // S[w] is free for this group's first tile
    bool ok = true;
    // K scales of a tile: INT8 four groups (index tile*4 + (key%8)/2); E4M3 blocks one scale per kq_tiles tiles
    auto load_ks = [&](int jj) -> float4 {
      if constexpr (QF8) {
        const float v = __ldg(p.ks + bh * p.nks + jj / p.kq_tiles);
        return make_float4(v, v, v, v);
      } else {
        return __ldg(reinterpret_cast<const float4*>(p.ks + bh * p.nks + jj * 4));
      }
    };
    float4 ksv_next = w < T ? load_ks(w) : make_float4(1, 1, 1, 1);
    for (int j = w; j < T; j += 2) {
      const int b = j & 1;   // == w
      const float4 ksv = ksv_next;
      if (j + 2 < T) ksv_next = load_ks(j + 2);
      const uint32_t scol = tmem + lane_base + (b ? kAColS1 : kAColS0);
      ok = mbar_wait_warp(&bar->s_full[b], (j >> 1) & 1, kErrTimeoutSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t raw[128];
      tmem_ld32(scol + 0, *reinterpret_cast<uint32_t(*)[32]>(raw + 0));
      tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(raw + 32));
      tmem_ld32(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(raw + 64));
      tmem_ld32(scol + 96, *reinterpret_cast<uint32_t(*)[32]>(raw + 96));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bar->s_free[b]);   // QK(j+2) may now overwrite S[b]
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
        if constexpr (QF8) {
          if (mx > -__int_as_float(0x7f800000)) lmax = fmaxf(lmax, __fmul_rn(mx, f1[g]));
        } else {
          if (mx > 0.f) lmax = fmaxf(lmax, __fmul_rn(__fsub_rn(mx, kBias), f1[g]));
        }
      }
      // running maximum handed over from the other group's previous tile
      float mprev = -5000000.0f;
      if (j >= 1) {
        ok = mbar_wait_warp(&bar->m_ready[b ^ 1][quarter], ((j - 1) >> 1) & 1, kErrTimeoutSoftmax);
        if (!ok) break;
        mprev = mbuf[(b ^ 1) * 128 + t];
      }
      const float mn = fmaxf(mprev, lmax);
      const float alpha = expf(mprev - mn);
      mbuf[b * 128 + t] = mn;
      mbar_arrive(&bar->m_ready[b][quarter]);
      uint32_t pw[32];
      float gain[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) gain[g] = __fmul_rn(f1[g], kExpA);
      const float cb = __fmaf_rn(-mn, kExpA, kExpB);
      const bool safe = !p.exact_expcast && fabsf(mn) <= 128.f && scale >= 1.1754943508222875e-38f &&
                        isfinite(gain[0]) && isfinite(gain[1]) && isfinite(gain[2]) && isfinite(gain[3]);
      if (__all_sync(0xffffffffu, safe)) {
        uint64_t gain2[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) gain2[g] = pk2f(gain[g], gain[g]);
        const uint64_t cb2 = pk2f(cb, cb);
#pragma unroll
        for (int wd = 0; wd < 32; ++wd) {
          uint32_t e[4];
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int c = 4 * wd + 2 * q2;
            const int g = (c >> 1) & 3;
            // u = fma(float(raw), RN(f A), fma(-m, A, B)) (the folded affine encoder)
            const uint64_t x2 = QF8 ? pk2(raw[c], raw[c + 1]) : f2_sub(pk2(raw[c], raw[c + 1]), bias2);
            const uint64_t u2 = f2_fma(x2, gain2[g], cb2);
            up2(f2_mul(u2, tiny2), e[2 * q2], e[2 * q2 + 1]);
          }
          pw[wd] = pack_u8x2(e[1], e[0], pack_u8x2(e[3], e[2], 0u));
        }
      } else {
        const uint64_t m2 = pk2f(mn, mn);
#pragma unroll
        for (int wd = 0; wd < 32; ++wd) {
          uint32_t e[4];
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int c = 4 * wd + 2 * q2;
            const int g = (c >> 1) & 3;
            // u = fma(RN(RN(float(raw) f) - m), A, B) (the unfused contract)
            const uint64_t x2 = QF8 ? pk2(raw[c], raw[c + 1]) : f2_sub(pk2(raw[c], raw[c + 1]), bias2);
            const uint64_t sh = f2_sub(f2_mul(x2, pk2f(f1[g], f1[g])), m2);
            up2(f2_mul(f2_fma(sh, expa2, expb2), tiny2), e[2 * q2], e[2 * q2 + 1]);
          }
          pw[wd] = pack_u8x2(e[1], e[0], pack_u8x2(e[3], e[2], 0u));
        }
      }
      // PV(j-1) complete (hence PV(j-2) too): P[b] is free and O may be rescaled
      uint32_t draw = 0;   // block means: denominator column after PV(j-1), read before P(j) is released
      if (j >= 1) {
        ok = mbar_wait_warp(&bar->pv_done[b], ((j - 1) >> 1) & 1, kErrTimeoutSoftmax);
        if (!ok) break;
        if constexpr (BV) {
          tc_fence_after();
          draw = tmem_ld1(tmem + lane_base + kAColO + D);
        }
      }
      // rescale O (and the denominator column) between PV(j-1) and PV(j) if any max grew
      const bool grew = j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f);
      if (grew) {
        tc_fence_after();
        const uint32_t ocol = tmem + lane_base + kAColO;
        const uint64_t alpha2 = pk2f(alpha, alpha);
        // all of O's columns in flight at once (the score registers are free by
        // now): one tensor-memory load latency on the chain instead of D/32
        uint32_t o[D];
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tmem_ld32(ocol + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(o + cc * 32));
        // the denominator: column D (columns D+1.. of the block only ever hold zeros)
        if constexpr (!BV) draw = tmem_ld1(ocol + D);
        tmem_wait_ld_reg(draw);
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tmem_wait_ld_tie32(o + cc * 32);
#pragma unroll
        for (int i = 0; i < D / 2; ++i) up2(f2_mul(pk2(o[2 * i], o[2 * i + 1]), alpha2), o[2 * i], o[2 * i + 1]);
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tmem_st32(ocol + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(o + cc * 32));
        tmem_st1(ocol + D, __float_as_uint(__fmul_rn(__uint_as_float(draw), alpha)));
      }
      float4* pend = reinterpret_cast<float4*>(smem + L::kOffPend);
      float* dbuf = reinterpret_cast<float*>(smem + L::kOffD);
      // P(j) into this group's P buffer (PV(j-2) has consumed it, see above)
      tc_fence_after();
      tmem_st32(tmem + lane_base + (b ? kAColP1 : kAColP0), pw);
      tmem_wait_st();
      if constexpr (BV) tmem_wait_ld_reg(draw);   // the column read completes before PV(j) may start
      tc_fence_before();
      mbar_arrive(&bar->p_full[b]);
      if constexpr (BV) {
        // bookkeeping off the critical chain, while PV(j) runs: the pending
        // masses times alpha_j, mass_{j-1} alpha_j into slot (j-1)%8, the A
        // operand when that completes a batch, the handover to tile j+1
        const float dcur = __uint_as_float(draw);
        if (j >= 1) {
          ok = mbar_wait_warp(&bar->d_ready[b ^ 1][quarter], ((j - 1) >> 1) & 1, kErrTimeoutSoftmax);
          if (!ok) break;
          const int slot = (j - 1) & 7;
          if (grew) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float4 v = pend[h * 128 + t];
              v.x = __fmul_rn(v.x, alpha); v.y = __fmul_rn(v.y, alpha);
              v.z = __fmul_rn(v.z, alpha); v.w = __fmul_rn(v.w, alpha);
              pend[h * 128 + t] = v;
            }
          }
          reinterpret_cast<float*>(pend + (slot >> 2) * 128 + t)[slot & 3] =
              __fmul_rn(__fsub_rn(dcur, dbuf[(b ^ 1) * 128 + t]), alpha);
          if (slot == 7) {
            write_mass_operand(smem + L::kOffMassA, pend, t, 8);
            mbar_arrive(&bar->a_full);
          }
        }
        // the denominator column just before PV(j), for the group of tile j+1
        dbuf[b * 128 + t] = j >= 1 ? __fmul_rn(dcur, alpha) : 0.f;
        mbar_arrive(&bar->d_ready[b][quarter]);
      }
    }
    if constexpr (BV) {
      // the group of parity T%2 completes the open batches for the last means MMAs
      if (ok && (T & 1) == w) {
        ok = mbar_wait_warp(&bar->pv_done[T & 1], ((T - 1) >> 1) & 1, kErrTimeoutSoftmax) &&
             mbar_wait_warp(&bar->d_ready[(T - 1) & 1][quarter], ((T - 1) >> 1) & 1, kErrTimeoutSoftmax);
        if (ok) {
          tc_fence_after();
          const float dlast = __uint_as_float(tmem_ld1(tmem + lane_base + kAColO + D));
          tmem_wait_ld();
          float4* pend = reinterpret_cast<float4*>(smem + L::kOffPend);
          const int slot = (T - 1) & 7;
          reinterpret_cast<float*>(pend + (slot >> 2) * 128 + t)[slot & 3] =
              __fsub_rn(dlast, reinterpret_cast<const float*>(smem + L::kOffD)[((T - 1) & 1) * 128 + t]);
          write_mass_operand(smem + L::kOffMassA, pend, t, slot + 1);
          tc_fence_before();
          mbar_arrive(&bar->p_full[T & 1]);
        }
      }
    }
    // epilogue: group w writes output channels [w*D/2, (w+1)*D/2)
    if (ok) ok = mbar_wait_warp(&bar->o_final, 0, kErrTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      uint32_t dn[16];
      tmem_ld16(tmem + lane_base + kAColO + D, dn);
      tmem_wait_ld();
      const float denom = __uint_as_float(dn[0]);
      OutT* orow = reinterpret_cast<OutT*>(p.out) + (bh / p.H) * p.osb + (bh % p.H) * p.osh + row * p.oss;
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int cbase = w * (D / 2) + cc * 32;
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + kAColO + cbase, o);
        tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int c0 = cbase + c8 * 8;
            const float4 vsa = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c0));
            const float4 vsb = __ldg(reinterpret_cast<const float4*>(p.vs + bh * D + c0 + 4));
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
            for (int ww = 0; ww < kWords; ++ww) reinterpret_cast<uint4*>(orow + c0)[ww] = u[ww];
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
