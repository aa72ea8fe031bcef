// Paired-tile fused attention kernel (ExpCast, channel-scaled V, with or
// without 128-token block means): the default kernel for those modes.
// Included by attention.cu after attention_alt.cuh.
//
// One CTA owns two 128-row Q tiles of one (batch, head): tile A = 2p and
// tile B = 2p + 1.  Each softmax group owns one tile for the whole K loop,
// so every tile is an independent online-softmax chain
//   QK_X(j) -> scores -> max, ExpCast codes -> P_X(j) -> PV_X(j) -> rescale
// with its running maximum in registers: the two chains only share the K/V
// stream.  While one group waits for its own PV(j-1) (the rescale of O has to
// follow it), the other group's work keeps the tensor pipe busy.
//
// Warp roles (384 threads):
//   warps 0-3   softmax group A (tile A), thread t owns row t = TMEM lane t
//   warps 4-7   softmax group B (tile B)
//   warp 8      K producer (TMA, 4-deep ring) [+ both Q tiles once at D = 128]
//   warp 9      TMEM allocator + QK^T issuer: QK_A(j), QK_B(j), QK_A(j+1), ...
//   warp 10     V producer (3-deep ring) [+ the block means operand]
//   warp 11     P.V issuer: PV_A(j), PV_B(j), PV_A(j+1), ... [+ means MMAs]
// The issuers run their loops in the whole warp (descriptor arithmetic stays
// warp-uniform) and one elected lane issues each MMA and commit.
//
// QK^T is kind::i8 (kind::f8f6f4 for E4M3 block Q/K).  At D = 64, Q lives in
// tensor memory (each softmax thread stores its own row) and QK^T reads only
// K from shared memory: measured on B200, an M=128 N=128 K=32 MMA takes about
// 73 cycles with A in tensor memory and about 103 with both operands in
// shared memory.  At D = 128 there is no room for Q in tensor memory next to
// P, and P there is worth more (moving P to shared memory to make room was
// measured 3% slower), so Q is staged in shared memory by TMA.  Before each
// INT8 QK^T one kind::f16 MMA presets the score slot to the bits of 1.5*2^23
// (2048 x 6144 from constant operands; at D = 128 the A operand sits in
// tensor memory), so s32 scores read back as the floats 1.5*2^23 + s.
//
// Tensor memory (512 columns):
//   S [0,128): one score slot, used in the order A(0), B(0), A(1), ...
//   D = 128: O_A [128,272)  O_B [288,432)  preset A operand [432,440)
//            P_A [448,480)  P_B [480,512);  Q_A, Q_B in shared memory
//   D = 64:  O_A [256,336)  O_B [336,416)  Q_A [416,432)  Q_B [432,448)
//            P_A [448,480)  P_B [480,512)
// QK^T issue n = 2j + X overwrites the slot once the scores of issue n - 1
// (the other chain's) have been read, so the two groups alternate.  At
// D = 128 a second slot does not fit; at D = 64 it does, but two slots let
// the groups run in phase (both computing, then both waiting) and measured
// 8% slower.  The round trip (issuer wake-up, preset and QK^T MMAs, group
// wake-up, score read) bounds the tile period.
// O_X holds D FP32 output columns plus a 16-column block whose first column
// accumulates P.1 (the ExpCast denominator) through a row of E4M3 1.0
// appended to every V tile.
//
// Block means (V smoothing, channel scales): O_X needs mass_t * mean_t/s per
// tile besides P.V.  The mass of tile t is the growth of the denominator
// column over PV_X(t): group X reads the column after PV_X(t) (it waits for
// PV_X(t) before tile t+1 anyway) and keeps the value it had just before
// PV_X(t) in a register.  Pending masses wait in registers at O's scale;
// every 8 tiles one kind::f16 MMA (K = 16) adds them: row r of the 128x16
// FP16 A operand holds [hi_0, lo_0, ..., hi_7, lo_7], the FP16 hi + lo split
// (exact to ~2^-22) of the batch's masses, and channel c of the Dx16 B
// operand holds [mean_0, mean_0, ..., mean_7, mean_7] (written by the V
// producer warp, two batch buffers shared by both tiles).  Batch k is
// complete after tile 8k+8's bookkeeping (its masses are then at O's scale for
// PV_X(8k+8)); the P.V issuer issues its MMA right after PV_X(8k+8) and
// commits pv_done_X after it, so the next rescale of O follows it.
//
// Tail balance.  A CTA with one tile would cost about as much as a pair (one
// group's softmax work per tile sets its period), so when the last wave of
// pairs would be at most half full the host runs those pairs' tiles on the
// alternating-tile kernel instead (both groups on one tile, about 0.6 of a
// pair period) and launches this kernel on the full waves only.
//
// Barrier phases.  Every wait is unconditional and taken once per phase in
// order, and no barrier can complete a phase ahead of its waiter: s_full_X,
// p_full_X and pv_done_X advance once per tile of chain X, each only after
// the waiter's own previous release; s_free_X gates the next QK^T into the
// slot, which itself precedes chain X's next scores.
#pragma once

constexpr int kPairThreads = 384;
constexpr int kPKS = 4;   // K ring depth
constexpr int kPVS = 3;   // V ring depth

template <int D>
struct PairCols {
  static constexpr bool kQTmem = D == 64;                     // Q in tensor memory (else shared, by TMA)
  static constexpr bool kPresetTmem = D == 128;               // preset A operand in tensor memory
  static constexpr uint32_t kS = 0;                           // the score slot
  static constexpr uint32_t kOA = D == 64 ? 256 : 128;
  static constexpr uint32_t kOB = D == 64 ? 336 : 288;
  static constexpr uint32_t kQA = 416, kQB = 432;             // D = 64 only
  static constexpr uint32_t kPA = 448, kPB = 480;
  static constexpr uint32_t kPresetA = 432;                   // D = 128 only
  static_assert(kOA + D + 16 <= kOB && kOB + D + 16 <= (D == 64 ? kQA : kPresetA), "tensor-memory columns overlap");
};

struct __align__(8) PairBarriers {
  uint64_t k_full[kPKS], k_empty[kPKS], v_full[kPVS], v_empty[kPVS];
  uint64_t q_ready[2];     // Q in tensor memory: tile X's rows stored (count 128)
  uint64_t q_full;         // Q in shared memory: both tiles loaded (TMA)
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], o_final[2];
  uint64_t mean_full[2];   // block means: batch buffer k%2 of the means operand written
  uint64_t a_full[2];      // block means: tile X's mass operand of a batch written (count 128)
};

template <int D>
struct PairSmem {
  static constexpr int kK = 128 * D;              // K stage
  static constexpr int kV = (D + 16) * 128;       // V^T rows + ones row + zero rows
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kPKS * kK;
  static constexpr int kOffQ = kOffV + kPVS * kV;                 // Q_A, Q_B (Q in shared memory)
  static constexpr int kOffMassA = kOffQ + (PairCols<D>::kQTmem ? 0 : 2 * kK);
  static constexpr int kMassA = 128 * 32;                         // 128 x 16 FP16 per tile
  static constexpr int kMean = D * 32;                            // D x 16 FP16
  static constexpr int kOffMean = kOffMassA + 2 * kMassA;         // two batch buffers
  static constexpr int kOffPresetA = kOffMean + 2 * kMean;
  static constexpr int kOffPresetB = kOffPresetA + 128 * 32;
  static constexpr int kOffBar = kOffPresetB + 128 * 32;
  static constexpr int kOffSlot = kOffBar + int(sizeof(PairBarriers));
  static constexpr int kBytes = kOffSlot + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kOffQ % 1024 == 0, "Q tiles need 1024-byte alignment (128-byte swizzle)");
  static_assert(kAlloc <= 227 * 1024, "shared memory");
};

// Row t of a means MMA's A operand from the row's pending masses: the first
// n as FP16 hi + lo pairs, the rest zero; then made visible to the MMA.
__device__ __forceinline__ void write_mass_row(uint8_t* a, const float (&x)[8], int t, int n) {
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
__global__ void __launch_bounds__(kPairThreads, 1)
    vc_attention_pair_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                             const __grid_constant__ CUtensorMap tmv, Params p) {
  using L = PairSmem<D>;
  using C = PairCols<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBarriers* bar = reinterpret_cast<PairBarriers*>(smem + L::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pair = p.pair_begin + static_cast<int64_t>(blockIdx.x);
  const int64_t bh = pair / p.qpairs;
  const int64_t qt0 = (pair - bh * p.qpairs) * 2;   // tile A; tile B = qt0 + 1
  const int T = static_cast<int>(p.ktiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPKS; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
    }
    for (int s = 0; s < kPVS; ++s) {
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bar->q_ready[x], 128);
      mbar_init(&bar->s_full[x], 1);
      mbar_init(&bar->s_free[x], 128);
      mbar_init(&bar->p_full[x], 128);
      mbar_init(&bar->pv_done[x], 1);
      mbar_init(&bar->o_final[x], 1);
      mbar_init(&bar->mean_full[x], 32);
      mbar_init(&bar->a_full[x], 128);
    }
    mbar_init(&bar->q_full, 1);
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < kPVS * 16 * 8; i += kPairThreads) {
    const int s = i / (16 * 8), r = (i / 8) % 16, c = i % 8;
    const uint32_t fill = r == 0 ? 0x38383838u : 0u;   // E4M3 1.0 in row D, zeros below
    *reinterpret_cast<uint4*>(smem + L::kOffV + s * L::kV + (D + r) * 128 + c * 16) = make_uint4(fill, fill, fill, fill);
  }
  for (int r = threadIdx.x; r < 128; r += kPairThreads) {
    *reinterpret_cast<uint4*>(smem + L::kOffPresetA + plain32_offset(r)) = make_uint4(0x6800u, 0, 0, 0);   // FP16 2048
    *reinterpret_cast<uint4*>(smem + L::kOffPresetA + plain32_offset(r) + 128) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(smem + L::kOffPresetB + plain32_offset(r)) = make_uint4(0x6E00u, 0, 0, 0);   // FP16 6144
    *reinterpret_cast<uint4*>(smem + L::kOffPresetB + plain32_offset(r) + 128) = make_uint4(0, 0, 0, 0);
  }
  if constexpr (BV) {
    for (int i = threadIdx.x; i < (2 * L::kMassA + 2 * L::kMean) / 16; i += kPairThreads)
      *reinterpret_cast<uint4*>(smem + L::kOffMassA + i * 16) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    if constexpr (!C::kQTmem) tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
  }
  if (warp == 10 && lane == 0) tma_prefetch_desc(&tmv);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    setmaxnreg_dec<56>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------------- K producer
      if constexpr (!C::kQTmem) {
        // both Q tiles; a tile B past the end of the head reads as zeros (its rows are never written)
        mbar_expect_tx(&bar->q_full, 2 * L::kK);
        tma_load_3d(smem + L::kOffQ, &tmq, &bar->q_full, 0, static_cast<int>(qt0 * 128), static_cast<int>(bh));
        tma_load_3d(smem + L::kOffQ + L::kK, &tmq, &bar->q_full, 0, static_cast<int>(qt0 * 128 + 128),
                    static_cast<int>(bh));
      }
      for (int j = 0; j < T; ++j) {
        const int s = j % kPKS;
        if (j >= kPKS && !mbar_wait(&bar->k_empty[s], ((j / kPKS) & 1) ^ 1, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->k_full[s], L::kK);
        tma_load_3d(smem + L::kOffK + s * L::kK, &tmk, &bar->k_full[s], 0, j * 128, static_cast<int>(bh));
      }
    } else if (warp == 10 && !BV && lane == 0) {
      // ---------------------------------------------------------- V producer
      for (int j = 0; j < T; ++j) {
        const int s = j % kPVS;
        if (j >= kPVS && !mbar_wait(&bar->v_empty[s], ((j / kPVS) & 1) ^ 1, kErrTimeoutProducer)) break;
        mbar_expect_tx(&bar->v_full[s], D * 128);
        tma_load_3d(smem + L::kOffV + s * L::kV, &tmv, &bar->v_full[s], j * 128, 0, static_cast<int>(bh));
      }
    } else if (warp == 10 && BV) {
      // ------------------------------------- V producer + means operand (warp)
      // lane l writes channels l, l+32, ... of tile j's means into slot j%8 of
      // batch buffer (j/8)%2.  Buffer k%2 is written again for batch k+2 only
      // after both tiles' PV(8k+13) have completed (the v_empty wait below),
      // and both means MMAs of batch k are issued right after PV_X(8k+8).
      const uint16_t* mbase = reinterpret_cast<const uint16_t*>(p.means) + bh * T * D;
      uint32_t mnext[D / 32];
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) mnext[cc] = __ldg(mbase + lane + 32 * cc);
      for (int j = 0; j < T; ++j) {
        const int s = j % kPVS;
        if (j >= kPVS && !mbar_wait_warp(&bar->v_empty[s], ((j / kPVS) & 1) ^ 1, kErrTimeoutProducer)) break;
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
    } else if (warp == 9) {
      // ------------------------------------------------------- QK^T issuer
      // issue n = 2j + X into the slot once the scores of issue n - 1 are read
      constexpr uint32_t idesc_qk = QF8 ? idesc_make(1, 0, 0, 128, 128) : idesc_make(2, 1, 1, 128, 128);
      constexpr uint32_t idesc_preset = idesc_make(1, 0, 0, 128, 128);   // f32 <- f16 x f16
      const uint64_t adesc_preset = smem_desc_plain(smem_u32(smem + L::kOffPresetA), 128, 256);
      const uint64_t bdesc_preset = smem_desc_plain(smem_u32(smem + L::kOffPresetB), 128, 256);
      const uint64_t kdesc0 = kmajor_desc<D>(smem_u32(smem + L::kOffK));
      const uint64_t qdesc0 = kmajor_desc<D>(smem_u32(smem + L::kOffQ));
      constexpr uint64_t kStep = (L::kK >> 4);   // descriptor start-address units per K stage / Q tile
      bool ok = mbar_wait_warp(&bar->q_ready[0], 0, kErrTimeoutMma) && mbar_wait_warp(&bar->q_ready[1], 0, kErrTimeoutMma);
      if constexpr (!C::kQTmem) ok = ok && mbar_wait_warp(&bar->q_full, 0, kErrTimeoutMma);
      for (int j = 0; j < T && ok; ++j) {
        const int s = j % kPKS;
        if (!mbar_wait_warp(&bar->k_full[s], (j / kPKS) & 1, kErrTimeoutMma)) break;
        const uint64_t kd = kdesc0 + s * kStep;
        for (int x = 0; x < 2; ++x) {
          // issue n = 2j + x after the read of issue n - 1 (chain prev & 1, its
          // (prev >> 1)-th read)
          const int prev = 2 * j + x - 1;
          const bool waited = prev < 0 || mbar_wait_warp(&bar->s_free[prev & 1], (prev >> 1) & 1, kErrTimeoutMma);
          if (!waited) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t scol = tmem + C::kS;
          const uint32_t qcol = tmem + (x ? C::kQB : C::kQA);
          const uint64_t qd = qdesc0 + x * kStep;
          if (elect_one()) {
            if constexpr (!QF8) {
              // S = the bits of 1.5*2^23, then QK^T accumulates onto it
              if constexpr (C::kPresetTmem) mma_f16_ts(scol, tmem + C::kPresetA, bdesc_preset, idesc_preset, 0u);
              else mma_f16_ss(scol, adesc_preset, bdesc_preset, idesc_preset, 0u);
            }
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk) {
              const uint32_t acc = QF8 ? (kk > 0 ? 1u : 0u) : 1u;
              if constexpr (C::kQTmem) {
                if constexpr (QF8) mma_f8_ts(scol, qcol + kk * 8, kd + 2 * kk, idesc_qk, acc);
                else mma_i8_ts(scol, qcol + kk * 8, kd + 2 * kk, idesc_qk, acc);
              } else {
                if constexpr (QF8) mma_f8_ss(scol, qd + 2 * kk, kd + 2 * kk, idesc_qk, acc);
                else mma_i8_ss(scol, qd + 2 * kk, kd + 2 * kk, idesc_qk, acc);
              }
            }
            mma_commit(&bar->s_full[x]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) mma_commit(&bar->k_empty[s]);
        __syncwarp();
      }
    } else if (warp == 11) {
      // ---------------------------------------------------------- P.V issuer
      constexpr uint32_t idesc_pv = idesc_make(1, 0, 0, 128, D + 16);  // f32 <- e4m3 x e4m3
      constexpr uint32_t idesc_mean = idesc_make(1, 0, 0, 128, D);     // f32 <- f16 x f16
      const uint64_t vdesc0 = smem_desc_sw128(smem_u32(smem + L::kOffV));
      constexpr uint64_t kStepV = (L::kV >> 4);
      const uint64_t meandesc0 = smem_desc_plain(smem_u32(smem + L::kOffMean), 128, 256);
      constexpr uint64_t kStepMean = (L::kMean >> 4);
      constexpr uint64_t kStepMass = (L::kMassA >> 4);
      const uint64_t massdesc0 = smem_desc_plain(smem_u32(smem + L::kOffMassA), 128, 256);
      bool ok = true;
      for (int j = 0; j < T && ok; ++j) {
        const int s = j % kPVS;
        if (!mbar_wait_warp(&bar->v_full[s], (j / kPVS) & 1, kErrTimeoutMma)) break;
        const uint64_t vd = vdesc0 + s * kStepV;
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait_warp(&bar->p_full[x], j & 1, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ocol = tmem + (x ? C::kOB : C::kOA);
          if (elect_one()) {
            const uint32_t pcol = tmem + (x ? C::kPB : C::kPA);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f8_ts(ocol, pcol + kk * 8, vd + 2 * kk, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          __syncwarp();
          if (BV && j >= 8 && (j & 7) == 0) {
            // batch kb of tile X, completed by its tile-j bookkeeping while PV_X(j) runs
            const int kb = (j >> 3) - 1;
            if (!mbar_wait_warp(&bar->a_full[x], kb & 1, kErrTimeoutMma) ||
                !mbar_wait_warp(&bar->mean_full[kb & 1], (kb >> 1) & 1, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (elect_one())
              mma_f16_ss(ocol, massdesc0 + x * kStepMass, meandesc0 + (kb & 1) * kStepMean, idesc_mean, 1u);
            __syncwarp();
          }
          if (elect_one()) mma_commit(&bar->pv_done[x]);
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) mma_commit(&bar->v_empty[s]);
        __syncwarp();
      }
      for (int x = 0; x < 2; ++x) {
        if constexpr (BV) {
          // the open batch of tile X, written by its group after the loop
          const int kb = (T - 1) >> 3;
          if (ok) ok = mbar_wait_warp(&bar->a_full[x], kb & 1, kErrTimeoutMma) &&
                       mbar_wait_warp(&bar->mean_full[kb & 1], (kb >> 1) & 1, kErrTimeoutMma);
          if (ok) {
            tc_fence_after();
            if (elect_one())
              mma_f16_ss(tmem + (x ? C::kOB : C::kOA), massdesc0 + x * kStepMass, meandesc0 + (kb & 1) * kStepMean,
                         idesc_mean, 1u);
            __syncwarp();
          }
        }
        if (ok && elect_one()) mma_commit(&bar->o_final[x]);
        __syncwarp();
      }
    }
  } else {
    setmaxnreg_inc<224>();
    // ------------------------------------------------------ softmax group X
    const int x = warp >> 2;
    const int quarter = warp & 3;
    const int t = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t qt = qt0 + x;
    const int64_t row = qt * 128 + t;
    const bool row_valid = row < p.Sq;   // (row < Sq implies qt < qtiles)
    const int64_t unit = bh * p.qtiles + qt;
    const bool write_row = row_valid && unit >= p.unit_begin && unit < p.unit_end;
    const uint32_t scol = tmem + lane_base + C::kS;
    const uint32_t ocol = tmem + lane_base + (x ? C::kOB : C::kOA);
    {
      if constexpr (C::kQTmem) {
        // this row of Q into tensor memory (the A operand of QK^T); rows past Sq are zeros
        uint32_t qw[D / 4];
        const int8_t* qrow = p.q8 + (bh * p.Sq + (row_valid ? row : 0)) * D;
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          const uint4 u = row_valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + i) : make_uint4(0, 0, 0, 0);
          qw[4 * i] = u.x; qw[4 * i + 1] = u.y; qw[4 * i + 2] = u.z; qw[4 * i + 3] = u.w;
        }
        tmem_st16(tmem + lane_base + (x ? C::kQB : C::kQA), qw);
      }
      if constexpr (C::kPresetTmem) {
        if (x == 0) {   // the preset's A operand: FP16 2048 in K element 0 of every row
          const uint32_t pre[8] = {0x6800u, 0, 0, 0, 0, 0, 0, 0};
          tmem_st8(tmem + lane_base + C::kPresetA, pre);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->q_ready[x]);
    }
    // INT8: the Sage per-thread Q scale of the row; E4M3 blocks: one scale per 128-row Q tile
    const float qscale = !row_valid ? 0.f : QF8 ? p.qs[bh * p.nqs + qt] : p.qs[bh * p.nqs + (row >> 4) * 8 + (row & 7)];
    const float scale = p.sm_scale;
    const uint64_t bias2 = pk2f(kBias, kBias);
    const uint64_t tiny2 = pk2(kDenormOne, kDenormOne);
    const uint64_t expa2 = pk2f(kExpA, kExpA), expb2 = pk2f(kExpB, kExpB);
    // K scales of a tile: INT8 four groups (index tile*4 + (key%8)/2); E4M3 blocks one scale per kq_tiles tiles
    auto load_ks = [&](int jj) -> float4 {
      if constexpr (QF8) {
        const float v = __ldg(p.ks + bh * p.nks + jj / p.kq_tiles);
        return make_float4(v, v, v, v);
      } else {
        return __ldg(reinterpret_cast<const float4*>(p.ks + bh * p.nks + jj * 4));
      }
    };
    float4 ksv_next = load_ks(0);
    float m = -5000000.0f;   // running row maximum (the reference's initial value)
    float dprev = 0.f;       // block means: denominator just before PV_X(j-1)
    float pend[8];           // block means: pending masses of the open batch at O's scale
#pragma unroll
    for (int i = 0; i < 8; ++i) pend[i] = 0.f;
    uint8_t* massa = smem + L::kOffMassA + x * L::kMassA;
    bool ok = true;
    for (int j = 0; ok && j < T; ++j) {
      const float4 ksv = ksv_next;
      if (j + 1 < T) ksv_next = load_ks(j + 1);
      ok = mbar_wait_warp(&bar->s_full[x], j & 1, kErrTimeoutSoftmax);
      if (!ok) break;
      tc_fence_after();
      uint32_t raw[128];
      tmem_ld32(scol + 0, *reinterpret_cast<uint32_t(*)[32]>(raw + 0));
      tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(raw + 32));
      tmem_ld32(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(raw + 64));
      tmem_ld32(scol + 96, *reinterpret_cast<uint32_t(*)[32]>(raw + 96));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bar->s_free[x]);   // the next QK^T may now overwrite the slot
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
        float mx;
        if constexpr (D == 64) {
          // two independent chains over K rows 0-7 and 8-15 of the group (a
          // maximum is exact in any order): half the dependency depth, where
          // the group's own chain sets the period (config 4: 3.019 vs
          // 3.047 ms; at D = 128, bound by the score round trip, no gain)
          float ma = max3f(__uint_as_float(raw[2 * g]), __uint_as_float(raw[2 * g + 1]), __uint_as_float(raw[2 * g + 8]));
          float mb = max3f(__uint_as_float(raw[64 + 2 * g]), __uint_as_float(raw[64 + 2 * g + 1]),
                           __uint_as_float(raw[64 + 2 * g + 8]));
          ma = fmaxf(ma, __uint_as_float(raw[2 * g + 9]));
          mb = fmaxf(mb, __uint_as_float(raw[64 + 2 * g + 9]));
#pragma unroll
          for (int k = 2; k < 8; ++k) {
            ma = max3f(ma, __uint_as_float(raw[8 * k + 2 * g]), __uint_as_float(raw[8 * k + 2 * g + 1]));
            mb = max3f(mb, __uint_as_float(raw[64 + 8 * k + 2 * g]), __uint_as_float(raw[64 + 8 * k + 2 * g + 1]));
          }
          mx = fmaxf(ma, mb);
        } else {
          mx = max3f(__uint_as_float(raw[2 * g]), __uint_as_float(raw[2 * g + 1]), __uint_as_float(raw[2 * g + 8]));
          mx = fmaxf(mx, __uint_as_float(raw[2 * g + 9]));
#pragma unroll
          for (int k = 2; k < 16; ++k)
            mx = max3f(mx, __uint_as_float(raw[8 * k + 2 * g]), __uint_as_float(raw[8 * k + 2 * g + 1]));
        }
        if constexpr (QF8) {
          if (mx > -__int_as_float(0x7f800000)) lmax = fmaxf(lmax, __fmul_rn(mx, f1[g]));
        } else {
          if (mx > 0.f) lmax = fmaxf(lmax, __fmul_rn(__fsub_rn(mx, kBias), f1[g]));
        }
      }
      const float mn = fmaxf(m, lmax);
      const float alpha = expf(m - mn);
      m = mn;
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
      // PV_X(j-1) complete: P_X is free and O_X may be rescaled
      uint32_t draw = 0;   // block means: denominator column after PV_X(j-1)
      if (j >= 1) {
        ok = mbar_wait_warp(&bar->pv_done[x], (j - 1) & 1, kErrTimeoutSoftmax);
        if (!ok) break;
        if constexpr (BV) {
          tc_fence_after();
          draw = tmem_ld1(ocol + D);
        }
      }
      const bool grew = j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f);
      if (grew) {
        tc_fence_after();
        const uint64_t alpha2 = pk2f(alpha, alpha);
        // all of O's columns in flight at once: one tensor-memory load latency
        uint32_t o[D];
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) tmem_ld32(ocol + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(o + cc * 32));
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
      tc_fence_after();
      tmem_st32(tmem + lane_base + (x ? C::kPB : C::kPA), pw);
      tmem_wait_st();
      if constexpr (BV) tmem_wait_ld_reg(draw);   // the column read completes before PV_X(j) may start
      tc_fence_before();
      mbar_arrive(&bar->p_full[x]);
      if constexpr (BV) {
        // bookkeeping while PV_X(j) runs: mass_{j-1} at O's scale into slot
        // (j-1)%8, the pending masses times alpha_j, the operand when a batch completes
        const float dcur = __uint_as_float(draw);
        if (j >= 1) {
          const int slot = (j - 1) & 7;
          const float mass = __fmul_rn(__fsub_rn(dcur, dprev), alpha);
          if (grew) {
#pragma unroll
            for (int i = 0; i < 8; ++i) pend[i] = __fmul_rn(pend[i], alpha);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (i == slot) pend[i] = mass;
          if (slot == 7) {
            write_mass_row(massa, pend, t, 8);
            mbar_arrive(&bar->a_full[x]);
          }
        }
        dprev = j >= 1 ? __fmul_rn(dcur, alpha) : 0.f;   // the column just before PV_X(j)
      }
    }
    if constexpr (BV) {
      // the open batch: mass_{T-1} once PV_X(T-1) has completed
      if (ok) ok = mbar_wait_warp(&bar->pv_done[x], (T - 1) & 1, kErrTimeoutSoftmax);
      if (ok) {
        tc_fence_after();
        const float dlast = __uint_as_float(tmem_ld1(ocol + D));
        tmem_wait_ld();
        const int slot = (T - 1) & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i == slot) pend[i] = __fsub_rn(dlast, dprev);
        write_mass_row(massa, pend, t, slot + 1);
        tc_fence_before();
        mbar_arrive(&bar->a_full[x]);
      }
    }
    // epilogue: group X writes all D channels of its rows
    if (ok) ok = mbar_wait_warp(&bar->o_final[x], 0, kErrTimeoutSoftmax);
    if (ok) {
      tc_fence_after();
      uint32_t dn[16];
      tmem_ld16(ocol + D, dn);
      tmem_wait_ld();
      const float denom = __uint_as_float(dn[0]);
      OutT* orow = reinterpret_cast<OutT*>(p.out) + (bh / p.H) * p.osb + (bh % p.H) * p.osh + row * p.oss;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        tmem_ld32(ocol + cc * 32, o);
        tmem_wait_ld();
        if (write_row) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const int c0 = cc * 32 + c8 * 8;
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
