// INT8 Q/K preparation for sm_100a: K channel mean, centring, and the Sage
// per-thread INT8 quantisers.  HBM-bound passes with 16-byte vector loads.
//
// Arithmetic contract (bit exact with the reference given the same km):
//   quant_per_thread.py:39-45 / :89-97 --
//     scale = max|x| / 127 + 1e-7   (FP32, IEEE division)
//     q     = x / scale ; q += 0.5 * sign(q) ; int8(trunc(q))
//   K is first centred as RN_dtype(K - km) (quant_per_thread.py:158-159).
#include "common.cuh"
#include "kernels.h"

namespace vcb {

namespace {

constexpr int kSumRows = 512;     // rows per partial-sum chunk
constexpr int kSumThreads = 256;

template <typename T>
__device__ __forceinline__ const T* row_ptr(const T* base, int64_t bh, int64_t H, int64_t sb, int64_t sh, int64_t ss,
                                            int64_t s) {
  const int64_t b = bh / H, h = bh - b * H;
  return base + b * sb + h * sh + s * ss;
}

// Partial channel sums of K over chunks of kSumRows tokens: part[bh][chunk][d].
template <typename T, int D>
__global__ void __launch_bounds__(kSumThreads) k_partial_sums(const T* __restrict__ k, int64_t H, int64_t S,
                                                              int64_t sb, int64_t sh, int64_t ss,
                                                              float* __restrict__ part, int nchunks) {
  constexpr int EPT = 16 / sizeof(T);        // elements per 16-byte load
  constexpr int TPR = D / EPT;               // threads per row
  constexpr int RPI = kSumThreads / TPR;     // rows per iteration
  __shared__ float red[RPI][D];
  const int64_t bh = blockIdx.y;
  const int chunk = blockIdx.x;
  const int tr = threadIdx.x / TPR, tc = threadIdx.x % TPR;
  float acc[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) acc[i] = 0.f;
  const int64_t r0 = int64_t(chunk) * kSumRows;
  const int64_t r1 = min64(S, r0 + kSumRows);
  for (int64_t r = r0 + tr; r < r1; r += RPI) {
    float x[EPT];
    load_vec<T, EPT>(row_ptr(k, bh, H, sb, sh, ss, r) + tc * EPT, x);
#pragma unroll
    for (int i = 0; i < EPT; ++i) acc[i] += x[i];
  }
#pragma unroll
  for (int i = 0; i < EPT; ++i) red[tr][tc * EPT + i] = acc[i];
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += kSumThreads) {
    float s = 0.f;
#pragma unroll 8
    for (int j = 0; j < RPI; ++j) s += red[j][d];
    part[(bh * nchunks + chunk) * D + d] = s;
  }
}

// km[bh][d] = RN_dtype(sum_chunks(part) * factor), factor = float(n_out)/float(n_in)
// (torch's CUDA mean: accumulate in FP32, project by the float factor).
template <typename T, int D>
__global__ void k_mean_finalize(const float* __restrict__ part, int nchunks, float factor, T* __restrict__ km,
                                T* __restrict__ km_out) {
  const int64_t bh = blockIdx.x;
  const int d = threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int c = 0; c < nchunks; ++c) s += part[(bh * nchunks + c) * D + d];
  const float m = s * factor;
  T v;
  if constexpr (sizeof(T) == 4) v = m;
  else if constexpr (std::is_same<T, __half>::value) v = __float2half_rn(m);
  else v = __float2bfloat16_rn(m);
  km[bh * D + d] = v;
  if (km_out) km_out[bh * D + d] = v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One Sage INT8 value: q = RN(x/scale), q += 0.5*sign(q), truncate toward 0.
// Done without conversion-unit instructions (the quantiser is otherwise
// bound by them):
//  * RN(x/scale) by Markstein's correction step (Handbook of Floating-Point
//    Arithmetic, Muller et al., 2nd ed., sec. 4.7): with y = RN(1/scale)
//    (rscale, correctly rounded, computed once per scale group) and
//    q0 = RN(x*y) within one ulp of x/scale, the remainder
//    r = fma(-q0, scale, x) is exact and RN(q0 + r*y) = RN(x/scale).
//    Tiny quotients (|q| < 0.5) give 0 whatever their last bits.
//  * trunc(RN(q + 0.5*sign q)) = sign(q) * floor(RN(|q| + 0.5)) (RN is
//    symmetric): u = RN(|q| + 0.5) as the reference's addition rounds it, and
//    for 0 <= u < 2^23 the low byte of the bits of RD(u + 2^23) is floor(u)
//    (the ulp there is 1), so no conversion is needed.  |q| < 127.5 here, so
//    floor(u) <= 127; the sign is applied as (i ^ s) - s with s = 0 or -1.
__device__ __forceinline__ int8_t sage_i8(float x, float scale, float rscale) {
  const float q0 = __fmul_rn(x, rscale);
  const float r = __fmaf_rn(-q0, scale, x);
  const float q = __fmaf_rn(r, rscale, q0);
  const float u = __fadd_rn(fabsf(q), 0.5f);
  const int mag = static_cast<int>(__float_as_uint(__fadd_rd(u, 8388608.f)) & 0xFFu);
  const int s = static_cast<int>(__float_as_uint(q)) >> 31;
  return static_cast<int8_t>((mag ^ s) - s);
}

// sage_i8 for two values at once: the three operations of the quotient and
// the round-down add run as packed FP32 pairs, each half rounded exactly as
// the scalar instruction rounds it (fma(q0, -scale, x) is fma(-q0, scale, x):
// negating a factor is exact).  nscale2 = (-scale, -scale), rscale2 = (rscale, rscale).
__device__ __forceinline__ uint64_t f2_add_rd(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ void sage_i8x2(float xa, float xb, uint64_t nscale2, uint64_t rscale2, int8_t& oa,
                                          int8_t& ob) {
  const uint64_t x2 = pk2f(xa, xb);
  const uint64_t q0 = f2_mul(x2, rscale2);
  const uint64_t q2 = f2_fma(f2_fma(q0, nscale2, x2), rscale2, q0);
  uint32_t qa, qb;
  up2(q2, qa, qb);
  const float ua = __fadd_rn(fabsf(__uint_as_float(qa)), 0.5f), ub = __fadd_rn(fabsf(__uint_as_float(qb)), 0.5f);
  uint32_t ma, mb;
  up2(f2_add_rd(pk2f(ua, ub), pk2f(8388608.f, 8388608.f)), ma, mb);
  const int sa = static_cast<int>(qa) >> 31, sb = static_cast<int>(qb) >> 31;
  oa = static_cast<int8_t>((static_cast<int>(ma & 0xFFu) ^ sa) - sa);
  ob = static_cast<int8_t>((static_cast<int>(mb & 0xFFu) ^ sb) - sb);
}

// Two values rounded to T (RN) and held packed; unpack is exact.
template <typename T>
struct Pair;
template <>
struct Pair<float> {
  using type = float2;
  static __device__ __forceinline__ float2 pack(float a, float b) { return make_float2(a, b); }
  static __device__ __forceinline__ float2 unpack(float2 v) { return v; }
};
template <>
struct Pair<__half> {
  using type = __half2;
  static __device__ __forceinline__ __half2 pack(float a, float b) { return __floats2half2_rn(a, b); }
  static __device__ __forceinline__ float2 unpack(__half2 v) { return __half22float2(v); }
};
template <>
struct Pair<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static __device__ __forceinline__ __nv_bfloat162 pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
  static __device__ __forceinline__ float2 unpack(__nv_bfloat162 v) { return __bfloat1622float2(v); }
};

template <int N>
__device__ __forceinline__ void store_i8(int8_t* p, const int8_t (&v)[N]) {
  if constexpr (N == 8) {
    uint2 u;
    u.x = (uint32_t(uint8_t(v[0]))) | (uint32_t(uint8_t(v[1])) << 8) | (uint32_t(uint8_t(v[2])) << 16) |
          (uint32_t(uint8_t(v[3])) << 24);
    u.y = (uint32_t(uint8_t(v[4]))) | (uint32_t(uint8_t(v[5])) << 8) | (uint32_t(uint8_t(v[6])) << 16) |
          (uint32_t(uint8_t(v[7])) << 24);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    static_assert(N == 4, "4 or 8 values");
    *reinterpret_cast<uint32_t*>(p) = (uint32_t(uint8_t(v[0]))) | (uint32_t(uint8_t(v[1])) << 8) |
                                      (uint32_t(uint8_t(v[2])) << 16) | (uint32_t(uint8_t(v[3])) << 24);
  }
}

// ---------------------------------------------------------------------------
// Q and K quantisation tiles, one persistent kernel.
//
// A tile is 128 tokens of one (b,h): Q tiles first, then K tiles.  A producer
// warp streams each tile into a shared-memory ring: one untiled bulk copy per
// tile when its rows are contiguous, else (arbitrary row strides, the K
// permutation gather) 16-byte cp.async by all 32 lanes, whole rows per
// instruction, tracked by the stage's mbarrier.  One bulk copy per gathered
// row measured 2.6x slower than the contiguous tiles.  Three groups of eight
// compute warps take every third tile, quantise from shared memory and write
// int8 rows and scales with coalesced stores (three groups in 72 registers
// measured 7% faster than two in 89: more warps hide the shared-memory and
// shuffle latencies of the quantiser).
//   Q tile: warp w owns the 16-row Sage block w; scale group g = rows g, g+8.
//   K tile: scale group tld = rows 8i + 2 tld + {0,1}; warps w and w+4 split
//           the 16 i values of group tld = w & 3 and combine their maxima
//           through shared memory (one named barrier per tile).
// ---------------------------------------------------------------------------
constexpr int kTileWarps = 8;                              // per compute group
constexpr int kTileGroups = 3;
constexpr int kTileThreads = (kTileGroups * kTileWarps + 1) * 32;   // + producer warp

template <typename T, int D>
struct TileRing {
  static constexpr int kRow = D * int(sizeof(T));
  static constexpr int kStage = 128 * kRow;
  static constexpr int kStages = (196608 / kStage) < 4 ? (196608 / kStage) : 4;
  static constexpr int kOffBar = kStages * kStage;
  static constexpr int kOffRed = kOffBar + 2 * kStages * 8;
  static constexpr int kBytes = kOffRed + kTileGroups * 2 * kTileWarps * 4;
  static_assert(kStages >= 2, "two stages at least");
};

struct QKTileParams {
  const void* q;
  const void* k;
  int64_t H, Sq, Sk;
  int64_t qsb, qsh, qss, ksb, ksh, kss;
  const int64_t* perm;
  const void* km;
  int8_t* q8;
  float* qs;
  int8_t* k8;
  float* ks;
  int64_t qtiles, ktiles, nq, total;   // tiles per head (Q, K); Q tile count; all tiles
  int64_t nscale;                       // Q scales per head
};

template <typename T, int D>
__global__ void __launch_bounds__(kTileThreads, 1) qk_tiles(QKTileParams p) {
  using L = TileRing<T, D>;
  constexpr int E = D / 16;
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::kOffBar);
  uint64_t* empty = full + L::kStages;
  const int gwarp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = gwarp / kTileWarps, warp = gwarp % kTileWarps;
  float* red = reinterpret_cast<float*>(sm + L::kOffRed) + grp * 2 * kTileWarps;   // [K-tile parity][warp]
  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTileWarps * 32);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (gwarp == kTileGroups * kTileWarps) {
    // ------------------------------------------------------------ producer
    int n = 0;
    for (int64_t t = blockIdx.x; t < p.total; t += gridDim.x, ++n) {
      const int s = n % L::kStages;
      const bool isq = t < p.nq;
      const int64_t tt = isq ? t : t - p.nq;
      const int64_t tiles = isq ? p.qtiles : p.ktiles;
      const int64_t bh = tt / tiles, r0 = (tt - bh * tiles) * 128;
      const int64_t S = isq ? p.Sq : p.Sk;
      const int rows = static_cast<int>(min64(128, S - r0));
      const int64_t b = bh / p.H, h = bh - b * p.H;
      const T* base = static_cast<const T*>(isq ? p.q : p.k) + b * (isq ? p.qsb : p.ksb) + h * (isq ? p.qsh : p.ksh);
      const int64_t ss = isq ? p.qss : p.kss;
      const bool contiguous = ss == D && (isq || !p.perm);
      // source rows of this lane (rows lane + 32i), the permutation entries
      // loaded before the slot wait so that their latency overlaps it
      int64_t src[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = lane + 32 * i;
        src[i] = r0 + r;
        if (!contiguous && !isq && p.perm && r < rows) src[i] = __ldg(p.perm + bh * S + r0 + r);
      }
      if (n >= L::kStages && !mbar_wait(&empty[s], ((n / L::kStages) & 1) ^ 1, kErrTimeoutProducer)) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (lane + 32 * i < rows && (src[i] < 0 || src[i] >= S)) {
          raise_error(kErrBadIndex);   // out-of-range permutation entry: read row 0 instead
          src[i] = 0;
        }
      }
      uint8_t* dst = sm + s * L::kStage;
      if (contiguous) {   // contiguous rows: one copy for the tile
        if (lane == 0) {
          mbar_expect_tx(&full[s], static_cast<uint32_t>(rows * L::kRow));
          bulk_load(dst, base + r0 * ss, static_cast<uint32_t>(rows * L::kRow), &full[s]);
        }
        __syncwarp();
        continue;
      }
      // gathered or strided rows: chunk k of the tile is 16-byte piece k % CPR
      // of row k / CPR; a warp instruction covers RPI whole rows, all inside
      // one 32-row block, whose source rows lane r & 31 holds in src[r >> 5]
      constexpr int CPR = L::kRow / 16, RPI = 32 / CPR;
      static_assert(CPR <= 32 && 32 % CPR == 0, "a row is a divisor of 32 sixteen-byte pieces");
      const int c = lane % CPR;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll 4
        for (int it = 0; it < 32 / RPI; ++it) {
          const int r = 32 * i + it * RPI + lane / CPR;
          const int64_t sr = __shfl_sync(0xffffffffu, src[i], r & 31);
          if (r < rows) cp_async16(dst + r * L::kRow + c * 16, reinterpret_cast<const uint8_t*>(base + sr * ss) + c * 16, 16u);
        }
      }
      cp_async_mbar_arrive(&full[s]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);   // the phase's one counted arrival, after every lane's
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int col = (lane & 15) * E;
  const int hf = lane >> 4;
  int n = grp, nk = 0;
  for (int64_t t = blockIdx.x + int64_t(grp) * gridDim.x; t < p.total; t += kTileGroups * int64_t(gridDim.x), n += kTileGroups) {
    const int s = n % L::kStages;
    if (!mbar_wait_warp(&full[s], (n / L::kStages) & 1, kErrTimeoutProducer)) return;
    const T* tile = reinterpret_cast<const T*>(sm + s * L::kStage);
    const bool isq = t < p.nq;
    const int64_t tt = isq ? t : t - p.nq;
    const int64_t tiles = isq ? p.qtiles : p.ktiles;
    const int64_t bh = tt / tiles, r0 = (tt - bh * tiles) * 128;
    const int64_t S = isq ? p.Sq : p.Sk;
    const int rows = static_cast<int>(min64(128, S - r0));
    if (isq) {
      // Sage Q block: rows 16w .. 16w+15 of the tile, scale groups g = rows {g, g+8}.
      // The eight group maxima first; then lane g & 7 computes group g's scale,
      // so the warp runs one division and one reciprocal instead of eight
      float am[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int r = 16 * warp + g + 8 * hf;
        float x[E];
        if (r < rows) {
          load_vec_smem<T, E>(tile + r * D + col, x);
        } else {
#pragma unroll
          for (int i = 0; i < E; ++i) x[i] = 0.f;
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(x[i]));
        am[g] = warp_max(amax);
      }
      float mine = am[0];
#pragma unroll
      for (int g = 1; g < 8; ++g) mine = (lane & 7) == g ? am[g] : mine;
      const float my_scale = __fadd_rn(__fdiv_rn(mine, 127.f), 1e-7f);
      const float my_rscale = __frcp_rn(my_scale);
      // scales exist for the 16-row blocks of Sq padded to 64 rows (all-padding blocks get 1e-7)
      const int64_t blk16 = (r0 >> 4) + warp;
      if (lane < 8 && blk16 * 8 < p.nscale) p.qs[bh * p.nscale + blk16 * 8 + lane] = my_scale;
#pragma unroll 2
      for (int g = 0; g < 8; ++g) {
        const int r = 16 * warp + g + 8 * hf;
        const float scale = __shfl_sync(0xffffffffu, my_scale, g);
        const float rscale = __shfl_sync(0xffffffffu, my_rscale, g);
        const uint64_t nscale2 = pk2f(-scale, -scale), rscale2 = pk2f(rscale, rscale);
        float x[E];
        if (r < rows) {
          load_vec_smem<T, E>(tile + r * D + col, x);
        } else {
#pragma unroll
          for (int i = 0; i < E; ++i) x[i] = 0.f;
        }
        int8_t o[E];
#pragma unroll
        for (int i = 0; i < E; i += 2) sage_i8x2(x[i], x[i + 1], nscale2, rscale2, o[i], o[i + 1]);
        if (r < rows) store_i8<E>(p.q8 + (bh * S + r0 + r) * D + col, o);
      }
    } else {
      // K: centre as RN_T(k - km), then Sage per-thread groups of 32 rows
      const int tld = warp & 3, ih = warp >> 2;
      float kmv[E];
      {
        const T* kmp = static_cast<const T*>(p.km) + bh * D + col;
#pragma unroll
        for (int i = 0; i < E; ++i) kmv[i] = to_f32(kmp[i]);
      }
      // centred values RN_T(k - km), exactly representable in T: kept narrow,
      // and for 16-bit T rounded two at a time by the packed conversion
      using P = Pair<T>;
      typename P::type x[8][E / 2];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 8 * (8 * ih + i) + 2 * tld + hf;
        if (r < rows) {
          float raw[E];
          load_vec_smem<T, E>(tile + r * D + col, raw);
#pragma unroll
          for (int j = 0; j < E; j += 2) {
            x[i][j / 2] = P::pack(__fsub_rn(raw[j], kmv[j]), __fsub_rn(raw[j + 1], kmv[j + 1]));
            const float2 c = P::unpack(x[i][j / 2]);
            amax = fmaxf(amax, fmaxf(fabsf(c.x), fabsf(c.y)));
          }
        } else {
#pragma unroll
          for (int j = 0; j < E; j += 2) x[i][j / 2] = P::pack(0.f, 0.f);
        }
      }
      amax = warp_max(amax);
      // double-buffered by K-tile parity: every K tile has a barrier, so no warp
      // rewrites a slot another warp may still be reading
      float* rb = red + (nk & 1) * kTileWarps;
      ++nk;
      if (lane == 0) rb[warp] = amax;
      asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "n"(kTileWarps * 32) : "memory");
      amax = fmaxf(rb[tld], rb[tld + 4]);
      const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
      const float rscale = __frcp_rn(scale);
      const uint64_t nscale2 = pk2f(-scale, -scale), rscale2 = pk2f(rscale, rscale);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = 8 * (8 * ih + i) + 2 * tld + hf;
        int8_t o[E];
#pragma unroll
        for (int j = 0; j < E; j += 2) {
          const float2 c = P::unpack(x[i][j / 2]);
          sage_i8x2(c.x, c.y, nscale2, rscale2, o[j], o[j + 1]);
        }
        if (r < rows) store_i8<E>(p.k8 + (bh * S + r0 + r) * D + col, o);
      }
      if (lane == 0 && ih == 0) p.ks[bh * (p.ktiles * 4) + (r0 >> 7) * 4 + tld] = scale;
    }
    mbar_arrive(&empty[s]);
  }
}

template <typename T, int D>
int launch_prep_qk(const PrepQKArgs& a, cudaStream_t st) {
  const int64_t BH = a.B * a.H;
  const int nchunks = static_cast<int>((a.Sk + kSumRows - 1) / kSumRows);
  const T* km = static_cast<const T*>(a.km_in);
  if (!km) {
    float* part = static_cast<float*>(a.workspace);
    T* kmbuf = reinterpret_cast<T*>(part + BH * nchunks * D);
    k_partial_sums<T, D><<<dim3(nchunks, BH), kSumThreads, 0, st>>>(static_cast<const T*>(a.k), a.H, a.Sk, a.ksb,
                                                                    a.ksh, a.kss, part, nchunks);
    const float factor = (a.mean_numel_out > 0 && a.mean_numel_in > 0)
                             ? static_cast<float>(a.mean_numel_out) / static_cast<float>(a.mean_numel_in)
                             : 1.0f / static_cast<float>(a.Sk);
    k_mean_finalize<T, D><<<BH, D, 0, st>>>(part, nchunks, factor, kmbuf, static_cast<T*>(a.km_out));
    km = kmbuf;
  } else if (a.km_out) {
    cudaMemcpyAsync(a.km_out, a.km_in, BH * D * sizeof(T), cudaMemcpyDeviceToDevice, st);
  }
  QKTileParams tp;
  tp.q = a.q;
  tp.k = a.k;
  tp.H = a.H;
  tp.Sq = a.Sq;
  tp.Sk = a.Sk;
  tp.qsb = a.qsb; tp.qsh = a.qsh; tp.qss = a.qss;
  tp.ksb = a.ksb; tp.ksh = a.ksh; tp.kss = a.kss;
  tp.perm = a.perm;
  tp.km = km;
  tp.q8 = a.q8; tp.qs = a.qs; tp.k8 = a.k8; tp.ks = a.ks;
  tp.qtiles = (a.Sq + 127) / 128;
  tp.ktiles = (a.Sk + 127) / 128;
  tp.nq = BH * tp.qtiles;
  tp.total = tp.nq + BH * tp.ktiles;
  tp.nscale = (a.Sq + 63) / 64 * 32;
  auto kern = qk_tiles<T, D>;
  constexpr int smem = TileRing<T, D>::kBytes;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return VC_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = min64(tp.total, static_cast<int64_t>(sms));
  kern<<<static_cast<unsigned>(grid), kTileThreads, smem, st>>>(tp);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

}  // namespace

int64_t prep_qk_workspace(int64_t B, int64_t H, int64_t Sk, int64_t D) {
  const int64_t nchunks = (Sk + kSumRows - 1) / kSumRows;
  return B * H * nchunks * D * 4 + B * H * D * 4 + 256;
}

int prep_qk(const PrepQKArgs& a, cudaStream_t st) {
#define VCB_QK(DT, T)                                              \
  if (a.dtype == DT) {                                             \
    return a.D == 64 ? launch_prep_qk<T, 64>(a, st) : launch_prep_qk<T, 128>(a, st); \
  }
  VCB_QK(VC_DTYPE_BF16, __nv_bfloat16)
  VCB_QK(VC_DTYPE_F16, __half)
  VCB_QK(VC_DTYPE_F32, float)
#undef VCB_QK
  return VC_ERR_ARG;
}

cudaError_t prep_qk_error_word(uint32_t* code, bool clear) { return read_tu_error_word(code, clear); }

}  // namespace vcb
