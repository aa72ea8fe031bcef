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

// One Sage INT8 value: q = x/scale, q += 0.5*sign(q), truncate.
__device__ __forceinline__ int8_t sage_i8(float x, float scale) {
  float q = __fdiv_rn(x, scale);
  q = __fadd_rn(q, q >= 0.f ? 0.5f : -0.5f);
  return static_cast<int8_t>(__float2int_rz(q));
}

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

// Q: one warp per 16-row block; group g in 0..7 holds rows g and g+8.
// Lanes 0-15 read row g, lanes 16-31 row g+8, D/16 channels each.
template <typename T, int D>
__global__ void __launch_bounds__(256) quant_q(const T* __restrict__ q, int64_t H, int64_t S, int64_t sb, int64_t sh,
                                               int64_t ss, int8_t* __restrict__ q8, float* __restrict__ qs,
                                               int64_t nblk16) {
  constexpr int E = D / 16;
  const int lane = threadIdx.x & 31;
  const int64_t blk = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t bh = blockIdx.y;
  if (blk >= nblk16) return;
  const int col = (lane & 15) * E;
  const int half = lane >> 4;
  const int64_t nscale = nblk16 * 8;
#pragma unroll 2
  for (int g = 0; g < 8; ++g) {
    const int64_t row = blk * 16 + g + half * 8;
    float x[E];
    if (row < S) {
      load_vec<T, E>(row_ptr(q, bh, H, sb, sh, ss, row) + col, x);
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) x[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = warp_max(amax);
    const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
    int8_t o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = sage_i8(x[i], scale);
    if (row < S) store_i8<E>(q8 + (bh * S + row) * D + col, o);
    if (lane == 0) qs[bh * nscale + blk * 8 + g] = scale;
  }
}

// K: one warp per (128-row block, tld); its 32 rows are blk*128 + 8i + 2tld + {0,1}.
template <typename T, int D>
__global__ void __launch_bounds__(128) quant_k(const T* __restrict__ k, int64_t H, int64_t S, int64_t sb, int64_t sh,
                                               int64_t ss, const int64_t* __restrict__ perm,
                                               const T* __restrict__ km, int8_t* __restrict__ k8,
                                               float* __restrict__ ks, int64_t nblk) {
  constexpr int E = D / 16;
  const int lane = threadIdx.x & 31;
  const int tld = threadIdx.x >> 5;  // 4 warps
  const int64_t blk = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int col = (lane & 15) * E;
  const int half = lane >> 4;
  float kmv[E];
#pragma unroll
  for (int i = 0; i < E; ++i) kmv[i] = to_f32(km[bh * D + col + i]);
  float x[16][E];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t row = blk * 128 + 8 * i + 2 * tld + half;
    if (row < S) {
      const int64_t src = perm ? perm[bh * S + row] : row;
      float raw[E];
      if (src >= 0 && src < S) {
        load_vec<T, E>(row_ptr(k, bh, H, sb, sh, ss, src) + col, raw);
      } else {
        raise_error(kErrBadIndex);   // out-of-range permutation entry: the row reads as zeros
#pragma unroll
        for (int j = 0; j < E; ++j) raw[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < E; ++j) {
        x[i][j] = round_as(__fsub_rn(raw[j], kmv[j]), static_cast<T*>(nullptr));
        amax = fmaxf(amax, fabsf(x[i][j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) x[i][j] = 0.f;
    }
  }
  amax = warp_max(amax);
  const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t row = blk * 128 + 8 * i + 2 * tld + half;
    int8_t o[E];
#pragma unroll
    for (int j = 0; j < E; ++j) o[j] = sage_i8(x[i][j], scale);
    if (row < S) store_i8<E>(k8 + (bh * S + row) * D + col, o);
  }
  if (lane == 0) ks[bh * (nblk * 4) + blk * 4 + tld] = scale;
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
  const int64_t nblk16 = (a.Sq + 63) / 64 * 4;
  quant_q<T, D><<<dim3((nblk16 + 7) / 8, BH), 256, 0, st>>>(static_cast<const T*>(a.q), a.H, a.Sq, a.qsb, a.qsh,
                                                            a.qss, a.q8, a.qs, nblk16);
  const int64_t nblk = (a.Sk + 127) / 128;
  quant_k<T, D><<<dim3(nblk, BH), 128, 0, st>>>(static_cast<const T*>(a.k), a.H, a.Sk, a.ksb, a.ksh, a.kss, a.perm,
                                                km, a.k8, a.ks, nblk);
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
