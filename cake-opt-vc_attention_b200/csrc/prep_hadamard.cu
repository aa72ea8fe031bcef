// Q/K preparation of the Config contract's own QK path (qk_hadamard=True),
// src/vc_attention/core.py:79-107 (hadamard, preprocess_qk) and :128-150
// (_divide_fp32, _encode, _quantize_qk):
//   * K centred by its FP32 channel mean over all tokens (k_smooth);
//   * Q and K rotated by the normalised Sylvester transform on channels:
//     butterfly stages step = 1, 2, 4, ... (pair (i, i+step) -> (a+b, a-b)),
//     then a multiply by FP32(D^-1/2);
//   * E4M3 block quantisation: one scale amax/448 (FP32 division, 1 when the
//     block is all zeros) per block of q_block = 128 rows (Q) or k_quant_block
//     rows (K) by all D <= 128 channels; payload e4m3_rn_satfinite(x / scale).
// One warp rotates one row (D/32 consecutive channels per lane; stages with a
// step below D/32 stay in the lane, the others pair lanes by xor shuffles);
// every output is the same sequence of FP32 adds as the reference's.  Pass 0
// takes each block's amax (order-free atomicMax on the FP32 bits of |x|),
// pass 1 recomputes the rows and writes the payloads and the scales.
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kHadWarps = 8;     // 256 threads per 128-row tile
constexpr int kHadChunk = 512;   // rows per K-sum chunk

template <int D>
__device__ __forceinline__ float had_norm() {
  if constexpr (D == 128) return __uint_as_float(0x3DB504F3u);   // FP32(128^-1/2)
  else return 0.125f;                                             // 64^-1/2, exact
}

struct HadParams {
  const void* q;
  const void* k;
  int64_t H, Sq, Sk;
  int64_t qsb, qsh, qss, ksb, ksh, kss;
  const int64_t* perm;
  const float* km;        // [BH][D] or null (no centring)
  uint8_t* q8;
  float* qs;
  uint8_t* k8;
  float* ks;
  uint32_t* amax;         // [BH][nqb] then [BH][nkb]: FP32 bits of the blocks' max |x|
  int64_t qtiles, ktiles, nqb, nkb, kqb;
};

// Per-chunk FP32 channel sums of K in row order; thread d owns channel d.
template <typename T, int D>
__global__ void __launch_bounds__(D) had_k_sums(const T* __restrict__ k, int64_t H, int64_t S, int64_t sb, int64_t sh,
                                                int64_t ss, float* __restrict__ part, int64_t nchunk) {
  const int64_t bh = blockIdx.y, c = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const T* base = k + b * sb + h * sh + threadIdx.x;
  float s = 0.f;
  const int64_t r1 = min64(S, (c + 1) * kHadChunk);
  for (int64_t r = c * kHadChunk; r < r1; ++r) s = __fadd_rn(s, to_f32(base[r * ss]));
  part[(bh * nchunk + c) * D + threadIdx.x] = s;
}

// km = (chunk sums in chunk order) / S.
template <int D>
__global__ void __launch_bounds__(D) had_k_mean(const float* __restrict__ part, int64_t nchunk, int64_t S,
                                                float* __restrict__ km) {
  const int64_t bh = blockIdx.x;
  float s = 0.f;
  for (int64_t c = 0; c < nchunk; ++c) s = __fadd_rn(s, part[(bh * nchunk + c) * D + threadIdx.x]);
  km[bh * D + threadIdx.x] = __fdiv_rn(s, static_cast<float>(S));
}

__global__ void had_clear(uint32_t* __restrict__ w, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) w[i] = 0u;
}

// D/32 consecutive elements of a row, as floats.
template <typename T, int E>
__device__ __forceinline__ void load_row_part(const T* p, float (&x)[E]) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (E == 4) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(p));
      x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
    } else {
      const float2 u = __ldg(reinterpret_cast<const float2*>(p));
      x[0] = u.x; x[1] = u.y;
    }
  } else {
    uint32_t w[E / 2];
    if constexpr (E == 4) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = u.x; w[1] = u.y;
    } else {
      w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
    }
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      T lo, hi;
      const uint16_t a = static_cast<uint16_t>(w[i] & 0xffffu), b = static_cast<uint16_t>(w[i] >> 16);
      memcpy(&lo, &a, 2);
      memcpy(&hi, &b, 2);
      x[2 * i] = to_f32(lo);
      x[2 * i + 1] = to_f32(hi);
    }
  }
}

// Centre (optional) and rotate one row held by a warp: lane l owns channels
// [l*E, (l+1)*E).
template <int D>
__device__ __forceinline__ void had_rotate(float (&x)[D / 32], const float* km, int lane) {
  constexpr int E = D / 32;
  if (km) {
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = __fsub_rn(x[i], km[lane * E + i]);
  }
#pragma unroll
  for (int step = 1; step < E; step <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i)
      if (!(i & step)) {
        const float a = x[i], b = x[i + step];
        x[i] = __fadd_rn(a, b);
        x[i + step] = __fsub_rn(a, b);
      }
  }
#pragma unroll
  for (int step = E; step < D; step <<= 1) {
    const int m = step / E;
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, x[i], m);
      x[i] = upper ? __fsub_rn(o, x[i]) : __fadd_rn(x[i], o);
    }
  }
#pragma unroll
  for (int i = 0; i < E; ++i) x[i] = __fmul_rn(x[i], had_norm<D>());
}

// One 128-row tile of Q (tiles [0, BH*qtiles)) or K (the rest).  PASS 0: block
// amax; PASS 1: payload rows and block scales.
template <typename T, int D, int PASS>
__global__ void __launch_bounds__(kHadWarps * 32) had_tiles(HadParams p) {
  constexpr int E = D / 32;
  __shared__ float km_s[D];
  __shared__ float red[kHadWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t t = blockIdx.x;
  const bool isq = t < p.qtiles;
  if (!isq) t -= p.qtiles;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.H, h = bh - b * p.H;
  const int64_t S = isq ? p.Sq : p.Sk;
  const int64_t r0 = t * 128;
  const int rows = static_cast<int>(min64(128, S - r0));
  const bool centre = !isq && p.km;
  if (centre)
    for (int d = threadIdx.x; d < D; d += blockDim.x) km_s[d] = p.km[bh * D + d];
  __syncthreads();
  const T* base = static_cast<const T*>(isq ? p.q : p.k) + b * (isq ? p.qsb : p.ksb) + h * (isq ? p.qsh : p.ksh);
  const int64_t ss = isq ? p.qss : p.kss;
  // block of this tile and its words
  const int64_t nb = isq ? p.nqb : p.nkb;
  const int64_t block = isq ? t : (r0 / p.kqb);
  uint32_t* amax = p.amax + (isq ? 0 : int64_t(gridDim.y) * p.nqb) + bh * nb + block;
  float scale = 1.f;
  if constexpr (PASS == 1) {
    scale = __fdiv_rn(__uint_as_float(*amax), 448.f);
    if (scale == 0.f) scale = 1.f;
  }
  // x / scale correctly rounded by Markstein's correction step (Handbook of
  // Floating-Point Arithmetic, Muller et al., 2nd ed., sec. 4.7): with
  // y = RN(1/scale), q0 = RN(x*y) and the exact remainder r = fma(-q0, scale, x),
  // RN(q0 + r*y) = RN(x/scale) for normal quotients; a subnormal quotient
  // encodes to a signed E4M3 zero either way.
  const float rscale = __frcp_rn(scale);
  auto div_scale = [&](float x) {
    const float q0 = __fmul_rn(x, rscale);
    return __fmaf_rn(__fmaf_rn(-q0, scale, x), rscale, q0);
  };
  float mx = 0.f;
  for (int r = warp; r < rows; r += kHadWarps) {
    int64_t src = r0 + r;
    if (!isq && p.perm) {
      src = p.perm[bh * S + src];
      if (src < 0 || src >= S) {
        if (lane == 0 && PASS == 0) raise_error(kErrBadIndex);   // out-of-range entry: row 0 instead
        src = 0;
      }
    }
    float x[E];
    load_row_part<T, E>(base + src * ss + lane * E, x);
    had_rotate<D>(x, centre ? km_s : nullptr, lane);
    if constexpr (PASS == 0) {
#pragma unroll
      for (int i = 0; i < E; ++i) mx = fmaxf(mx, fabsf(x[i]));
    } else {
      uint32_t packed[E / 2];
#pragma unroll
      for (int i = 0; i < E / 2; ++i)
        packed[i] = e4m3x2(div_scale(x[2 * i]), div_scale(x[2 * i + 1]));
      uint8_t* dst = (isq ? p.q8 : p.k8) + ((bh * S) + r0 + r) * D + lane * E;
      if constexpr (E == 4) *reinterpret_cast<uint32_t*>(dst) = packed[0] | (packed[1] << 16);
      else *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(packed[0]);
    }
  }
  if constexpr (PASS == 0) {
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      float m = red[0];
      for (int w = 1; w < kHadWarps; ++w) m = fmaxf(m, red[w]);
      atomicMax(amax, __float_as_uint(m));   // |x| >= 0: bit order is value order
    }
  } else {
    // the block's first tile writes its scale
    const bool first = isq || (r0 % p.kqb) == 0;
    if (first && threadIdx.x == 0) (isq ? p.qs : p.ks)[bh * nb + block] = scale;
  }
}

template <typename T, int D>
int launch_had(const PrepHadArgs& a, cudaStream_t st) {
  const int64_t BH = a.B * a.H;
  const int64_t qtiles = (a.Sq + 127) / 128, ktiles = (a.Sk + 127) / 128;
  const int64_t nqb = qtiles, nkb = (a.Sk + a.kqb - 1) / a.kqb;
  const int64_t nchunk = (a.Sk + kHadChunk - 1) / kHadChunk;
  uint8_t* w = static_cast<uint8_t*>(a.workspace);
  auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
  float* part = reinterpret_cast<float*>(w);
  w += up(BH * nchunk * D * 4);
  float* km = reinterpret_cast<float*>(w);
  w += up(BH * D * 4);
  uint32_t* amax = reinterpret_cast<uint32_t*>(w);
  const float* km_use = nullptr;
  if (a.k_smooth) {
    if (a.km_in) {
      km_use = a.km_in;
    } else {
      had_k_sums<T, D><<<dim3(nchunk, BH), D, 0, st>>>(static_cast<const T*>(a.k), a.H, a.Sk, a.ksb, a.ksh, a.kss,
                                                        part, nchunk);
      had_k_mean<D><<<BH, D, 0, st>>>(part, nchunk, a.Sk, km);
      km_use = km;
    }
    if (a.km_out) cudaMemcpyAsync(a.km_out, km_use, BH * D * 4, cudaMemcpyDeviceToDevice, st);
  }
  had_clear<<<64, 256, 0, st>>>(amax, BH * (nqb + nkb));
  HadParams p{a.q, a.k, a.H, a.Sq, a.Sk, a.qsb, a.qsh, a.qss, a.ksb, a.ksh, a.kss, a.perm, km_use,
              a.q8, a.qs, a.k8, a.ks, amax, qtiles, ktiles, nqb, nkb, a.kqb};
  const dim3 grid(static_cast<unsigned>(qtiles + ktiles), static_cast<unsigned>(BH));
  had_tiles<T, D, 0><<<grid, kHadWarps * 32, 0, st>>>(p);
  had_tiles<T, D, 1><<<grid, kHadWarps * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

}  // namespace

int64_t prep_hadamard_workspace(int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int64_t kqb) {
  const int64_t BH = B * H, nchunk = (Sk + kHadChunk - 1) / kHadChunk;
  const int64_t nqb = (Sq + 127) / 128, nkb = (Sk + kqb - 1) / kqb;
  auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
  return up(BH * nchunk * D * 4) + up(BH * D * 4) + up(BH * (nqb + nkb) * 4);
}

int prep_hadamard(const PrepHadArgs& a, cudaStream_t st) {
  if (a.dtype == VC_DTYPE_BF16) return a.D == 64 ? launch_had<__nv_bfloat16, 64>(a, st) : launch_had<__nv_bfloat16, 128>(a, st);
  if (a.dtype == VC_DTYPE_F16) return a.D == 64 ? launch_had<__half, 64>(a, st) : launch_had<__half, 128>(a, st);
  if (a.dtype == VC_DTYPE_F32) return a.D == 64 ? launch_had<float, 64>(a, st) : launch_had<float, 128>(a, st);
  return VC_ERR_ARG;
}

cudaError_t prep_hadamard_error_word(uint32_t* code, bool clear) { return read_tu_error_word(code, clear); }

}  // namespace vcb
