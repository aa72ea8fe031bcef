// V preparation for sm_100a: per-channel E4M3 (unsmoothed) and 128-token
// block de-meaning with an E4M3 residual (V smoothing).  Output payload is V
// transposed to [B, H, D, Npad] (Npad = 128 * ceil(S/128)) in token order:
// the K-major B operand of the P.V tcgen05 MMA.
//
// Each CTA stages one 128-token tile (optionally gathered through ``perm``)
// in shared memory with coalesced 16-byte loads, converts token pairs with
// cvt.rn.satfinite.e4m3x2, transposes through shared memory and writes
// 128-byte channel rows.
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kTileThreads = 256;

template <typename T, int D>
struct TileGeom {
  static constexpr int kRowBytes = D * int(sizeof(T));
  static constexpr int kPitch = kRowBytes + 16;          // padded row pitch (bytes)
  static constexpr int kInBytes = 128 * kPitch;
  static constexpr int kOutBytes = D * 128;              // [D][128] E4M3
  static constexpr int kSmem = kInBytes + kOutBytes + 4 * D * 4;
};

// Stage rows [tile*128, tile*128+128) of head bh into smem (zeros past S and
// for out-of-range permutation entries, which also raise kErrBadIndex).  Each
// thread first loads the source indices of all its chunks, then issues every
// chunk as a cp.async, so no load waits on another; the caller synchronises.
template <typename T, int D>
__device__ __forceinline__ void stage_tile(uint8_t* sin, const T* __restrict__ v, int64_t bh, int64_t H, int64_t S,
                                           int64_t sb, int64_t sh, int64_t ss, const int64_t* __restrict__ perm,
                                           int64_t tile) {
  using G = TileGeom<T, D>;
  constexpr int CPR = G::kRowBytes / 16;  // 16-byte chunks per row
  constexpr int EL = 16 / int(sizeof(T));
  constexpr int IT = (128 * CPR + kTileThreads - 1) / kTileThreads;
  const int64_t b = bh / H, h = bh - b * H;
  const T* base = v + b * sb + h * sh;
  int64_t src[IT];
#pragma unroll
  for (int k = 0; k < IT; ++k) {
    const int i = threadIdx.x + k * kTileThreads;
    const int64_t row = tile * 128 + i / CPR;
    src[k] = -1;
    if (i < 128 * CPR && row < S) src[k] = perm ? __ldg(perm + bh * S + row) : row;
  }
#pragma unroll
  for (int k = 0; k < IT; ++k) {
    const int i = threadIdx.x + k * kTileThreads;
    if (i >= 128 * CPR) break;
    const int r = i / CPR, c = i - r * CPR;
    const bool in = tile * 128 + r < S;
    const bool ok = src[k] >= 0 && src[k] < S;
    if (in && !ok) raise_error(kErrBadIndex);
    cp_async16(sin + r * G::kPitch + c * 16, base + (ok ? src[k] : 0) * ss + c * EL, ok ? 16u : 0u);
  }
  cp_async_wait_all();
}

template <typename T>
__device__ __forceinline__ float smem_elem(const uint8_t* sin, int pitch, int r, int d) {
  return to_f32(*reinterpret_cast<const T*>(sin + r * pitch + d * int(sizeof(T))));
}

// Write the [D][128] E4M3 tile to v8[bh][d][tile*128 ...] with 16-byte stores.
template <int D>
__device__ __forceinline__ void store_out_tile(const uint8_t* sout, uint8_t* __restrict__ v8, int64_t bh,
                                               int64_t npad, int64_t tile) {
  for (int i = threadIdx.x; i < D * 8; i += blockDim.x) {
    const int d = i >> 3, c = i & 7;
    const uint4 val = *reinterpret_cast<const uint4*>(sout + d * 128 + c * 16);
    *reinterpret_cast<uint4*>(v8 + (bh * D + d) * npad + tile * 128 + c * 16) = val;
  }
}

// Per-channel |V| maximum over all tokens, combined across CTAs with an
// order-independent atomicMax on the FP32 bit pattern (values are >= 0).
template <typename T, int D>
__global__ void __launch_bounds__(256) v_channel_amax(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb,
                                                      int64_t sh, int64_t ss, uint32_t* __restrict__ amax_bits) {
  constexpr int EPT = 16 / sizeof(T);
  constexpr int TPR = D / EPT;
  constexpr int RPI = 256 / TPR;
  __shared__ float red[RPI][D];
  const int64_t bh = blockIdx.y;
  const int tr = threadIdx.x / TPR, tc = threadIdx.x % TPR;
  const int64_t b = bh / H, h = bh - b * H;
  float m[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) m[i] = 0.f;
  const int64_t r0 = int64_t(blockIdx.x) * 512, r1 = min64(S, r0 + 512);
  for (int64_t r = r0 + tr; r < r1; r += RPI) {
    float x[EPT];
    load_vec<T, EPT>(v + b * sb + h * sh + r * ss + tc * EPT, x);
#pragma unroll
    for (int i = 0; i < EPT; ++i) m[i] = fmaxf(m[i], fabsf(x[i]));
  }
#pragma unroll
  for (int i = 0; i < EPT; ++i) red[tr][tc * EPT + i] = m[i];
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += 256) {
    float a = 0.f;
    for (int j = 0; j < RPI; ++j) a = fmaxf(a, red[j][d]);
    atomicMax(amax_bits + bh * D + d, __float_as_uint(a));
  }
}

enum QuantMode { kPlainChannel = 0, kResidualChannel = 1, kResidualBlock = 2 };

// Tree sum of 128 rows of one channel in the reference's warp order
// (csrc/vc/preprocess.cu:72-77 with sum_warp :17-20): lane l accumulates
// rows l, l+32, l+64, l+96 from 0, then xor-butterflies 16..1.
template <typename T, int D>
__device__ __forceinline__ float block_sum(const uint8_t* sin, int d) {
  using G = TileGeom<T, D>;
  float s[32];
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) t = __fadd_rn(t, smem_elem<T>(sin, G::kPitch, l + 32 * j, d));
    s[l] = t;
  }
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
#pragma unroll
    for (int l = 0; l < w; ++l) s[l] = __fadd_rn(s[l], s[l + w]);
  }
  return s[0];
}

// max over the tile's first ``count`` rows of |x - mean| in channel d, as four
// independent chains (a maximum is exact in any order).
template <typename T, int D>
__device__ __forceinline__ float residual_peak(const uint8_t* sin, int d, int count, float mean) {
  using G = TileGeom<T, D>;
  float pk[4] = {0.f, 0.f, 0.f, 0.f};
  int r = 0;
  for (; r + 4 <= count; r += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) pk[u] = fmaxf(pk[u], fabsf(__fsub_rn(smem_elem<T>(sin, G::kPitch, r + u, d), mean)));
  }
  for (; r < count; ++r) pk[0] = fmaxf(pk[0], fabsf(__fsub_rn(smem_elem<T>(sin, G::kPitch, r, d), mean)));
  return fmaxf(fmaxf(pk[0], pk[1]), fmaxf(pk[2], pk[3]));
}

// Block statistics pass (channel-scale mode): the mean per (bh, tile, d) into
// the workspace, and the maxima over tiles of the residual peak and of |mean|
// per (bh, d) (csrc/vc/preprocess.cu:68-88).  The maxima are combined across
// CTAs by atomicMax on the FP32 bits (values >= 0, so the bit order is the
// value order; a maximum does not depend on the order of its operands); NaN
// operands are skipped, as fmaxf skips them.
template <typename T, int D>
__global__ void __launch_bounds__(kTileThreads) v_block_stats(const T* __restrict__ v, int64_t H, int64_t S,
                                                              int64_t sb, int64_t sh, int64_t ss,
                                                              const int64_t* __restrict__ perm,
                                                              float* __restrict__ ws_mean, uint32_t* __restrict__ peak_bits,
                                                              uint32_t* __restrict__ mabs_bits, int64_t tiles) {
  using G = TileGeom<T, D>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int64_t tile = blockIdx.x, bh = blockIdx.y;
  stage_tile<T, D>(smem, v, bh, H, S, sb, sh, ss, perm, tile);
  __syncthreads();
  const int count = static_cast<int>(min64(128, S - tile * 128));
  for (int d = threadIdx.x; d < D; d += kTileThreads) {
    const float mean = __fdiv_rn(block_sum<T, D>(smem, d), static_cast<float>(count));
    const float peak = residual_peak<T, D>(smem, d, count, mean);
    ws_mean[(bh * tiles + tile) * D + d] = mean;
    const float mabs = fabsf(mean);
    if (peak == peak) atomicMax(peak_bits + bh * D + d, __float_as_uint(peak));
    if (mabs == mabs) atomicMax(mabs_bits + bh * D + d, __float_as_uint(mabs));
  }
}

// Channel scale s = max(max_t peak/448 (1 if 0), max_t |mean|/65504)
// (csrc/vc/preprocess.cu:90-106), from the two maxima over tiles that
// v_block_stats accumulated.
template <int D>
__global__ void v_channel_scales(const uint32_t* __restrict__ peak_bits, const uint32_t* __restrict__ mabs_bits,
                                 float* __restrict__ vs) {
  const int64_t bh = blockIdx.x;
  const int d = threadIdx.x;
  if (d >= D) return;
  const float pk = __uint_as_float(peak_bits[bh * D + d]), mp = __uint_as_float(mabs_bits[bh * D + d]);
  const float s = pk > 0.f ? __fdiv_rn(pk, 448.f) : 1.0f;
  vs[bh * D + d] = fmaxf(s, __fdiv_rn(mp, 65504.f));
}

// Quantise one staged tile into E4M3 and store it transposed.
//   kPlainChannel    : e4m3(x * recp[d])            (fused.cu:399-423)
//   kResidualChannel : e4m3((x - mean[d]) / s[d])   (preprocess.cu:108-123)
//   kResidualBlock   : statistics computed here, per-tile scale
//                      (preprocess.cu:25-56)
template <typename T, int D, int MODE>
__global__ void __launch_bounds__(kTileThreads) v_tile_quant(const T* __restrict__ v, int64_t H, int64_t S,
                                                             int64_t sb, int64_t sh, int64_t ss,
                                                             const int64_t* __restrict__ perm,
                                                             const uint32_t* __restrict__ amax_bits,
                                                             const float* __restrict__ ws_mean,
                                                             float* __restrict__ vs, __half* __restrict__ means,
                                                             uint8_t* __restrict__ v8, int64_t tiles, int demean) {
  using G = TileGeom<T, D>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sin = smem;
  uint8_t* sout = smem + G::kInBytes;
  float* s_mul = reinterpret_cast<float*>(smem + G::kInBytes + G::kOutBytes);  // recp or scale
  float* s_mean = s_mul + D;
  float* s_rcp = s_mean + D;   // RN(1/s) for the residual modes' quotients
  const int64_t tile = blockIdx.x, bh = blockIdx.y;
  const int count = static_cast<int>(min64(128, S - tile * 128));
  stage_tile<T, D>(sin, v, bh, H, S, sb, sh, ss, perm, tile);
  if constexpr (MODE == kPlainChannel) {
    for (int d = threadIdx.x; d < D; d += kTileThreads) {
      const float amax = __uint_as_float(amax_bits[bh * D + d]);
      s_mul[d] = amax == 0.f ? 0.f : __fdiv_rn(448.f, amax);
      if (tile == 0) vs[bh * D + d] = __fdiv_rn(amax, 448.f);
    }
  } else if constexpr (MODE == kResidualChannel) {
    for (int d = threadIdx.x; d < D; d += kTileThreads) {
      const float mean = ws_mean[(bh * tiles + tile) * D + d];
      const float s = vs[bh * D + d];
      s_mul[d] = s;
      s_mean[d] = mean;
      s_rcp[d] = __frcp_rn(s);
      means[(bh * tiles + tile) * D + d] = __float2half_rn(__fdiv_rn(mean, s));
    }
  }
  __syncthreads();
  if constexpr (MODE == kResidualBlock) {
    for (int d = threadIdx.x; d < D; d += kTileThreads) {
      const float mean = demean ? __fdiv_rn(block_sum<T, D>(sin, d), static_cast<float>(count)) : 0.f;
      const float peak = residual_peak<T, D>(sin, d, count, mean);
      float s = peak > 0.f ? __fdiv_rn(peak, 448.f) : 1.0f;
      s = fmaxf(s, __fdiv_rn(fabsf(mean), 65504.f));
      s_mul[d] = s;
      s_mean[d] = mean;
      s_rcp[d] = __frcp_rn(s);
      vs[(bh * tiles + tile) * D + d] = s;
      means[(bh * tiles + tile) * D + d] = __float2half_rn(__fdiv_rn(mean, s));
    }
    __syncthreads();
  }
  // token pair t2 (rows 2t2, 2t2+1) x channel group of 8: each row's 8
  // channels are contiguous in the staged tile, read as one vector
  constexpr int NG = D / 8;
  for (int i = threadIdx.x; i < 64 * NG; i += kTileThreads) {
    const int t2 = i % 64, g = i / 64;
    const int r0 = 2 * t2;
    float xa[8], xb[8];
    load_vec_smem<T, 8>(reinterpret_cast<const T*>(sin + r0 * G::kPitch + g * 8 * int(sizeof(T))), xa);
    load_vec_smem<T, 8>(reinterpret_cast<const T*>(sin + (r0 + 1) * G::kPitch + g * 8 * int(sizeof(T))), xb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = g * 8 + j;
      float x0 = xa[j];
      float x1 = xb[j];
      if constexpr (MODE == kPlainChannel) {
        x0 = __fmul_rn(x0, s_mul[d]);
        x1 = __fmul_rn(x1, s_mul[d]);
      } else {
        // (x - mean) / s correctly rounded by Markstein's correction step
        // (Handbook of Floating-Point Arithmetic, sec. 4.7); a subnormal
        // quotient encodes to a signed E4M3 zero either way
        const float sd = s_mul[d], rd = s_rcp[d];
        const float n0 = __fsub_rn(x0, s_mean[d]), n1 = __fsub_rn(x1, s_mean[d]);
        const float a0 = __fmul_rn(n0, rd), a1 = __fmul_rn(n1, rd);
        x0 = r0 < count ? __fmaf_rn(__fmaf_rn(-a0, sd, n0), rd, a0) : 0.f;
        x1 = r0 + 1 < count ? __fmaf_rn(__fmaf_rn(-a1, sd, n1), rd, a1) : 0.f;
      }
      *reinterpret_cast<uint16_t*>(sout + d * 128 + r0) = e4m3x2(x0, x1);
    }
  }
  __syncthreads();
  store_out_tile<D>(sout, v8, bh, tiles * 128, tile);
}

template <typename T, int D>
int launch_v_channel(const PrepVArgs& a, cudaStream_t st) {
  using G = TileGeom<T, D>;
  const int64_t BH = a.B * a.H, tiles = (a.S + 127) / 128;
  uint32_t* amax = static_cast<uint32_t*>(a.workspace);
  if (cudaMemsetAsync(amax, 0, BH * D * 4, st) != cudaSuccess) return VC_ERR_LAUNCH;
  v_channel_amax<T, D><<<dim3((a.S + 511) / 512, BH), 256, 0, st>>>(static_cast<const T*>(a.v), a.H, a.S, a.sb, a.sh,
                                                                    a.ss, amax);
  auto k = v_tile_quant<T, D, kPlainChannel>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
  k<<<dim3(tiles, BH), kTileThreads, G::kSmem, st>>>(static_cast<const T*>(a.v), a.H, a.S, a.sb, a.sh, a.ss, a.perm,
                                                     amax, nullptr, a.vs, nullptr, a.v8, tiles, 0);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

template <typename T, int D>
int launch_v_blocks(const PrepVArgs& a, cudaStream_t st) {
  using G = TileGeom<T, D>;
  const int64_t BH = a.B * a.H, tiles = (a.S + 127) / 128;
  __half* means = reinterpret_cast<__half*>(a.means);
  if (a.channel_scale && a.demean) {
    float* ws_mean = static_cast<float*>(a.workspace);
    uint32_t* peak_bits = reinterpret_cast<uint32_t*>(ws_mean + BH * tiles * D);
    uint32_t* mabs_bits = peak_bits + BH * D;
    if (cudaMemsetAsync(peak_bits, 0, 2 * BH * D * 4, st) != cudaSuccess) return VC_ERR_LAUNCH;
    auto ks = v_block_stats<T, D>;
    cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
    ks<<<dim3(tiles, BH), kTileThreads, G::kSmem, st>>>(static_cast<const T*>(a.v), a.H, a.S, a.sb, a.sh, a.ss,
                                                        a.perm, ws_mean, peak_bits, mabs_bits, tiles);
    v_channel_scales<D><<<BH, D, 0, st>>>(peak_bits, mabs_bits, a.vs);
    auto kq = v_tile_quant<T, D, kResidualChannel>;
    cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
    kq<<<dim3(tiles, BH), kTileThreads, G::kSmem, st>>>(static_cast<const T*>(a.v), a.H, a.S, a.sb, a.sh, a.ss,
                                                        a.perm, nullptr, ws_mean, a.vs, means, a.v8, tiles, 1);
  } else {
    auto kq = v_tile_quant<T, D, kResidualBlock>;
    cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
    kq<<<dim3(tiles, BH), kTileThreads, G::kSmem, st>>>(static_cast<const T*>(a.v), a.H, a.S, a.sb, a.sh, a.ss,
                                                        a.perm, nullptr, nullptr, a.vs, means, a.v8, tiles, a.demean);
  }
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

}  // namespace

int64_t prep_v_channel_workspace(int64_t B, int64_t H, int64_t, int64_t D) { return B * H * D * 4 + 256; }

int64_t prep_v_blocks_workspace(int64_t B, int64_t H, int64_t S, int64_t D) {
  return (B * H * ((S + 127) / 128) * D + 2 * B * H * D) * 4 + 256;   // tile means + two maxima per channel
}

#define VCB_DISPATCH_V(FN)                                                    \
  if (a.dtype == VC_DTYPE_BF16)                                               \
    return a.D == 64 ? FN<__nv_bfloat16, 64>(a, st) : FN<__nv_bfloat16, 128>(a, st); \
  if (a.dtype == VC_DTYPE_F16) return a.D == 64 ? FN<__half, 64>(a, st) : FN<__half, 128>(a, st); \
  if (a.dtype == VC_DTYPE_F32) return a.D == 64 ? FN<float, 64>(a, st) : FN<float, 128>(a, st); \
  return VC_ERR_ARG;

int prep_v_channel(const PrepVArgs& a, cudaStream_t st) { VCB_DISPATCH_V(launch_v_channel) }
int prep_v_blocks(const PrepVArgs& a, cudaStream_t st) { VCB_DISPATCH_V(launch_v_blocks) }
#undef VCB_DISPATCH_V

cudaError_t prep_v_error_word(uint32_t* code, bool clear) { return read_tu_error_word(code, clear); }

}  // namespace vcb
