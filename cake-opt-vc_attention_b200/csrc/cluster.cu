// V grouping for sm_100a: Lloyd clustering of V tokens per head and a stable
// counting sort of the final labels (the token permutation used by V
// smoothing).
//
// Policy (csrc/vc/clustering.cu:22-166, src/vc_attention/core.py:153-178):
//   * count = min(clusters, S) centres initialised from tokens
//     trunc(linspace_fp32(0, S-1, count));
//   * ``iterations`` assignments; all but the last also update centres
//     (sum / count, empty centres keep their value);
//   * distance = (|x|^2 + |c|^2) - 2 x.c with the reference's four-lanes-per-
//     row FP32 arithmetic; ties pick the lowest centre index;
//   * stable order of tokens inside each cluster.
// Unlike the reference (shared-memory atomics), the centre statistics here are
// accumulated in a fixed order, so results are bitwise reproducible.
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kMaxC = 8;
constexpr int kRows = 128;
constexpr int kChunk = 1024;  // tokens per sort chunk

// trunc(at::linspace(0, n-1, count) as FP32): index i < count/2 uses
// start + step*i, otherwise end - step*(count-1-i).
__device__ __forceinline__ int64_t linspace_id(int64_t n, int count, int i) {
  if (count == 1) return 0;
  const float end = static_cast<float>(n - 1);
  const float step = __fdiv_rn(end, static_cast<float>(count - 1));
  float v;
  if (i < count / 2) v = __fadd_rn(0.f, __fmul_rn(step, static_cast<float>(i)));
  else v = __fsub_rn(end, __fmul_rn(step, static_cast<float>(count - 1 - i)));
  return static_cast<int64_t>(truncf(v));
}

template <typename T, int D>
__global__ void grp_init(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb, int64_t sh, int64_t ss, int count,
                         float* __restrict__ centers) {
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  for (int i = threadIdx.x; i < count * D; i += blockDim.x) {
    const int c = i / D, d = i % D;
    const int64_t id = linspace_id(S, count, c);
    centers[(bh * count + c) * D + d] = to_f32(v[b * sb + h * sh + id * ss + d]);
  }
}

__device__ __forceinline__ float sum_four(float x) {
  x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, 1, 4));
  return __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, 2, 4));
}

// Assign each token of a 128-token tile to its nearest centre.  With STATS,
// also write this tile's per-centre channel sums and counts, accumulated by
// thread d over the tile's rows in token order.
template <typename T, int D, bool STATS>
__global__ void __launch_bounds__(128) grp_assign(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb, int64_t sh,
                                                  int64_t ss, int count, const float* __restrict__ centers,
                                                  int32_t* __restrict__ labels, float* __restrict__ psum,
                                                  int32_t* __restrict__ pcnt, int64_t tiles) {
  extern __shared__ __align__(16) float grp_smem[];
  float(*cen)[D] = reinterpret_cast<float(*)[D]>(grp_smem);
  float* cnorm = grp_smem + kMaxC * D;
  float(*xs)[D + 1] = reinterpret_cast<float(*)[D + 1]>(grp_smem + kMaxC * D + kMaxC);
  int* lab = reinterpret_cast<int*>(grp_smem + kMaxC * D + kMaxC + kRows * (D + 1));
  const int64_t bh = blockIdx.y, tile = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const int lane = threadIdx.x & 3, group = threadIdx.x >> 2;
  for (int i = threadIdx.x; i < kMaxC * D; i += 128)
    cen[i / D][i % D] = i < count * D ? centers[bh * count * D + i] : 0.f;
  // stage the tile as FP32 (zeros past S)
  constexpr int EPT = 16 / sizeof(T);
  constexpr int CPR = D / EPT;
  for (int i = threadIdx.x; i < kRows * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR;
    const int64_t row = tile * kRows + r;
    float x[EPT];
    if (row < S) {
      load_vec<T, EPT>(v + b * sb + h * sh + row * ss + c * EPT, x);
    } else {
#pragma unroll
      for (int e = 0; e < EPT; ++e) x[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < EPT; ++e) xs[r][c * EPT + e] = x[e];
  }
  __syncthreads();
  {
    float cn = 0.f;
    if (group < kMaxC) {
#pragma unroll 8
      for (int j = 0; j < D / 4; ++j) {
        const float x = cen[group][j * 4 + lane];
        cn = __fadd_rn(cn, __fmul_rn(x, x));
      }
    }
    cn = sum_four(cn);
    if (group < kMaxC && lane == 0) cnorm[group] = cn;
  }
  __syncthreads();
  for (int off = 0; off < kRows; off += 32) {
    const int r = off + group;
    const int64_t row = tile * kRows + r;
    // all centres' dot products advance together (8 independent FMA chains);
    // each one still sums its lane's elements in the same order
    float norm = 0.f;
    float dot[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) dot[c] = 0.f;
#pragma unroll 4
    for (int j = 0; j < D / 4; ++j) {
      const float x = xs[r][j * 4 + lane];
      norm = __fadd_rn(norm, __fmul_rn(x, x));
#pragma unroll
      for (int c = 0; c < kMaxC; ++c) dot[c] = __fmaf_rn(x, cen[c][j * 4 + lane], dot[c]);
    }
    norm = sum_four(norm);
    float best_d = __int_as_float(0x7f800000);
    int best = 0;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
      const float dc = sum_four(dot[c]);
      const float dist = __fsub_rn(__fadd_rn(norm, cnorm[c]), __fmul_rn(2.f, dc));
      if (c < count && dist < best_d) {
        best_d = dist;
        best = c;
      }
    }
    best = __shfl_sync(0xffffffffu, best, 0, 4);
    if (lane == 0) {
      lab[r] = row < S ? best : -1;
      if (row < S) labels[bh * S + row] = best;
    }
  }
  if constexpr (STATS) {
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += 128) {
      float acc[kMaxC];
#pragma unroll
      for (int c = 0; c < kMaxC; ++c) acc[c] = 0.f;
      for (int r = 0; r < kRows; ++r) {
        const int c = lab[r];
        const float x = xs[r][d];
#pragma unroll
        for (int cc = 0; cc < kMaxC; ++cc)
          if (cc == c) acc[cc] = __fadd_rn(acc[cc], x);
      }
#pragma unroll
      for (int c = 0; c < kMaxC; ++c)
        if (c < count) psum[((bh * tiles + tile) * count + c) * D + d] = acc[c];
    }
    if (threadIdx.x < count) {
      int n = 0;
      for (int r = 0; r < kRows; ++r) n += lab[r] == static_cast<int>(threadIdx.x);
      pcnt[(bh * tiles + tile) * count + threadIdx.x] = n;
    }
  }
}

// centre = (sum over tiles, in tile order) / count; empty centres unchanged.
template <int D>
__global__ void grp_update(float* __restrict__ centers, const float* __restrict__ psum,
                           const int32_t* __restrict__ pcnt, int count, int64_t tiles) {
  const int c = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int d = threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  int64_t n = 0;
  for (int64_t t = 0; t < tiles; ++t) {
    const int64_t idx = (bh * tiles + t) * count + c;
    s = __fadd_rn(s, psum[idx * D + d]);
    n += pcnt[idx];
  }
  if (n) centers[(bh * count + c) * D + d] = __fdiv_rn(s, static_cast<float>(n));
}

// Stable counting sort, step 1: label histogram per chunk of kChunk tokens.
__global__ void grp_hist(const int32_t* __restrict__ labels, int64_t S, int count, int32_t* __restrict__ hist,
                         int64_t nchunk) {
  __shared__ int h[kMaxC];
  const int64_t bh = blockIdx.y, chunk = blockIdx.x;
  if (threadIdx.x < kMaxC) h[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t i = chunk * kChunk + threadIdx.x; i < min64(S, (chunk + 1) * kChunk); i += blockDim.x)
    atomicAdd(&h[labels[bh * S + i]], 1);
  __syncthreads();
  if (threadIdx.x < count) hist[(bh * nchunk + chunk) * count + threadIdx.x] = h[threadIdx.x];
}

// Step 2: exclusive offsets, cluster-major then chunk order.
__global__ void grp_scan(int32_t* __restrict__ hist, int count, int64_t nchunk) {
  const int64_t bh = blockIdx.x;
  if (threadIdx.x != 0) return;
  int64_t run = 0;
  for (int c = 0; c < count; ++c)
    for (int64_t k = 0; k < nchunk; ++k) {
      int32_t* p = hist + (bh * nchunk + k) * count + c;
      const int32_t n = *p;
      *p = static_cast<int32_t>(run);
      run += n;
    }
}

// Step 3: one warp per chunk places tokens in order (ranks via match_any).
__global__ void grp_scatter(const int32_t* __restrict__ labels, int64_t S, int count, const int32_t* __restrict__ offs,
                            int64_t nchunk, int64_t* __restrict__ perm) {
  __shared__ int run[kMaxC];
  const int64_t bh = blockIdx.y, chunk = blockIdx.x;
  const int lane = threadIdx.x;
  if (lane < count) run[lane] = offs[(bh * nchunk + chunk) * count + lane];
  __syncwarp();
  const int64_t end = min64(S, (chunk + 1) * kChunk);
  for (int64_t base = chunk * kChunk; base < end; base += 32) {
    const int64_t i = base + lane;
    const bool active = i < end;
    const int lb = active ? labels[bh * S + i] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, lb);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (active) perm[bh * S + run[lb] + rank] = i;
    __syncwarp();
    if (active && rank == 0) run[lb] += __popc(peers);
    __syncwarp();
  }
}

template <typename T, int D>
int launch_group(const GroupArgs& a, cudaStream_t st) {
  const int64_t BH = a.B * a.H, S = a.S;
  const int count = static_cast<int>(min64(a.clusters, S));
  const int64_t tiles = (S + kRows - 1) / kRows, nchunk = (S + kChunk - 1) / kChunk;
  char* w = static_cast<char*>(a.workspace);
  float* centers = reinterpret_cast<float*>(w);
  w += BH * kMaxC * D * 4;
  int32_t* labels = reinterpret_cast<int32_t*>(w);
  w += ((BH * S * 4 + 255) / 256) * 256;
  float* psum = reinterpret_cast<float*>(w);
  w += BH * tiles * kMaxC * D * 4;
  int32_t* pcnt = reinterpret_cast<int32_t*>(w);
  w += ((BH * tiles * kMaxC * 4 + 255) / 256) * 256;
  int32_t* hist = reinterpret_cast<int32_t*>(w);
  const T* v = static_cast<const T*>(a.v);
  const int smem = (kMaxC * D + kMaxC + kRows * (D + 1) + kRows) * 4;
  cudaFuncSetAttribute(grp_assign<T, D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(grp_assign<T, D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (a.centers_in)
    cudaMemcpyAsync(centers, a.centers_in, BH * count * D * 4, cudaMemcpyDeviceToDevice, st);
  else
    grp_init<T, D><<<BH, 128, 0, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, centers);
  for (int it = 0; it < a.iterations; ++it) {
    if (it + 1 < a.iterations) {
      grp_assign<T, D, true><<<dim3(tiles, BH), 128, smem, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, centers, labels,
                                                              psum, pcnt, tiles);
      grp_update<D><<<dim3(count, BH), D, 0, st>>>(centers, psum, pcnt, count, tiles);
    } else {
      grp_assign<T, D, false><<<dim3(tiles, BH), 128, smem, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, centers, labels,
                                                               nullptr, nullptr, tiles);
    }
  }
  grp_hist<<<dim3(nchunk, BH), 256, 0, st>>>(labels, S, count, hist, nchunk);
  grp_scan<<<BH, 32, 0, st>>>(hist, count, nchunk);
  grp_scatter<<<dim3(nchunk, BH), 32, 0, st>>>(labels, S, count, hist, nchunk, a.perm_out);
  if (a.labels_out)
    cudaMemcpyAsync(a.labels_out, labels, BH * S * 4, cudaMemcpyDeviceToDevice, st);
  if (a.centers_out)
    cudaMemcpyAsync(a.centers_out, centers, BH * count * D * 4, cudaMemcpyDeviceToDevice, st);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

}  // namespace

int64_t group_values_workspace(int64_t B, int64_t H, int64_t S, int64_t D, int) {
  const int64_t BH = B * H, tiles = (S + kRows - 1) / kRows, nchunk = (S + kChunk - 1) / kChunk;
  auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
  return up(BH * kMaxC * D * 4) + up(BH * S * 4) + up(BH * tiles * kMaxC * D * 4) + up(BH * tiles * kMaxC * 4) +
         up(BH * nchunk * kMaxC * 4) + 256;
}

int group_values(const GroupArgs& a, cudaStream_t st) {
  if (min64(a.clusters, a.S) > kMaxC) {
    set_last_error("vc_group_values: more than %d effective clusters is not supported by this build", kMaxC);
    return VC_ERR_UNSUPPORTED;
  }
  if (a.dtype == VC_DTYPE_BF16) return a.D == 64 ? launch_group<__nv_bfloat16, 64>(a, st) : launch_group<__nv_bfloat16, 128>(a, st);
  if (a.dtype == VC_DTYPE_F16) return a.D == 64 ? launch_group<__half, 64>(a, st) : launch_group<__half, 128>(a, st);
  if (a.dtype == VC_DTYPE_F32) return a.D == 64 ? launch_group<float, 64>(a, st) : launch_group<float, 128>(a, st);
  return VC_ERR_ARG;
}

}  // namespace vcb
