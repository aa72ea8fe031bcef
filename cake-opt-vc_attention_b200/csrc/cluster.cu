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
// accumulated in a fixed order (16-bit inputs: a tensor-core product whose
// accumulation order the hardware fixes; FP32 inputs: token order), so
// results are bitwise reproducible.
//
// More than 8 effective centres (up to 256) take the wide path, the policy of
// the reference's public entry for that range (csrc/vc/pybind.cpp:6-44, its
// legacy Lloyd loop): distances (|x|^2 + |c|^2) - 2 x.c in FP32 (the
// reference uses a matmul; rounding order differs, ties still pick the lowest
// centre), centre = member mean (empty centres keep their value), stable
// argsort of the final labels.  Here: assignment kernel with the head's
// centres in shared memory, one token per thread; then the stable counting
// sort below; then each centre's mean summed over its members in sorted
// token order (deterministic, no atomics).
#include "common.cuh"
#include "kernels.h"

namespace vcb {
namespace {

constexpr int kMaxC = 8;        // fused path
constexpr int kWideMaxC = 256;  // wide path (the reference's public maximum)
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

// Row stride of the staged tile: the row plus 16 bytes, so that 8 threads
// reading 16 bytes of 8 consecutive rows hit 8 different bank quads.
template <typename T, int D>
struct GrpTile {
  static constexpr int kRowBytes = D * int(sizeof(T)) + 16;
  static constexpr int kChunks = D * int(sizeof(T)) / 16;   // 16-byte chunks per row
  static constexpr int kEl = 16 / int(sizeof(T));           // elements per chunk
  static constexpr int kBytes = kRows * kRowBytes;
  static constexpr int kSmem = kMaxC * D * 4 + kMaxC * 4 + kBytes + kRows * 4;
};

// 16 bytes of a staged row as floats (exact conversions).
template <typename T>
__device__ __forceinline__ void chunk_f32(const uint8_t* p, float (&x)[16 / sizeof(T)]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __uint_as_float(w[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      T lo, hi;
      const uint16_t a = static_cast<uint16_t>(w[i] & 0xffffu), b = static_cast<uint16_t>(w[i] >> 16);
      memcpy(&lo, &a, 2);
      memcpy(&hi, &b, 2);
      x[2 * i] = to_f32(lo);
      x[2 * i + 1] = to_f32(hi);
    }
  }
}

// One m16n8k16 tensor-core product with FP32 accumulation, A row-major and B
// column-major (16-bit inputs).  Used for the grouping statistics: the sums
// of a tile's rows per centre are onehot(labels)^T x tile, whose products
// (x * 1 or x * 0) are exact; the accumulation order is the hardware's fixed
// one, so the sums are deterministic.
template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Four transposed 8x8 16-bit matrices from shared memory (lane l gives the
// address of row l % 8 of matrix l / 8).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Assign each token of a 128-token tile to its nearest centre.  With STATS,
// also write this tile's per-centre channel sums and counts: for 16-bit
// inputs as onehot(labels)^T x tile on the tensor core (warp w: channels
// 32w.. of D = 128, 16w.. of D = 64), for FP32 inputs by thread d over the
// tile's rows in token order.
//
// The tile is staged in its input type by cp.async (every copy in flight at
// once).  Thread r owns token r: for every centre it keeps the four partial
// dot products of channel residues 0..3 (channel 4j+l feeds partial l, in j
// order) and the four partial squared norms, and combines each as
// (p0 + p1) + (p2 + p3) -- the arithmetic of four lanes per row reduced by
// xor-shuffles, computed by one thread.
template <typename T, int D, bool STATS>
__global__ void __launch_bounds__(128) grp_assign(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb, int64_t sh,
                                                  int64_t ss, int count, const float* __restrict__ centers,
                                                  int32_t* __restrict__ labels, float* __restrict__ psum,
                                                  int32_t* __restrict__ pcnt, int64_t tiles) {
  using L = GrpTile<T, D>;
  extern __shared__ __align__(16) uint8_t grp_raw[];
  float(*cen)[D] = reinterpret_cast<float(*)[D]>(grp_raw);
  float* cnorm = reinterpret_cast<float*>(grp_raw + kMaxC * D * 4);
  uint8_t* xs = grp_raw + kMaxC * D * 4 + kMaxC * 4;
  int* lab = reinterpret_cast<int*>(xs + L::kBytes);
  const int64_t bh = blockIdx.y, tile = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const T* vbh = v + b * sb + h * sh;
  for (int i = threadIdx.x; i < kRows * L::kChunks; i += 128) {
    const int r = i / L::kChunks, c = i - r * L::kChunks;
    const int64_t row = tile * kRows + r;
    const bool in = row < S;
    cp_async16(xs + r * L::kRowBytes + c * 16, vbh + (in ? row : 0) * ss + c * L::kEl, in ? 16u : 0u);
  }
  for (int i = threadIdx.x; i < kMaxC * D / 4; i += 128) {
    const bool in = i < count * D / 4;
    cp_async16(&cen[0][0] + i * 4, centers + bh * count * D + (in ? i * 4 : 0), in ? 16u : 0u);
  }
  cp_async_wait_all();
  __syncthreads();
  if (threadIdx.x < 32) {
    // |c|^2 with four lanes per centre (lane l: channels 4j+l in j order)
    const int lane = threadIdx.x & 3, group = threadIdx.x >> 2;
    float cn = 0.f;
#pragma unroll 8
    for (int j = 0; j < D / 4; ++j) {
      const float x = cen[group][j * 4 + lane];
      cn = __fadd_rn(cn, __fmul_rn(x, x));
    }
    cn = sum_four(cn);
    if (lane == 0) cnorm[group] = cn;
  }
  __syncthreads();
  {
    const int r = threadIdx.x;
    const int64_t row = tile * kRows + r;
    const uint8_t* xrow = xs + r * L::kRowBytes;
    // partials l = 0, 1 and l = 2, 3 as packed FP32 pairs: every half is the
    // same chain of .rn operations as the scalar arithmetic, in half the
    // instructions
    uint64_t nrm01 = 0, nrm23 = 0;
    uint64_t dot01[kMaxC], dot23[kMaxC];
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) dot01[c] = dot23[c] = 0;
#pragma unroll 2
    for (int k = 0; k < L::kChunks; ++k) {
      float x[L::kEl];
      chunk_f32<T>(xrow + k * 16, x);
#pragma unroll
      for (int q = 0; q < L::kEl / 4; ++q) {
        const int j = k * (L::kEl / 4) + q;   // channels 4j .. 4j+3
        const uint64_t x01 = pk2f(x[4 * q], x[4 * q + 1]), x23 = pk2f(x[4 * q + 2], x[4 * q + 3]);
        nrm01 = f2_add(nrm01, f2_mul(x01, x01));
        nrm23 = f2_add(nrm23, f2_mul(x23, x23));
#pragma unroll
        for (int c = 0; c < kMaxC; ++c) {
          const ulonglong2 cv = *reinterpret_cast<const ulonglong2*>(&cen[c][4 * j]);   // (c0, c1), (c2, c3)
          dot01[c] = f2_fma(x01, cv.x, dot01[c]);
          dot23[c] = f2_fma(x23, cv.y, dot23[c]);
        }
      }
    }
    uint32_t n0, n1, n2, n3;
    up2(nrm01, n0, n1);
    up2(nrm23, n2, n3);
    const float norm = __fadd_rn(__fadd_rn(__uint_as_float(n0), __uint_as_float(n1)),
                                 __fadd_rn(__uint_as_float(n2), __uint_as_float(n3)));
    float best_d = __int_as_float(0x7f800000);
    int best = 0;
#pragma unroll
    for (int c = 0; c < kMaxC; ++c) {
      uint32_t d0, d1, d2, d3;
      up2(dot01[c], d0, d1);
      up2(dot23[c], d2, d3);
      const float dc = __fadd_rn(__fadd_rn(__uint_as_float(d0), __uint_as_float(d1)),
                                 __fadd_rn(__uint_as_float(d2), __uint_as_float(d3)));
      const float dist = __fsub_rn(__fadd_rn(norm, cnorm[c]), __fmul_rn(2.f, dc));
      if (c < count && dist < best_d) {
        best_d = dist;
        best = c;
      }
    }
    lab[r] = row < S ? best : -1;
    if (row < S) labels[bh * S + row] = best;
  }
  if constexpr (STATS && sizeof(T) == 2) {
    __syncthreads();
    constexpr int kNB = D / 8 / 4;   // 8-channel blocks per warp
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t one = std::is_same<T, __half>::value ? 0x3C00u : 0x3F80u;
    float acc[kNB][4];
#pragma unroll
    for (int nb = 0; nb < kNB; ++nb)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[nb][i] = 0.f;
    const uint32_t xs0 = smem_u32(xs);
#pragma unroll 2
    for (int kb = 0; kb < kRows / 16; ++kb) {
      // A = onehot: row g (centre g) of rows kb*16 + {2t, 2t+1, 2t+8, 2t+9}; centres 8..15 are zero
      const int r0 = kb * 16 + 2 * t;
      uint32_t a[4];
      a[0] = (lab[r0] == g ? one : 0u) | ((lab[r0 + 1] == g ? one : 0u) << 16);
      a[2] = (lab[r0 + 8] == g ? one : 0u) | ((lab[r0 + 9] == g ? one : 0u) << 16);
      a[1] = a[3] = 0u;
#pragma unroll
      for (int nb = 0; nb < kNB; nb += 2) {
        // B = rows kb*16 .. +15 of channel blocks 8*(warp*kNB + nb) and the next
        const int m = lane >> 3, k = (m & 1) * 8 + (lane & 7);
        const int cb = warp * kNB + nb + (m >> 1);
        uint32_t b[4];
        ldmatrix_x4_trans(b, xs0 + (kb * 16 + k) * L::kRowBytes + cb * 16);
        mma_16816<T>(acc[nb], a, b[0], b[1]);
        mma_16816<T>(acc[nb + 1], a, b[2], b[3]);
      }
    }
    if (g < count) {
#pragma unroll
      for (int nb = 0; nb < kNB; ++nb) {
        const int ch = (warp * kNB + nb) * 8 + 2 * t;
        *reinterpret_cast<float2*>(psum + ((bh * tiles + tile) * count + g) * D + ch) = make_float2(acc[nb][0], acc[nb][1]);
      }
    }
    if (threadIdx.x < count) {
      int n = 0;
      for (int r = 0; r < kRows; ++r) n += lab[r] == static_cast<int>(threadIdx.x);
      pcnt[(bh * tiles + tile) * count + threadIdx.x] = n;
    }
  } else if constexpr (STATS) {
    __syncthreads();
    // thread d sums channel d of each centre's rows in token order; the
    // label is the same for the whole warp, so the switch does not diverge
    for (int d = threadIdx.x; d < D; d += 128) {
      float acc[kMaxC];
#pragma unroll
      for (int c = 0; c < kMaxC; ++c) acc[c] = 0.f;
      const uint8_t* col = xs + (d / L::kEl) * 16 + (d % L::kEl) * int(sizeof(T));
      for (int r = 0; r < kRows; ++r) {
        T e;
        memcpy(&e, col + r * L::kRowBytes, sizeof(T));
        const float x = to_f32(e);
        switch (lab[r]) {
          case 0: acc[0] = __fadd_rn(acc[0], x); break;
          case 1: acc[1] = __fadd_rn(acc[1], x); break;
          case 2: acc[2] = __fadd_rn(acc[2], x); break;
          case 3: acc[3] = __fadd_rn(acc[3], x); break;
          case 4: acc[4] = __fadd_rn(acc[4], x); break;
          case 5: acc[5] = __fadd_rn(acc[5], x); break;
          case 6: acc[6] = __fadd_rn(acc[6], x); break;
          case 7: acc[7] = __fadd_rn(acc[7], x); break;
          default: break;
        }
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

// centre = (sum over tiles) / count; empty centres unchanged.  8*D threads
// per (centre, head): group g sums the g-th eighth of the tiles in tile order,
// and thread d of group 0 combines the eight sums in a fixed tree, so the
// order is deterministic while eight chains run at once.
constexpr int kUpdateGroups = 8;
template <int D>
__global__ void __launch_bounds__(kUpdateGroups * D) grp_update(float* __restrict__ centers,
                                                                 const float* __restrict__ psum,
                                                                 const int32_t* __restrict__ pcnt, int count,
                                                                 int64_t tiles) {
  __shared__ float part[kUpdateGroups][D];
  __shared__ int64_t npart[kUpdateGroups];
  const int c = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int d = threadIdx.x % D, g = threadIdx.x / D;
  const int64_t chunk = (tiles + kUpdateGroups - 1) / kUpdateGroups;
  const int64_t t0 = min64(tiles, g * chunk), t1 = min64(tiles, t0 + chunk);
  float s = 0.f;
  int64_t n = 0;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t idx = (bh * tiles + t) * count + c;
    s = __fadd_rn(s, psum[idx * D + d]);
    n += pcnt[idx];
  }
  part[g][d] = s;
  if (d == 0) npart[g] = n;
  __syncthreads();
  if (g == 0) {
    const float tot = __fadd_rn(__fadd_rn(__fadd_rn(part[0][d], part[1][d]), __fadd_rn(part[2][d], part[3][d])),
                                __fadd_rn(__fadd_rn(part[4][d], part[5][d]), __fadd_rn(part[6][d], part[7][d])));
    int64_t nt = 0;
#pragma unroll
    for (int i = 0; i < kUpdateGroups; ++i) nt += npart[i];
    if (nt) centers[(bh * count + c) * D + d] = __fdiv_rn(tot, static_cast<float>(nt));
  }
}

// Stable counting sort, step 1: label histogram per chunk of kChunk tokens.
__global__ void grp_hist(const int32_t* __restrict__ labels, int64_t S, int count, int32_t* __restrict__ hist,
                         int64_t nchunk) {
  __shared__ int h[kWideMaxC];
  const int64_t bh = blockIdx.y, chunk = blockIdx.x;
  if (threadIdx.x < kWideMaxC) h[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t i = chunk * kChunk + threadIdx.x; i < min64(S, (chunk + 1) * kChunk); i += blockDim.x)
    atomicAdd(&h[labels[bh * S + i]], 1);
  __syncthreads();
  if (threadIdx.x < count) hist[(bh * nchunk + chunk) * count + threadIdx.x] = h[threadIdx.x];
}

// Step 2: exclusive offsets, cluster-major then chunk order.  One warp per
// head: 32 chunks at a time, an inclusive shuffle scan plus the running total.
__global__ void grp_scan(int32_t* __restrict__ hist, int count, int64_t nchunk) {
  const int64_t bh = blockIdx.x;
  const int lane = threadIdx.x;
  int32_t run = 0;
  for (int c = 0; c < count; ++c)
    for (int64_t k0 = 0; k0 < nchunk; k0 += 32) {
      const int64_t k = k0 + lane;
      int32_t* p = hist + (bh * nchunk + k) * count + c;
      const int32_t n = k < nchunk ? *p : 0;
      int32_t incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (k < nchunk) *p = run + incl - n;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
}

// Step 3: one warp per chunk places tokens in order (ranks via match_any).
__global__ void grp_scatter(const int32_t* __restrict__ labels, int64_t S, int count, const int32_t* __restrict__ offs,
                            int64_t nchunk, int64_t* __restrict__ perm) {
  __shared__ int run[kWideMaxC];
  const int64_t bh = blockIdx.y, chunk = blockIdx.x;
  const int lane = threadIdx.x;
  for (int c = lane; c < count; c += 32) run[c] = offs[(bh * nchunk + chunk) * count + c];
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

// Wide path, assignment: the head's ``count`` centres (FP32) and their
// squared norms in shared memory; thread r owns token r of a 128-token tile
// with the token's channels in registers.  dist = (|x|^2 + |c|^2) - 2 x.c,
// the lowest index wins ties.
template <typename T, int D>
__global__ void __launch_bounds__(128) grp_assign_wide(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb,
                                                       int64_t sh, int64_t ss, int count,
                                                       const float* __restrict__ centers, int32_t* __restrict__ labels) {
  extern __shared__ __align__(16) float wide_sm[];
  float* cen = wide_sm;                 // [count][D]
  float* cnorm = wide_sm + count * D;   // [count]
  const int64_t bh = blockIdx.y, tile = blockIdx.x;
  const int64_t b = bh / H, h = bh - b * H;
  const float4* src = reinterpret_cast<const float4*>(centers + bh * count * D);
  for (int i = threadIdx.x; i < count * D / 4; i += 128) reinterpret_cast<float4*>(cen)[i] = src[i];
  __syncthreads();
  for (int c = threadIdx.x; c < count; c += 128) {
    float n = 0.f;
    for (int d = 0; d < D; ++d) n = __fadd_rn(n, __fmul_rn(cen[c * D + d], cen[c * D + d]));
    cnorm[c] = n;
  }
  __syncthreads();
  const int64_t row = tile * 128 + threadIdx.x;
  if (row >= S) return;
  float x[D];
  load_vec<T, D>(v + b * sb + h * sh + row * ss, x);
  float norm = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) norm = __fadd_rn(norm, __fmul_rn(x[d], x[d]));
  float best_d = __int_as_float(0x7f800000);
  int best = 0;
  for (int c = 0; c < count; ++c) {
    const float4* cr = reinterpret_cast<const float4*>(cen + c * D);
    float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int d4 = 0; d4 < D / 4; ++d4) {
      const float4 cv = cr[d4];
      p[0] = __fmaf_rn(x[4 * d4 + 0], cv.x, p[0]);
      p[1] = __fmaf_rn(x[4 * d4 + 1], cv.y, p[1]);
      p[2] = __fmaf_rn(x[4 * d4 + 2], cv.z, p[2]);
      p[3] = __fmaf_rn(x[4 * d4 + 3], cv.w, p[3]);
    }
    const float dot = __fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3]));
    const float dist = __fsub_rn(__fadd_rn(norm, cnorm[c]), __fmul_rn(2.f, dot));
    if (dist < best_d) {
      best_d = dist;
      best = c;
    }
  }
  labels[bh * S + row] = best;
}

// Wide path, update: centre c = the mean of its members, summed in sorted
// (stable, token) order; members are perm[start_c .. start_c+1) from the
// counting sort.  Thread d owns channel d; 16 member rows are loaded at once.
template <typename T, int D>
__global__ void grp_update_wide(const T* __restrict__ v, int64_t H, int64_t S, int64_t sb, int64_t sh, int64_t ss,
                                int count, const int32_t* __restrict__ offs, int64_t nchunk,
                                const int64_t* __restrict__ perm, float* __restrict__ centers) {
  const int c = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh - b * H;
  const int d = threadIdx.x;
  const int64_t start = offs[(bh * nchunk) * count + c];
  const int64_t end = c + 1 < count ? offs[(bh * nchunk) * count + c + 1] : S;
  const T* vbh = v + b * sb + h * sh + d;
  const int64_t* pr = perm + bh * S;
  float s = 0.f;
  int64_t i = start;
  for (; i + 16 <= end; i += 16) {
    float x[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) x[u] = to_f32(vbh[pr[i + u] * ss]);
#pragma unroll
    for (int u = 0; u < 16; ++u) s = __fadd_rn(s, x[u]);
  }
  for (; i < end; ++i) s = __fadd_rn(s, to_f32(vbh[pr[i] * ss]));
  if (end > start) centers[(bh * count + c) * D + d] = __fdiv_rn(s, static_cast<float>(end - start));
}

template <typename T, int D>
int launch_group_wide(const GroupArgs& a, cudaStream_t st) {
  const int64_t BH = a.B * a.H, S = a.S;
  const int count = static_cast<int>(min64(a.clusters, S));
  const int64_t tiles = (S + 127) / 128, nchunk = (S + kChunk - 1) / kChunk;
  char* w = static_cast<char*>(a.workspace);
  float* centers = reinterpret_cast<float*>(w);
  w += ((BH * count * D * 4 + 255) / 256) * 256;
  int32_t* labels = reinterpret_cast<int32_t*>(w);
  w += ((BH * S * 4 + 255) / 256) * 256;
  int32_t* hist = reinterpret_cast<int32_t*>(w);
  const T* v = static_cast<const T*>(a.v);
  const int smem = count * D * 4 + count * 4;
  if (cudaFuncSetAttribute(grp_assign_wide<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return VC_ERR_LAUNCH;
  if (a.centers_in)
    cudaMemcpyAsync(centers, a.centers_in, BH * count * D * 4, cudaMemcpyDeviceToDevice, st);
  else
    grp_init<T, D><<<BH, 128, 0, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, centers);
  for (int it = 0; it < a.iterations; ++it) {
    grp_assign_wide<T, D><<<dim3(tiles, BH), 128, smem, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, centers, labels);
    // the stable sort of the labels: the permutation (final) or the members per centre (update)
    grp_hist<<<dim3(nchunk, BH), 256, 0, st>>>(labels, S, count, hist, nchunk);
    grp_scan<<<BH, 32, 0, st>>>(hist, count, nchunk);
    grp_scatter<<<dim3(nchunk, BH), 32, 0, st>>>(labels, S, count, hist, nchunk, a.perm_out);
    if (it + 1 < a.iterations)
      grp_update_wide<T, D><<<dim3(count, BH), D, 0, st>>>(v, a.H, S, a.sb, a.sh, a.ss, count, hist, nchunk,
                                                           a.perm_out, centers);
  }
  if (a.labels_out)
    cudaMemcpyAsync(a.labels_out, labels, BH * S * 4, cudaMemcpyDeviceToDevice, st);
  if (a.centers_out)
    cudaMemcpyAsync(a.centers_out, centers, BH * count * D * 4, cudaMemcpyDeviceToDevice, st);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
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
  const int smem = GrpTile<T, D>::kSmem;
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
      grp_update<D><<<dim3(count, BH), kUpdateGroups * D, 0, st>>>(centers, psum, pcnt, count, tiles);
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

int64_t group_values_workspace(int64_t B, int64_t H, int64_t S, int64_t D, int clusters) {
  const int64_t BH = B * H, tiles = (S + kRows - 1) / kRows, nchunk = (S + kChunk - 1) / kChunk;
  auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
  const int64_t count = min64(clusters, S);
  if (count > kMaxC)   // wide path: centres, labels, sort histogram
    return up(BH * count * D * 4) + up(BH * S * 4) + up(BH * nchunk * count * 4) + 256;
  return up(BH * kMaxC * D * 4) + up(BH * S * 4) + up(BH * tiles * kMaxC * D * 4) + up(BH * tiles * kMaxC * 4) +
         up(BH * nchunk * kMaxC * 4) + 256;
}

int group_values(const GroupArgs& a, cudaStream_t st) {
  const bool wide = min64(a.clusters, a.S) > kMaxC;
  if (a.dtype == VC_DTYPE_BF16) {
    if (wide) return a.D == 64 ? launch_group_wide<__nv_bfloat16, 64>(a, st) : launch_group_wide<__nv_bfloat16, 128>(a, st);
    return a.D == 64 ? launch_group<__nv_bfloat16, 64>(a, st) : launch_group<__nv_bfloat16, 128>(a, st);
  }
  if (a.dtype == VC_DTYPE_F16) {
    if (wide) return a.D == 64 ? launch_group_wide<__half, 64>(a, st) : launch_group_wide<__half, 128>(a, st);
    return a.D == 64 ? launch_group<__half, 64>(a, st) : launch_group<__half, 128>(a, st);
  }
  if (a.dtype == VC_DTYPE_F32) {
    if (wide) return a.D == 64 ? launch_group_wide<float, 64>(a, st) : launch_group_wide<float, 128>(a, st);
    return a.D == 64 ? launch_group<float, 64>(a, st) : launch_group<float, 128>(a, st);
  }
  return VC_ERR_ARG;
}

}  // namespace vcb
