// C ABI of the sm_100a VC-attention library (declared in include/vc_b200.h).
// Host-side argument validation happens here, before any launch; the kernels
// live in prep_qk.cu, prep_v.cu, cluster.cu and attention.cu.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "common.cuh"
#include "kernels.h"

namespace vcb {

namespace {
thread_local char t_last_error[512] = "";

__global__ void expcast_kernel(const float* __restrict__ x, uint8_t* __restrict__ y, int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const float u = __fmaf_rn(x[i], 11.541560173034668f, 119.6500015258789f);
    uint32_t c;
    asm("cvt.rni.sat.u8.f32 %0, %1;" : "=r"(c) : "f"(u));
    y[i] = static_cast<uint8_t>(min(c, 120u));
  }
}

// Failure-detection self-test: warp 0 waits, through the same bounded wait
// the kernels use, for an mbarrier phase that nothing completes.  The wait
// gives up after ``budget_ns``, sets kErrTimeoutSelfTest in the error word
// and the kernel returns normally.  ok_out[0] = 1 if the wait had succeeded.
__global__ void wait_selftest_kernel(uint64_t budget_ns, int* ok_out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // one arrival completes phase 0; none is made
    fence_barrier_init();
  }
  __syncthreads();
  const bool ok = __all_sync(0xffffffffu, mbar_wait_budget(&bar, 0, kErrTimeoutSelfTest, budget_ns));
  if (threadIdx.x == 0 && ok_out) ok_out[0] = ok ? 1 : 0;
}

// sm_100 check, cached per device.
int check_device() {
  static std::mutex mu;
  static int cache[64] = {0};  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("no current CUDA device");
    return VC_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cache[dev] = major == 10 ? 1 : 2;
  }
  if (cache[dev] != 1) {
    set_last_error("device %d is not sm_100 (B200); this library has no fallback", dev);
    return VC_ERR_UNSUPPORTED;
  }
  return VC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int elem_size(int dtype) { return dtype == VC_DTYPE_F32 ? 4 : 2; }

int check_common(const char* fn, int dtype, int64_t B, int64_t H, int64_t S, int64_t D) {
  if (dtype != VC_DTYPE_F16 && dtype != VC_DTYPE_BF16 && dtype != VC_DTYPE_F32) {
    set_last_error("%s: dtype must be VC_DTYPE_F16/BF16/F32", fn);
    return VC_ERR_ARG;
  }
  if (B < 1 || H < 1 || S < 1 || B * H > 65535 || S > (int64_t(1) << 31) - 256) {
    set_last_error("%s: need B,H,S >= 1, B*H <= 65535 and S < 2^31 (got %lld, %lld, %lld)", fn, (long long)B,
                   (long long)H, (long long)S);
    return VC_ERR_ARG;
  }
  if (D != 64 && D != 128) {
    set_last_error("%s: head dim must be 64 or 128 (got %lld)", fn, (long long)D);
    return VC_ERR_ARG;
  }
  return VC_OK;
}

int check_input(const char* fn, const char* name, const void* p, int dtype, int64_t sb, int64_t sh, int64_t ss) {
  const int es = elem_size(dtype);
  if (!p || !aligned16(p) || (sb * es) % 16 || (sh * es) % 16 || (ss * es) % 16 || ss < 1) {
    set_last_error("%s: %s must be a non-null 16-byte aligned pointer with 16-byte multiple strides", fn, name);
    return VC_ERR_ARG;
  }
  return VC_OK;
}

int finish(const char* fn, int rc) {
  if (rc == VC_ERR_LAUNCH) {
    const cudaError_t e = cudaGetLastError();
    set_last_error("%s: CUDA error %s", fn, cudaGetErrorString(e));
  }
  return rc;
}
}  // namespace

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int expcast_codes(const float* x, uint8_t* y, int64_t n, cudaStream_t st) {
  if (n == 0) return VC_OK;
  expcast_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH;
}

// Library-owned scratch for vc_prep_v_channel_static: the per-channel amax
// words (B*H*D uint32).  One array per device, shared by every call on that
// device; each call zeroes the words it uses on its own stream first.
static __device__ __align__(256) uint32_t g_static_scratch[VC_STATIC_SCRATCH_BYTES / 4];

namespace {
// Device address of g_static_scratch on the current device, resolved once per
// device (cudaGetSymbolAddress with that device current) and cached.
void* static_scratch() {
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p) {
      set_last_error("cudaGetSymbolAddress(static scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = p;
  }
  return cache[dev];
}
}  // namespace

}  // namespace vcb

using namespace vcb;

extern "C" {

int vc_api_version(void) { return VC_B200_API_VERSION; }

const char* vc_build_info(void) {
  return "vc_b200 sm_100a: tcgen05 kind::i8 QK^T + ExpCast E4M3 P + kind::f8f6f4 PV, TMA K/V ring, "
         "HBM-bound INT8/FP8 preparation; api 1";
}

const char* vc_last_error(void) { return t_last_error; }

int vc_error_read(int device, uint32_t* code, int clear) {
  if (!code) return VC_ERR_ARG;
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) {
    set_last_error("vc_error_read: bad device %d", device);
    return VC_ERR_ARG;
  }
  uint32_t words[6] = {0, 0, 0, 0, 0, 0};
  cudaError_t e = attention_error_word(&words[0], clear != 0);
  if (e == cudaSuccess) e = read_tu_error_word(&words[5], clear != 0);   // this file: the wait self-test
  if (e == cudaSuccess) e = prep_qk_error_word(&words[1], clear != 0);
  if (e == cudaSuccess) e = prep_v_error_word(&words[2], clear != 0);
  if (e == cudaSuccess) e = prep_hadamard_error_word(&words[3], clear != 0);
  if (e == cudaSuccess) e = tensor_peak_error_word(&words[4], clear != 0);
  *code = words[0] | words[1] | words[2] | words[3] | words[4] | words[5];
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_last_error("vc_error_read: %s", cudaGetErrorString(e));
    return VC_ERR_LAUNCH;
  }
  return VC_OK;
}

int vc_expcast_codes(const float* x, uint8_t* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) {
    set_last_error("vc_expcast_codes: bad arguments");
    return VC_ERR_ARG;
  }
  if (int rc = check_device()) return rc;
  return finish("vc_expcast_codes", expcast_codes(x, y, n, static_cast<cudaStream_t>(stream)));
}

int64_t vc_prep_qk_workspace_bytes(int64_t B, int64_t H, int64_t Sk, int64_t D) {
  return prep_qk_workspace(B, H, Sk, D);
}

int vc_prep_qk_int8(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                    int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s, int64_t k_stride_b, int64_t k_stride_h,
                    int64_t k_stride_s, const int64_t* perm, const void* km_in, void* km_out, int64_t mean_numel_out,
                    int64_t mean_numel_in, int8_t* q8, float* qs, int8_t* k8, float* ks, void* workspace,
                    int64_t workspace_bytes, void* stream) {
  const char* fn = "vc_prep_qk_int8";
  if (int rc = check_common(fn, dtype, B, H, Sq, D)) return rc;
  if (int rc = check_common(fn, dtype, B, H, Sk, D)) return rc;
  if (int rc = check_input(fn, "q", q, dtype, q_stride_b, q_stride_h, q_stride_s)) return rc;
  if (int rc = check_input(fn, "k", k, dtype, k_stride_b, k_stride_h, k_stride_s)) return rc;
  if (!q8 || !k8 || !qs || !ks || !aligned16(q8) || !aligned16(k8) || !aligned16(ks)) {
    set_last_error("%s: q8/k8/qs/ks must be non-null and 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  if (!km_in && (!workspace || workspace_bytes < prep_qk_workspace(B, H, Sk, D) || !aligned16(workspace))) {
    set_last_error("%s: workspace needs %lld bytes (16-byte aligned)", fn, (long long)prep_qk_workspace(B, H, Sk, D));
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  PrepQKArgs a{q, k, dtype, B, H, Sq, Sk, D, q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
               perm, km_in, km_out, mean_numel_out, mean_numel_in, q8, qs, k8, ks, workspace};
  return finish(fn, prep_qk(a, static_cast<cudaStream_t>(stream)));
}

int64_t vc_prep_qk_hadamard_workspace_bytes(int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                            int64_t k_quant_block) {
  if (k_quant_block < 128 || k_quant_block % 128 || k_quant_block > 4096) return -1;
  return prep_hadamard_workspace(B, H, Sq, Sk, D, k_quant_block);
}

int vc_prep_qk_hadamard_e4m3(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                             int64_t D, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
                             int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s, const int64_t* perm,
                             int k_smooth, const float* km_in, float* km_out, int64_t k_quant_block, uint8_t* q8,
                             float* qs, uint8_t* k8, float* ks, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  const char* fn = "vc_prep_qk_hadamard_e4m3";
  if (int rc = check_common(fn, dtype, B, H, Sq, D)) return rc;
  if (int rc = check_common(fn, dtype, B, H, Sk, D)) return rc;
  if (int rc = check_input(fn, "q", q, dtype, q_stride_b, q_stride_h, q_stride_s)) return rc;
  if (int rc = check_input(fn, "k", k, dtype, k_stride_b, k_stride_h, k_stride_s)) return rc;
  if (k_quant_block < 128 || k_quant_block % 128 || k_quant_block > 4096) {
    set_last_error("%s: k_quant_block must be a multiple of 128 in [128, 4096] (got %lld)", fn,
                   (long long)k_quant_block);
    return VC_ERR_ARG;
  }
  if (!q8 || !k8 || !qs || !ks || !aligned16(q8) || !aligned16(k8)) {
    set_last_error("%s: q8/k8/qs/ks must be non-null and q8/k8 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  const int64_t need = prep_hadamard_workspace(B, H, Sq, Sk, D, k_quant_block);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_last_error("%s: workspace needs %lld bytes (16-byte aligned)", fn, (long long)need);
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  PrepHadArgs a{q, k, dtype, B, H, Sq, Sk, D, q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
                perm, k_smooth ? 1 : 0, km_in, km_out, k_quant_block, q8, qs, k8, ks, workspace};
  return finish(fn, prep_hadamard(a, static_cast<cudaStream_t>(stream)));
}

int64_t vc_prep_v_channel_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D) {
  return prep_v_channel_workspace(B, H, S, D);
}

int vc_prep_v_channel(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                      int64_t stride_h, int64_t stride_s, const int64_t* perm, uint8_t* v8, float* vs, void* workspace,
                      int64_t workspace_bytes, void* stream) {
  const char* fn = "vc_prep_v_channel";
  if (int rc = check_common(fn, dtype, B, H, S, D)) return rc;
  if (int rc = check_input(fn, "v", v, dtype, stride_b, stride_h, stride_s)) return rc;
  if (!v8 || !vs || !aligned16(v8) || !aligned16(vs)) {
    set_last_error("%s: v8/vs must be non-null and 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  if (!workspace || workspace_bytes < prep_v_channel_workspace(B, H, S, D) || !aligned16(workspace)) {
    set_last_error("%s: workspace needs %lld bytes", fn, (long long)prep_v_channel_workspace(B, H, S, D));
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  PrepVArgs a{v, dtype, B, H, S, D, stride_b, stride_h, stride_s, perm, 1, 1, v8, vs, nullptr, workspace};
  return finish(fn, prep_v_channel(a, static_cast<cudaStream_t>(stream)));
}

int vc_prep_v_channel_static(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                             int64_t stride_b, int64_t stride_h, int64_t stride_s, const int64_t* perm, uint8_t* v8,
                             float* vs, void* stream) {
  const char* fn = "vc_prep_v_channel_static";
  if (int rc = check_common(fn, dtype, B, H, S, D)) return rc;
  if (int rc = check_input(fn, "v", v, dtype, stride_b, stride_h, stride_s)) return rc;
  if (!v8 || !vs || !aligned16(v8) || !aligned16(vs)) {
    set_last_error("%s: v8/vs must be non-null and 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  const int64_t need = B * H * D * 4;   // amax words, zeroed by the launcher before use
  if (need > VC_STATIC_SCRATCH_BYTES) {
    set_last_error("%s: needs %lld bytes of scratch (B*H*D*4) but the static array holds %d (B*H*D <= %d); "
                   "use vc_prep_v_channel with a caller workspace",
                   fn, (long long)need, VC_STATIC_SCRATCH_BYTES, VC_STATIC_SCRATCH_BYTES / 4);
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  void* scratch = static_scratch();
  if (!scratch) return VC_ERR_LAUNCH;
  PrepVArgs a{v, dtype, B, H, S, D, stride_b, stride_h, stride_s, perm, 1, 1, v8, vs, nullptr, scratch};
  return finish(fn, prep_v_channel(a, static_cast<cudaStream_t>(stream)));
}

int64_t vc_prep_v_blocks_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D) {
  return prep_v_blocks_workspace(B, H, S, D);
}

int vc_prep_v_blocks(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                     int64_t stride_h, int64_t stride_s, const int64_t* perm, int channel_scale, int demean, uint8_t* v8,
                     float* vs, uint16_t* means, void* workspace, int64_t workspace_bytes, void* stream) {
  const char* fn = "vc_prep_v_blocks";
  if (int rc = check_common(fn, dtype, B, H, S, D)) return rc;
  if (int rc = check_input(fn, "v", v, dtype, stride_b, stride_h, stride_s)) return rc;
  if (!v8 || !vs || !means || !aligned16(v8) || !aligned16(vs) || !aligned16(means)) {
    set_last_error("%s: v8/vs/means must be non-null and 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  if (channel_scale && (!workspace || workspace_bytes < prep_v_blocks_workspace(B, H, S, D) || !aligned16(workspace))) {
    set_last_error("%s: workspace needs %lld bytes", fn, (long long)prep_v_blocks_workspace(B, H, S, D));
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  PrepVArgs a{v, dtype, B, H, S, D, stride_b, stride_h, stride_s, perm, channel_scale ? 1 : 0, demean ? 1 : 0,
              v8, vs, means, workspace};
  return finish(fn, prep_v_blocks(a, static_cast<cudaStream_t>(stream)));
}

int64_t vc_group_values_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D, int clusters) {
  return group_values_workspace(B, H, S, D, clusters);
}

int vc_group_values(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                    int64_t stride_h, int64_t stride_s, int clusters, int iterations, const float* centers_in,
                    int64_t* perm_out, int32_t* labels_out, float* centers_out, void* workspace,
                    int64_t workspace_bytes, void* stream) {
  const char* fn = "vc_group_values";
  if (int rc = check_common(fn, dtype, B, H, S, D)) return rc;
  if (int rc = check_input(fn, "v", v, dtype, stride_b, stride_h, stride_s)) return rc;
  if (clusters < 1 || clusters > 256 || iterations < 1 || iterations > 100) {
    set_last_error("%s: clusters must be in [1,256] and iterations in [1,100]", fn);
    return VC_ERR_ARG;
  }
  if (!perm_out) {
    set_last_error("%s: perm_out is required", fn);
    return VC_ERR_ARG;
  }
  const int64_t need = group_values_workspace(B, H, S, D, clusters);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_last_error("%s: workspace needs %lld bytes", fn, (long long)need);
    return VC_ERR_WORKSPACE;
  }
  if (int rc = check_device()) return rc;
  GroupArgs a{v, dtype, B, H, S, D, stride_b, stride_h, stride_s, clusters, iterations, centers_in, perm_out,
              labels_out, centers_out, workspace};
  return finish(fn, group_values(a, static_cast<cudaStream_t>(stream)));
}

int vc_attention_fwd(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8,
                     const float* vs, const uint16_t* means, void* out, int out_dtype, int64_t B, int64_t H, int64_t Sq,
                     int64_t Sk, int64_t D, int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s,
                     int expcast, int block_values, int vs_per_block, float sm_scale, int64_t unit_begin,
                     int64_t unit_end, void* stream) {
  const char* fn = "vc_attention_fwd";
  if (int rc = check_common(fn, VC_DTYPE_BF16, B, H, Sq, D)) return rc;
  if (int rc = check_common(fn, VC_DTYPE_BF16, B, H, Sk, D)) return rc;
  if (out_dtype != VC_DTYPE_F16 && out_dtype != VC_DTYPE_BF16 && out_dtype != VC_DTYPE_F32) {
    set_last_error("%s: out_dtype must be F16, BF16 or F32", fn);
    return VC_ERR_ARG;
  }
  if (!q8 || !qs || !k8 || !ks || !v8 || !vs || !out || (block_values && !means) ||
      !aligned16(q8) || !aligned16(k8) || !aligned16(v8) || !aligned16(vs) || !aligned16(ks) ||
      (block_values && !aligned16(means))) {
    set_last_error("%s: payload pointers must be non-null and 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  if (check_input(fn, "out", out, out_dtype, out_stride_b, out_stride_h, out_stride_s)) return VC_ERR_ARG;
  if (vs_per_block && !block_values) {
    set_last_error("%s: per-block V scales require block_values", fn);
    return VC_ERR_ARG;
  }
  if (!(sm_scale > 0.f) || !(sm_scale <= 3.4028234663852886e38f)) {
    set_last_error("%s: sm_scale must be positive and finite", fn);
    return VC_ERR_ARG;
  }
  if (expcast < 0 || expcast > 3) {
    set_last_error("%s: expcast must be 0 (FP8-P control), 1 (ExpCast), 2 (exact ExpCast) or 3 (FP8-P control, "
                   "Config scaling)", fn);
    return VC_ERR_ARG;
  }
  if (int rc = check_device()) return rc;
  AttnArgs a{q8, qs, k8, ks, v8, vs, means, out, out_dtype, B, H, Sq, Sk, D, out_stride_b, out_stride_h, out_stride_s,
             expcast == 3 ? 0 : expcast, block_values ? 1 : 0, vs_per_block ? 1 : 0, sm_scale, unit_begin,
             unit_end, 0, 128, expcast == 3 ? 1 : 0};
  return finish(fn, attention_fwd(a, static_cast<cudaStream_t>(stream)));
}

int vc_attention_fwd_e4m3qk(const uint8_t* q8, const float* qs, const uint8_t* k8, const float* ks,
                            const uint8_t* v8, const float* vs, const uint16_t* means, void* out, int out_dtype,
                            int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int64_t out_stride_b,
                            int64_t out_stride_h, int64_t out_stride_s, int expcast, int block_values,
                            int vs_per_block, int64_t k_quant_block, float sm_scale, int64_t unit_begin,
                            int64_t unit_end, void* stream) {
  const char* fn = "vc_attention_fwd_e4m3qk";
  if (int rc = check_common(fn, VC_DTYPE_BF16, B, H, Sq, D)) return rc;
  if (int rc = check_common(fn, VC_DTYPE_BF16, B, H, Sk, D)) return rc;
  if (out_dtype != VC_DTYPE_F16 && out_dtype != VC_DTYPE_BF16 && out_dtype != VC_DTYPE_F32) {
    set_last_error("%s: out_dtype must be F16, BF16 or F32", fn);
    return VC_ERR_ARG;
  }
  if (!q8 || !qs || !k8 || !ks || !v8 || !vs || !out || (block_values && !means) || !aligned16(q8) ||
      !aligned16(k8) || !aligned16(v8) || !aligned16(vs) || (block_values && !aligned16(means))) {
    set_last_error("%s: payload pointers must be non-null and q8/k8/v8/vs/means 16-byte aligned", fn);
    return VC_ERR_ARG;
  }
  if (check_input(fn, "out", out, out_dtype, out_stride_b, out_stride_h, out_stride_s)) return VC_ERR_ARG;
  if (expcast < 0 || expcast > 3) {
    set_last_error("%s: expcast must be 0 (FP8-P control), 1 (ExpCast), 2 (exact ExpCast) or 3 (FP8-P control, "
                   "Config scaling)", fn);
    return VC_ERR_ARG;
  }
  if (vs_per_block && !block_values) {
    set_last_error("%s: per-block V scales require block_values", fn);
    return VC_ERR_ARG;
  }
  if (k_quant_block < 128 || k_quant_block % 128 || k_quant_block > 4096) {
    set_last_error("%s: k_quant_block must be a multiple of 128 in [128, 4096]", fn);
    return VC_ERR_ARG;
  }
  if (!(sm_scale > 0.f) || !(sm_scale <= 3.4028234663852886e38f)) {
    set_last_error("%s: sm_scale must be positive and finite", fn);
    return VC_ERR_ARG;
  }
  if (int rc = check_device()) return rc;
  AttnArgs a{reinterpret_cast<const int8_t*>(q8), qs, reinterpret_cast<const int8_t*>(k8), ks, v8, vs, means, out,
             out_dtype, B, H, Sq, Sk, D, out_stride_b, out_stride_h, out_stride_s, expcast == 3 ? 0 : expcast,
             block_values ? 1 : 0, vs_per_block ? 1 : 0, sm_scale, unit_begin, unit_end, 1, k_quant_block,
             expcast == 3 ? 1 : 0};
  return finish(fn, attention_fwd(a, static_cast<cudaStream_t>(stream)));
}

int vc_tensor_peak(int kind, int n, int64_t iters, int ctas, int a_tmem, int issuers, unsigned long long* stamps,
                   void* stream) {
  const int64_t stride = (n + 31) / 32 * 32;
  if ((kind != 0 && kind != 1) || n < 16 || n > 256 || n % 16 || issuers < 1 || issuers > 4 || issuers * stride > (a_tmem ? 448 : 512) || iters < 1 || iters > (int64_t(1) << 22) ||
      ctas < 1 || ctas > 4096) {
    set_last_error("vc_tensor_peak: kind 0/1, n a multiple of 16 in [16, 256], 1-4 issuing warps whose accumulators of ceil(n/32)*32 columns fit in 512 (448 with A in tensor memory), iters in [1, 2^22], ctas in [1, 4096]");
    return VC_ERR_ARG;
  }
  if (int rc = check_device()) return rc;
  return finish("vc_tensor_peak", tensor_peak(kind, n, iters, ctas, a_tmem ? 1 : 0, issuers, stamps, static_cast<cudaStream_t>(stream)));
}

int vc_selftest_wait_timeout(int64_t budget_ns, int* ok_out, void* stream) {
  if (budget_ns < 1000 || budget_ns > 2000000000) {
    set_last_error("vc_selftest_wait_timeout: budget_ns must be in [1e3, 2e9]");
    return VC_ERR_ARG;
  }
  if (int rc = check_device()) return rc;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(budget_ns), ok_out);
  return finish("vc_selftest_wait_timeout", cudaGetLastError() == cudaSuccess ? VC_OK : VC_ERR_LAUNCH);
}

int vc_kernel_resources(int head_dim, int64_t* out4) {
  if (!out4 || (head_dim != 64 && head_dim != 128)) {
    set_last_error("vc_kernel_resources: head_dim must be 64 or 128");
    return VC_ERR_ARG;
  }
  return finish("vc_kernel_resources", attention_resources(head_dim, out4));
}

int vc_attention_plan(int64_t qtiles, int64_t unit_begin, int64_t unit_end, int sms, int64_t* out4) {
  if (!out4 || qtiles <= 0 || unit_begin < 0 || unit_end < unit_begin || sms < 0) {
    set_last_error("vc_attention_plan: needs out4, qtiles > 0, 0 <= unit_begin <= unit_end and sms >= 0");
    return VC_ERR_ARG;
  }
  const AttnPlan r = attention_plan(qtiles, unit_begin, unit_end, sms);
  out4[0] = r.pairs;
  out4[1] = r.tail_units;
  out4[2] = r.tail_begin;
  out4[3] = r.launches;
  return VC_OK;
}

}  // extern "C"
