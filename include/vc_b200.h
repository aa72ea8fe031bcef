/*
 * vc_b200.h -- C ABI of the B200 (sm_100a) VC-attention library.
 *
 * Plain pointers and sizes only.  Every entry point:
 *   - takes device pointers for tensors, int64 shapes/strides (in elements),
 *     and a cudaStream_t passed as ``void*`` (NULL = legacy default stream);
 *   - enqueues work on that stream and returns; it never synchronises and
 *     never allocates (scratch is caller-provided; size it with the matching
 *     ``*_workspace_bytes`` query);
 *   - returns VC_OK or a VC_ERR_* status; argument errors are detected on the
 *     host before anything is launched.
 * Device-side waits are bounded: a kernel that exceeds its wait budget sets a
 * bit in a per-device error word (read with vc_error_read) and returns.
 *
 * Layouts (row-major, last index fastest):
 *   q, k, v     input [B, H, S, D] addressed through (stride_b, stride_h,
 *               stride_s) with unit channel stride; dtype VC_DTYPE_*
 *   q8, k8      int8  [B, H, S, D] contiguous
 *   qs          fp32  [B, H, ceil(Sq/64)*32]  (Sage per-thread Q scales)
 *   ks          fp32  [B, H, ceil(Sk/128)*4]  (Sage per-thread K scales)
 *   v8          E4M3  [B, H, D, ceil(Sk/128)*128] (V transposed, token order)
 *   vs          fp32  [B, H, D] (channel) or [B, H, ceil(Sk/128), D] (block)
 *   means       fp16  [B, H, ceil(Sk/128), D] (V smoothing only)
 *   perm        int64 [B, H, Sk] token permutation (V grouping), or NULL
 */
#ifndef VC_B200_H
#define VC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VC_B200_API_VERSION 1

enum vc_status {
  VC_OK = 0,
  VC_ERR_ARG = 1,          /* bad shape / dtype / pointer / alignment */
  VC_ERR_LAUNCH = 2,       /* CUDA launch or runtime error */
  VC_ERR_UNSUPPORTED = 3,  /* device is not sm_100, or feature unsupported */
  VC_ERR_WORKSPACE = 4     /* workspace missing or too small */
};

enum vc_dtype { VC_DTYPE_F16 = 0, VC_DTYPE_BF16 = 1, VC_DTYPE_F32 = 2 };

/* Library identity. */
int vc_api_version(void);
const char* vc_build_info(void);
/* Human-readable description of the last error on this host thread. */
const char* vc_last_error(void);

/* Device error word (timeouts / invariant violations inside kernels).
 * Synchronous diagnostic call: copies the word of ``device`` into *code and
 * optionally clears it.  Bits: 0x01-0x10 a bounded wait gave up (TMA, MMA,
 * softmax, correction, producer), 0x20 tensor-memory allocation, 0x40 a bad
 * kernel argument, 0x80 a permutation entry outside [0, S) (that row was read
 * as zeros), 0x100 the wait of vc_selftest_wait_timeout gave up (as intended).
 * Replaces: no reference counterpart (the reference spins without bound,
 * third_party/sageattention_local/csrc/vc/vc_sm90.cu:114-128). */
int vc_error_read(int device, uint32_t* code, int clear);

/* ExpCast byte of each FP32 input: uint8(clamp(RNE(fma(x, 8 log2 e, 119.65)), 0, 120)).
 * Replaces _vc_sm90.expcast_codes (third_party/sageattention_local/csrc/vc/
 * preprocess.cu:170-179, pybind.cpp:63). */
int vc_expcast_codes(const float* x, uint8_t* y, int64_t n, void* stream);

/* INT8 Q/K quantisation with K channel-mean smoothing.
 *   km = mean of K over tokens (input dtype) unless ``km_in`` is given;
 *   K' = (K - km) rounded to the input dtype; Q, K' -> Sage per-thread INT8.
 * ``perm`` (nullable) gathers K rows: K'[s] = K[perm[s]].  ``km_out``
 * (nullable) receives km [B,H,D] in the input dtype.  ``mean_numel_out`` /
 * ``mean_numel_in`` reproduce torch's CUDA mean factor
 * float(mean_numel_out)/float(mean_numel_in); pass 0,0 for 1/Sk.
 * Replaces vc.py:158-159 (k.mean + per_thread_int8) -> triton
 * quant_per_thread.py:22-98,154-203. */
int64_t vc_prep_qk_workspace_bytes(int64_t B, int64_t H, int64_t Sk, int64_t D);
int vc_prep_qk_int8(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                    int64_t D, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s, int64_t k_stride_b,
                    int64_t k_stride_h, int64_t k_stride_s, const int64_t* perm, const void* km_in, void* km_out,
                    int64_t mean_numel_out, int64_t mean_numel_in, int8_t* q8, float* qs, int8_t* k8, float* ks,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Q/K for the Config contract's own QK path (qk_hadamard=True): K centred by
 * its FP32 channel mean over all tokens when k_smooth (km_in [B*H][D] FP32 if
 * given, else computed; written to km_out when non-null), Q and K rotated by
 * the normalised Sylvester transform on channels, then E4M3 block payloads:
 * q8 [B,H,Sq,D] with qs [B,H,ceil(Sq/128)] (q_block 128) and k8 [B,H,Sk,D]
 * (rows in permutation order when perm is given) with ks
 * [B,H,ceil(Sk/k_quant_block)]; scale = amax/448 (1 for an all-zero block),
 * payload = e4m3_rn_satfinite(x / scale).  k_quant_block must be a positive
 * multiple of 128 (at most 4096).
 * Replaces core.py:79-107 (hadamard, preprocess_qk) and :128-150 (_encode,
 * _quantize_qk) of src/vc_attention, the cuda_fp8 backend's Q/K preparation
 * (csrc/kernels.cu:104-152). */
int64_t vc_prep_qk_hadamard_workspace_bytes(int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                            int64_t k_quant_block);
int vc_prep_qk_hadamard_e4m3(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                             int64_t D, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
                             int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s, const int64_t* perm,
                             int k_smooth, const float* km_in, float* km_out, int64_t k_quant_block, uint8_t* q8,
                             float* qs, uint8_t* k8, float* ks, void* workspace, int64_t workspace_bytes,
                             void* stream);

/* Unsmoothed V: per-channel E4M3 (scale = amax/448, payload = e4m3(x*448/amax);
 * all-zero channels get scale 0 and payload 0).
 * Replaces vc.py:162-166 -> quant.py:223-292 per_channel_fp8(smooth_v=False)
 * -> csrc/fused/fused.cu:317-427 (MeanScaleKernel) and its zero-safe twin
 * csrc/vc/global_values.cuh:45-157. */
int64_t vc_prep_v_channel_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D);
int vc_prep_v_channel(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                      int64_t stride_h, int64_t stride_s, const int64_t* perm, uint8_t* v8, float* vs,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* vc_prep_v_channel without a caller workspace, for callers that cannot
 * allocate device memory.  It has no counterpart in the reference.
 * Same arguments, results and errors as vc_prep_v_channel; its scratch (the
 * per-channel amax words, B*H*D*4 bytes) lives in a library-owned static
 * device array of VC_STATIC_SCRATCH_BYTES (1 MiB), so B*H*D must not exceed
 * 262144 (e.g. B*H <= 2048 at D = 128); larger sizes return VC_ERR_WORKSPACE
 * and launch nothing.  It allocates nothing: no cudaMalloc, no cudaFree.
 *   - The first call on each device (that device current) resolves the
 *     array's device address once (cudaGetSymbolAddress) and keeps it for the
 *     life of the process; make that first call before any stream capture on
 *     that device.  Resetting the device (cudaDeviceReset) or switching the
 *     device's context after the first call is not supported: the kept
 *     address would no longer be valid.
 *   - Every call on a device shares the one array.  Each call zeroes the
 *     words it uses on ``stream`` before its kernels read them, so calls in
 *     stream order are independent; calls that overlap on the GPU (other
 *     streams, other host threads without ordering) race on the array and
 *     must be serialised by the caller. */
#define VC_STATIC_SCRATCH_BYTES (1 << 20)
int vc_prep_v_channel_static(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                             int64_t stride_b, int64_t stride_h, int64_t stride_s, const int64_t* perm, uint8_t* v8,
                             float* vs, void* stream);

/* Smoothed V: 128-token block de-meaning, E4M3 residual, FP16 mean/scale.
 * channel_scale=1: vs [B,H,D]; 0: vs [B,H,T,D] (per block).  demean=0 keeps
 * the block mean at zero (per-block amax scaling only, the Config-API
 * contract when smoothing is inactive, src/vc_attention/core.py:110-123).
 * Replaces _vc_sm90.prepare_values (csrc/vc/preprocess.cu:25-56, 68-168). */
int64_t vc_prep_v_blocks_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D);
int vc_prep_v_blocks(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                     int64_t stride_h, int64_t stride_s, const int64_t* perm, int channel_scale, int demean,
                     uint8_t* v8, float* vs, uint16_t* means, void* workspace, int64_t workspace_bytes,
                     void* stream);

/* V grouping: Lloyd clustering (linspace init, ``iterations`` assignments,
 * empty clusters keep their centre) and a stable sort of the final labels.
 * clusters in [1,256], iterations in [1,100].  ``centers_in`` (nullable,
 * fp32 [B,H,min(clusters,S),D]) replaces the linspace initialisation (warm
 * start across denoising steps, src/vc_attention/core.py:197-226).
 * perm_out int64 [B,H,S];
 * labels_out int32 [B,H,S] and centers_out fp32 [B,H,min(clusters,S),D]
 * (centres used by the final assignment) are optional.
 * Replaces _vc_sm90.group_values / group_values_debug
 * (csrc/vc/clustering.cu:22-166, pybind.cpp:38-44). */
int64_t vc_group_values_workspace_bytes(int64_t B, int64_t H, int64_t S, int64_t D, int clusters);
int vc_group_values(const void* v, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t stride_b,
                    int64_t stride_h, int64_t stride_s, int clusters, int iterations, const float* centers_in,
                    int64_t* perm_out, int32_t* labels_out, float* centers_out, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* Fused attention on prepared payloads (tcgen05 kind::i8 QK^T into tensor
 * memory, ExpCast P, kind::f8f6f4 PV, FP32 online accumulation, optional
 * block-mean restoration).  out [B,H,Sq,D] (out_dtype F16, BF16 or F32) through
 * (out_stride_b, out_stride_h, out_stride_s).  Work units are
 * (b*H + h) * ceil(Sq/128) + q_tile; [unit_begin, unit_end) selects a shard
 * (pass 0, -1 for all).  vs_per_block: vs is [B,H,T,D].  expcast: 0 = Sage
 * FP8 probabilities (control: P = e4m3(exp2(logit - max + 8.807)), exact
 * exp2 row sums, vc_reference.py:56-64), 1 = ExpCast with the reference's
 * folded affine encoder (csrc/vc/vc_math.cuh:17-106, exact fallback on
 * extreme ranges), 2 = ExpCast with the unfused decoded-payload contract
 * (vc_reference.py:52-54), 3 = the FP8-P control with the Config contract's
 * scaling (P8 = e4m3(256 exp(s - max)), exact exp row sums;
 * src/vc_attention/core.py:357-360).
 * Replaces _vc_sm90.forward (csrc/vc/vc_sm90.cu:1027-1123, vc_api.h:8-10). */
int vc_attention_fwd(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks, const uint8_t* v8,
                     const float* vs, const uint16_t* means, void* out, int out_dtype, int64_t B, int64_t H,
                     int64_t Sq, int64_t Sk, int64_t D, int64_t out_stride_b, int64_t out_stride_h,
                     int64_t out_stride_s, int expcast, int block_values, int vs_per_block, float sm_scale,
                     int64_t unit_begin, int64_t unit_end, void* stream);

/* vc_attention_fwd with E4M3 block Q/K payloads (vc_prep_qk_hadamard_e4m3):
 * QK^T is a tcgen05 kind::f8f6f4 MMA into FP32 and the logits are
 * raw * (sm_scale * (qs[q_tile] * ks[key / k_quant_block])).  expcast
 * 0-3, block_values and vs_per_block as vc_attention_fwd: ExpCast with
 * per-channel V scales runs the tensor-memory-accumulating kernel; the FP8-P
 * control and per-block V scales (the Config contract's own formats,
 * core.py:110-123) run the register-accumulating kernel, since a per-tile,
 * per-channel V scale cannot be applied inside a tensor-memory accumulation.
 * Replaces the cuda_fp8 backend's fused attention on its E4M3 block Q/K
 * (src/vc_attention/cuda_backend.py:37-88, core.py:335-345 semantics). */
int vc_attention_fwd_e4m3qk(const uint8_t* q8, const float* qs, const uint8_t* k8, const float* ks,
                            const uint8_t* v8, const float* vs, const uint16_t* means, void* out, int out_dtype,
                            int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int64_t out_stride_b,
                            int64_t out_stride_h, int64_t out_stride_s, int expcast, int block_values,
                            int vs_per_block, int64_t k_quant_block, float sm_scale, int64_t unit_begin,
                            int64_t unit_end, void* stream);

/* Failure-detection self-test (no counterpart in the reference, whose
 * kernels wait without bound, csrc/vc/vc_sm90.cu:114-128): one warp waits,
 * through the same bounded mbarrier wait every kernel here uses, for a
 * phase that nothing completes.  After ``budget_ns`` (1e3..2e9) it gives up,
 * sets bit 0x100 in the device error word (vc_error_read) and
 * returns; the context stays usable.  ``ok_out`` (optional, device int)
 * receives 0 (gave up) or 1. */
int vc_selftest_wait_timeout(int64_t budget_ns, int* ok_out, void* stream);

/* Compiled resources of the fused kernel (registers/thread, static+dynamic
 * shared bytes, threads) for head_dim 64/128 into out[0..3].
 * Replaces _vc_sm90.kernel_resources (csrc/vc/vc_sm90.cu:788-822). */
int vc_kernel_resources(int head_dim, int64_t* out4);

/* How vc_attention_fwd spreads the units [unit_begin, unit_end) over its
 * kernels for ExpCast with channel V scales (host arithmetic only, no device
 * work): out[0] = paired-tile CTAs (two consecutive 128-row Q tiles of one
 * head each), out[1] = units that run on the alternating-tile kernel after
 * them, out[2] = the first of those units, out[3] = attention launches.  The
 * tail exists when the last wave of pairs is at most half full on ``sms``
 * streaming multiprocessors (the device's count; 0 = pairs only).
 * No counterpart in the reference (launch accounting for this library). */
int vc_attention_plan(int64_t qtiles, int64_t unit_begin, int64_t unit_end, int sms, int64_t* out4);

/* Tensor-core throughput probe, the measured denominator of the attention
 * kernel's roofline (a measurement aid; the reference quotes a nominal peak
 * instead, scripts/profile_int8_h200.py).  Launches ``ctas`` CTAs (one per
 * SM) that each issue iters x 4 MMAs of M=128, N=n, K=32 from shared-memory
 * operands: kind 0 = tcgen05 kind::i8 (s32 accumulate), kind 1 = kind::f8f6f4
 * with E4M3 operands (f32 accumulate); ``a_tmem`` != 0 reads A from tensor
 * memory instead of shared memory; ``issuers`` warps (1-4) issue at once,
 * each into its own accumulator (issuers * ceil(n/32)*32 columns must fit in
 * 512, or in 448 with A in tensor memory).  ``stamps`` (optional, device, 3 per
 * CTA) receives the issue and completion cycles and an ok flag.  The caller
 * times the launch (ops = 2*128*n*32*4*iters*issuers*ctas).  n in [16,256] step 16,
 * iters in [1, 2^22]. */
int vc_tensor_peak(int kind, int n, int64_t iters, int ctas, int a_tmem, int issuers, unsigned long long* stamps,
                   void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VC_B200_H */
