// Internal launcher interfaces between the C ABI (capi.cu) and the kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "vc_b200.h"

namespace vcb {

struct PrepQKArgs {
  const void* q;
  const void* k;
  int dtype;
  int64_t B, H, Sq, Sk, D;
  int64_t qsb, qsh, qss, ksb, ksh, kss;
  const int64_t* perm;
  const void* km_in;
  void* km_out;
  int64_t mean_numel_out, mean_numel_in;
  int8_t* q8;
  float* qs;
  int8_t* k8;
  float* ks;
  void* workspace;
};
int64_t prep_qk_workspace(int64_t B, int64_t H, int64_t Sk, int64_t D);
int prep_qk(const PrepQKArgs& a, cudaStream_t st);

struct PrepHadArgs {
  const void* q;
  const void* k;
  int dtype;
  int64_t B, H, Sq, Sk, D;
  int64_t qsb, qsh, qss, ksb, ksh, kss;
  const int64_t* perm;
  int k_smooth;
  const float* km_in;   // [B*H][D] FP32 or null (computed)
  float* km_out;        // optional
  int64_t kqb;          // K rows per scale block (a multiple of 128)
  uint8_t* q8;
  float* qs;
  uint8_t* k8;
  float* ks;
  void* workspace;
};
int64_t prep_hadamard_workspace(int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D, int64_t kqb);
int prep_hadamard(const PrepHadArgs& a, cudaStream_t st);
cudaError_t prep_hadamard_error_word(uint32_t* code, bool clear);

struct PrepVArgs {
  const void* v;
  int dtype;
  int64_t B, H, S, D;
  int64_t sb, sh, ss;
  const int64_t* perm;
  int channel_scale;  // blocks mode only
  int demean;         // blocks mode only
  uint8_t* v8;
  float* vs;
  uint16_t* means;    // blocks mode only
  void* workspace;
};
int64_t prep_v_channel_workspace(int64_t B, int64_t H, int64_t S, int64_t D);
int prep_v_channel(const PrepVArgs& a, cudaStream_t st);
int64_t prep_v_blocks_workspace(int64_t B, int64_t H, int64_t S, int64_t D);
int prep_v_blocks(const PrepVArgs& a, cudaStream_t st);

struct GroupArgs {
  const void* v;
  int dtype;
  int64_t B, H, S, D;
  int64_t sb, sh, ss;
  int clusters, iterations;
  const float* centers_in;
  int64_t* perm_out;
  int32_t* labels_out;
  float* centers_out;
  void* workspace;
};
int64_t group_values_workspace(int64_t B, int64_t H, int64_t S, int64_t D, int clusters);
int group_values(const GroupArgs& a, cudaStream_t st);

struct AttnArgs {
  const int8_t* q8;
  const float* qs;
  const int8_t* k8;
  const float* ks;
  const uint8_t* v8;
  const float* vs;
  const uint16_t* means;
  void* out;
  int out_dtype;
  int64_t B, H, Sq, Sk, D;
  int64_t osb, osh, oss;
  int expcast, block_values, vs_per_block;
  float sm_scale;
  int64_t unit_begin, unit_end;
  int qk_e4m3;        // 1: E4M3 block Q/K payloads (qs per 128-row Q tile, ks per kqb K rows)
  int64_t kqb;
  int config_control; // FP8-P control with the Config contract's scaling (offset 8) instead of Sage's (8.807)
};
int attention_fwd(const AttnArgs& a, cudaStream_t st);
// How attention_fwd spreads units [ub, ue) over its ExpCast kernels (channel
// V scales): paired-tile CTAs, then tail units on the alternating-tile kernel.
struct AttnPlan {
  int64_t pairs = 0, tail_units = 0, tail_begin = 0, launches = 0;
};
AttnPlan attention_plan(int64_t qtiles, int64_t ub, int64_t ue, int64_t sms);
// Copy (and optionally clear) the device error word of each kernel file on the
// current device.  Synchronous.
cudaError_t attention_error_word(uint32_t* code, bool clear);
cudaError_t prep_qk_error_word(uint32_t* code, bool clear);
cudaError_t prep_v_error_word(uint32_t* code, bool clear);
int attention_resources(int head_dim, int64_t* out4);

int expcast_codes(const float* x, uint8_t* y, int64_t n, cudaStream_t st);

// Tensor-core throughput measurement (tensor_peak.cu): ``ctas`` CTAs, each
// issuing ``iters`` x 4 MMAs of M=128 x n x K=32 (kind 0: kind::i8, 1: E4M3
// kind::f8f6f4); ``stamps`` (optional, device, 3 per CTA): issue cycles,
// completion cycles, ok flag.  ``a_tmem``: A read from tensor memory; ``issuers`` warps issue concurrently.
int tensor_peak(int kind, int n, int64_t iters, int ctas, int a_tmem, int issuers, unsigned long long* stamps,
                cudaStream_t st);
cudaError_t tensor_peak_error_word(uint32_t* code, bool clear);

// Host-side error text for the calling thread.
void set_last_error(const char* fmt, ...);

}  // namespace vcb
