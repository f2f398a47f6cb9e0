// Shared device helpers for the tree-training sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tree_training_b200.h"

#define TT_CUDA_OK(expr)                         \
  do {                                           \
    cudaError_t _e = (expr);                     \
    if (_e != cudaSuccess) return TT_ERR_CUDA;   \
  } while (0)

namespace tt {

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Key-visibility test shared by every attention kernel: key j with row
// interval [lo, hi) is visible to row i iff lo <= i < hi.
__device__ __forceinline__ bool visible(int32_t lo, int32_t hi, int32_t row) {
  return (row >= lo) & (row < hi);
}

// Row stride of the per-(head, row) fp32 terms (LSE, delta): rows padded to a
// multiple of 128 so tensor-core kernels read whole tiles with vector loads.
// Padding rows hold LSE = +inf (no probability mass) and delta = 0.
__host__ __device__ __forceinline__ int lse_ld(int n_q) { return (n_q + 127) & ~127; }

// Record the first error code a kernel hits (never traps).
__device__ __forceinline__ void set_status(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace tt

// Count of kernels launched by the library (tt_kernel_launches).
void tt_count_launches(int n);

// Launchers implemented in the .cu files (host side, called from tt_api.cu).
int tt_launch_attn_fwd_simt(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                            int32_t D, const void* q, int64_t q_st, int64_t q_sh, const void* k,
                            int64_t k_st, int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                            const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                            const int32_t* fwd_list, float scale, void* out, float* lse,
                            cudaStream_t stream);
int tt_launch_attn_bwd_simt(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                            int32_t D, const void* q, int64_t q_st, int64_t q_sh, const void* k,
                            int64_t k_st, int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                            const void* out, const void* dout, int64_t do_st, int64_t do_sh,
                            const float* lse, const int32_t* kv_lo, const int32_t* kv_hi,
                            const int32_t* fwd_ptr, const int32_t* fwd_list,
                            const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
                            void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st,
                            int64_t dk_sh, void* dv, int64_t dv_st, int64_t dv_sh, float* delta,
                            int phases, cudaStream_t stream);
int tt_launch_mask_to_intervals(int mask_dtype, int32_t n_q, int32_t n_kv, const void* mask,
                                int64_t stride_q, int64_t stride_kv, int32_t* kv_lo,
                                int32_t* kv_hi, int32_t* status, cudaStream_t stream);
// tcgen05 path (bf16/f16, head_dim 128).  Returns TT_ERR_UNSUPPORTED when the
// shape/stride/alignment is not covered so the caller can use the SIMT path.
int tt_launch_attn_fwd_sm100(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                             int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, const int32_t* kv_lo,
                             const int32_t* kv_hi, const int32_t* fwd_ptr,
                             const int32_t* fwd_list, float scale, void* out, float* lse,
                             int32_t* status, cudaStream_t stream);
int tt_launch_attn_bwd_sm100(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                             int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, const void* out, const void* dout,
                             int64_t do_st, int64_t do_sh, const float* lse,
                             const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                             const int32_t* fwd_list, const int32_t* bwd_ptr,
                             const int32_t* bwd_list, float scale, void* dq, int64_t dq_st,
                             int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
                             int64_t dv_st, int64_t dv_sh, float* delta, int32_t* kt_order,
                             int phases, int32_t* status, cudaStream_t stream);
int tt_launch_attn_bwd_sm100_stored(
    int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv, int32_t D, const void* q,
    int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh, const void* v,
    int64_t v_st, int64_t v_sh, const void* out, const void* dout, int64_t do_st, int64_t do_sh,
    const float* lse, const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
    const int32_t* fwd_list, const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
    void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
    int64_t dv_st, int64_t dv_sh, float* delta, int32_t* kt_order, int32_t* e2f, void* ds_ws,
    int64_t n_pairs, int32_t kv_heads_per_pass, int phases, int32_t* status,
    cudaStream_t stream);

// Bytes of the fp32 row terms (delta) at the start of the backward workspace.
inline int64_t tt_attn_bwd_delta_bytes(int32_t n_q, int32_t hq) {
  const int64_t bytes = (int64_t)hq * tt::lse_ld(n_q) * 4;
  return (bytes + 255) / 256 * 256;
}
