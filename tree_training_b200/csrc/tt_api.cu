// C-ABI entry points for the device-side operations: argument checks, tile
// shape policy, path selection (tcgen05 for bf16/f16 head_dim 128, exact SIMT
// otherwise), workspace accounting.
#include <atomic>
#include <cstdlib>

#include "tt_common.cuh"

namespace {

// 0 = automatic, 1 = force the exact SIMT kernels (cross-checks and fp32).
int g_kernel_path = -1;

int kernel_path() {
  if (g_kernel_path < 0) {
    const char* e = std::getenv("TT_KERNEL_PATH");
    g_kernel_path = (e && e[0] == '1') ? 1 : 0;
  }
  return g_kernel_path;
}

bool tc_path(int dtype, int D) {
  return kernel_path() == 0 && (dtype == TT_BF16 || dtype == TT_F16) && D == 128;
}

bool valid_dims(int n_q, int n_kv, int hq, int hkv, int D) {
  return n_q >= 0 && n_kv >= 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && D > 0;
}

std::atomic<int64_t> g_launches{0};

}  // namespace

void tt_count_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

extern "C" int64_t tt_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int tt_set_kernel_path(int path) {
  const int prev = kernel_path();
  g_kernel_path = path == 1 ? 1 : 0;
  return prev;
}

extern "C" int tt_attn_tile_shape(int dtype, int32_t D, int kind, int32_t* tile_q,
                                  int32_t* tile_kv) {
  if (!tile_q || !tile_kv || (kind != 0 && kind != 1)) return TT_ERR_INVALID_ARG;
  if (tc_path(dtype, D)) {
    *tile_q = 128;
    *tile_kv = 128;
  } else {
    *tile_q = 64;
    *tile_kv = 64;
  }
  return TT_OK;
}

extern "C" int tt_mask_to_intervals(int mask_dtype, int32_t n_q, int32_t n_kv, const void* mask,
                                    int64_t stride_q, int64_t stride_kv, int32_t* kv_lo,
                                    int32_t* kv_hi, int32_t* status, void* stream) {
  if (n_q < 0 || n_kv < 0 || (n_kv > 0 && (!mask || !kv_lo || !kv_hi))) return TT_ERR_INVALID_ARG;
  return tt_launch_mask_to_intervals(mask_dtype, n_q, n_kv, mask, stride_q, stride_kv, kv_lo,
                                     kv_hi, status, (cudaStream_t)stream);
}

extern "C" int tt_tree_attn_fwd(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                                int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                                const void* k, int64_t k_st, int64_t k_sh, const void* v,
                                int64_t v_st, int64_t v_sh, const int32_t* kv_lo,
                                const int32_t* kv_hi, const int32_t* fwd_ptr,
                                const int32_t* fwd_list, float scale, void* out, float* lse,
                                int32_t* status, void* stream) {
  if (!valid_dims(n_q, n_kv, hq, hkv, D)) return TT_ERR_INVALID_ARG;
  if (n_q == 0) return TT_OK;
  if (!q || !k || !v || !out || !lse || !fwd_ptr || (n_kv > 0 && (!kv_lo || !kv_hi)))
    return TT_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (tc_path(dtype, D)) {
    const int rc = tt_launch_attn_fwd_sm100(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st,
                                            k_sh, v, v_st, v_sh, kv_lo, kv_hi, fwd_ptr, fwd_list,
                                            scale, out, lse, status, st);
    return rc;
  }
  return tt_launch_attn_fwd_simt(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v,
                                 v_st, v_sh, kv_lo, kv_hi, fwd_ptr, fwd_list, scale, out, lse, st);
}

extern "C" int64_t tt_tree_attn_bwd_workspace_size(int dtype, int32_t n_q, int32_t n_kv,
                                                   int32_t hq, int32_t hkv, int32_t D) {
  (void)dtype;
  (void)hkv;
  (void)D;
  // fp32 delta = rowsum(dO * O) per (head, row), rows padded like the LSE;
  // then the dK/dV tile order (one int32 per 128-key tile)
  const int64_t order = ((int64_t)(n_kv + 127) / 128 * 4 + 255) / 256 * 256;
  return tt_attn_bwd_delta_bytes(n_q, hq) + order;
}

extern "C" int tt_tree_attn_bwd(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                                int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                                const void* k, int64_t k_st, int64_t k_sh, const void* v,
                                int64_t v_st, int64_t v_sh, const void* out, const void* dout,
                                int64_t do_st, int64_t do_sh, const float* lse,
                                const int32_t* kv_lo, const int32_t* kv_hi,
                                const int32_t* fwd_ptr, const int32_t* fwd_list,
                                const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
                                void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st,
                                int64_t dk_sh, void* dv, int64_t dv_st, int64_t dv_sh,
                                void* workspace, int64_t workspace_bytes, int phases,
                                int32_t* status, void* stream) {
  if (!valid_dims(n_q, n_kv, hq, hkv, D)) return TT_ERR_INVALID_ARG;
  // the row terms are required; the tile-order part is used when present
  const int64_t delta_bytes = tt_attn_bwd_delta_bytes(n_q, hq);
  if (workspace_bytes < delta_bytes) return TT_ERR_WORKSPACE;
  int32_t* kt_order =
      workspace_bytes >= tt_tree_attn_bwd_workspace_size(dtype, n_q, n_kv, hq, hkv, D)
          ? reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + delta_bytes)
          : nullptr;
  if ((n_q > 0 && (!q || !out || !dout || !lse || !dq || !fwd_ptr)) ||
      (n_kv > 0 && (!k || !v || !dk || !dv || !kv_lo || !kv_hi || !bwd_ptr)))
    return TT_ERR_INVALID_ARG;
  if (tc_path(dtype, D))
    return tt_launch_attn_bwd_sm100(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v,
                                    v_st, v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi,
                                    fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh,
                                    dk, dk_st, dk_sh, dv, dv_st, dv_sh, (float*)workspace, kt_order,
                                    phases, status, (cudaStream_t)stream);
  return tt_launch_attn_bwd_simt(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v,
                                 v_st, v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi, fwd_ptr,
                                 fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh, dk, dk_st,
                                 dk_sh, dv, dv_st, dv_sh, (float*)workspace, phases,
                                 (cudaStream_t)stream);
}

namespace {
int64_t round256(int64_t b) { return (b + 255) / 256 * 256; }
constexpr int64_t kDsSlotBytes = 32768;   // one 16-bit 128 x 128 dS tile
}  // namespace

extern "C" int64_t tt_tree_attn_bwd_stored_workspace_size(int dtype, int32_t n_q, int32_t n_kv,
                                                          int32_t hq, int32_t hkv, int32_t D,
                                                          int64_t n_tile_pairs,
                                                          int32_t kv_heads_per_pass) {
  const int64_t regular = tt_tree_attn_bwd_workspace_size(dtype, n_q, n_kv, hq, hkv, D);
  if (!valid_dims(n_q, n_kv, hq, hkv, D) || !tc_path(dtype, D) || n_q == 0 || n_kv == 0)
    return regular;
  if (n_tile_pairs < 1 || kv_heads_per_pass < 1 || kv_heads_per_pass > hkv) return -1;
  return regular + round256(n_tile_pairs * 4) +
         static_cast<int64_t>(hq / hkv) * kv_heads_per_pass * n_tile_pairs * kDsSlotBytes;
}

extern "C" int tt_tree_attn_bwd_stored(
    int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv, int32_t D, const void* q,
    int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh, const void* v,
    int64_t v_st, int64_t v_sh, const void* out, const void* dout, int64_t do_st, int64_t do_sh,
    const float* lse, const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
    const int32_t* fwd_list, const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
    void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
    int64_t dv_st, int64_t dv_sh, int64_t n_tile_pairs, int32_t kv_heads_per_pass,
    void* workspace, int64_t workspace_bytes, int phases, int32_t* status, void* stream) {
  if (!valid_dims(n_q, n_kv, hq, hkv, D)) return TT_ERR_INVALID_ARG;
  if (!tc_path(dtype, D) || n_q == 0 || n_kv == 0)
    return tt_tree_attn_bwd(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v, v_st,
                            v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi, fwd_ptr, fwd_list,
                            bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh, dk, dk_st, dk_sh, dv,
                            dv_st, dv_sh, workspace, workspace_bytes, phases, status, stream);
  if (n_tile_pairs < 1 || kv_heads_per_pass < 1 || kv_heads_per_pass > hkv)
    return TT_ERR_INVALID_ARG;
  const int64_t need = tt_tree_attn_bwd_stored_workspace_size(dtype, n_q, n_kv, hq, hkv, D,
                                                              n_tile_pairs, kv_heads_per_pass);
  if (need < 0) return TT_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < need) return TT_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) || !q || !out || !dout || !lse || !dq ||
      !fwd_ptr || !fwd_list || !k || !v || !dk || !dv || !kv_lo || !kv_hi || !bwd_ptr ||
      !bwd_list)
    return TT_ERR_INVALID_ARG;
  char* ws = static_cast<char*>(workspace);
  const int64_t delta_bytes = tt_attn_bwd_delta_bytes(n_q, hq);
  const int64_t regular = tt_tree_attn_bwd_workspace_size(dtype, n_q, n_kv, hq, hkv, D);
  int32_t* kt_order = reinterpret_cast<int32_t*>(ws + delta_bytes);
  int32_t* e2f = reinterpret_cast<int32_t*>(ws + regular);
  void* ds = ws + regular + round256(n_tile_pairs * 4);
  return tt_launch_attn_bwd_sm100_stored(
      dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v, v_st, v_sh, out, dout, do_st,
      do_sh, lse, kv_lo, kv_hi, fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh, dk,
      dk_st, dk_sh, dv, dv_st, dv_sh, reinterpret_cast<float*>(ws), kt_order, e2f, ds,
      n_tile_pairs, kv_heads_per_pass, phases, status, static_cast<cudaStream_t>(stream));
}

