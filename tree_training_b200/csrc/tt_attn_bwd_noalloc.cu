// Tree attention backward for callers that cannot allocate device memory.
//
// Some callers of this library cannot hand it a scratch buffer and must not let
// it call cudaMalloc: a binding whose signature mirrors the reference's
// attention call (inputs and outputs only, no workspace argument), or a host
// runtime whose device memory is owned by its own pooling allocator, where a
// hidden cudaMalloc would bypass its accounting and can synchronise the device.
// tt_tree_attn_bwd_noalloc serves them: it runs tt_tree_attn_bwd with a full
// workspace (the fp32 row terms and the dK/dV tile order) carved out of a fixed
// array that is part of the library's device image, so the kernels, their
// schedule and their results are those of tt_tree_attn_bwd given a workspace
// of tt_tree_attn_bwd_workspace_size bytes.
//
// The array is a file-scope __device__ object, so every GPU that loads the
// library holds it (8 MiB + 64 KiB) until the process exits.  Host code cannot
// use the array's name as a device address; the first call on each device
// (with that device current) looks the address up with cudaGetSymbolAddress
// and caches it, so make that first call before any stream capture.  The cache
// is per device for the life of the process: after a cudaDeviceReset the
// library must not be called again in that process.  All calls share the
// array: two calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on it.  Nothing in it needs clearing: the
// backward's first kernels write every entry that the later kernels read.
#include <mutex>

#include "tt_common.cuh"

namespace {

// fp32 row terms: hq * round_up(n_q, 128) entries at most (8 MiB) ...
constexpr int64_t kNoAllocMaxRowTerms = int64_t(1) << 21;
// ... followed by one int32 per 128-key tile, n_kv <= 16384 * 128 keys (64 KiB)
constexpr int64_t kNoAllocMaxKvTiles = int64_t(1) << 14;
constexpr int64_t kNoAllocBytes = kNoAllocMaxRowTerms * 4 + kNoAllocMaxKvTiles * 4;

static __device__ __align__(256) unsigned char g_bwd_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_bwd_scratch on the current device (looked up once).
int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bwd_scratch) != cudaSuccess || p == nullptr)
      return TT_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TT_OK;
}

}  // namespace

extern "C" int64_t tt_tree_attn_bwd_noalloc_max_row_terms(void) { return kNoAllocMaxRowTerms; }

extern "C" int tt_tree_attn_bwd_noalloc(
    int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv, int32_t D, const void* q,
    int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh, const void* v,
    int64_t v_st, int64_t v_sh, const void* out, const void* dout, int64_t do_st, int64_t do_sh,
    const float* lse, const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
    const int32_t* fwd_list, const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
    void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
    int64_t dv_st, int64_t dv_sh, int32_t* status, void* stream) {
  // size limits first, in 64-bit arithmetic: nothing is touched for a problem
  // that does not fit
  if (n_q < 0 || n_kv < 0 || hq <= 0) return TT_ERR_INVALID_ARG;
  const int64_t row_terms = (static_cast<int64_t>(n_q) + 127) / 128 * 128 * hq;
  const int64_t kv_tiles = (static_cast<int64_t>(n_kv) + 127) / 128;
  if (row_terms > kNoAllocMaxRowTerms || kv_tiles > kNoAllocMaxKvTiles) return TT_ERR_WORKSPACE;
  const int64_t ws_bytes = tt_tree_attn_bwd_workspace_size(dtype, n_q, n_kv, hq, hkv, D);
  if (ws_bytes < 0 || ws_bytes > kNoAllocBytes) return TT_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = scratch_on_current_device(&scratch);
  if (rc != TT_OK) return rc;
  return tt_tree_attn_bwd(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v, v_st,
                          v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi, fwd_ptr, fwd_list,
                          bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh, dk, dk_st, dk_sh, dv, dv_st,
                          dv_sh, scratch, ws_bytes, TT_BWD_ALL, status, stream);
}
