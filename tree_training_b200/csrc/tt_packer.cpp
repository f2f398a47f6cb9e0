// Host packer and tile work-list builder (C ABI, no CUDA).
//
// tt_pack_forest restates the per-token/per-node outputs of
// build_dfs_tree_info (dfs_tree_forward.py:91-139) for a forest that the
// caller already walked in pre-order, and replaces the O(visible pairs) dense
// mask loop (dfs_tree_forward.py:157-172) by one [lo, hi) row interval per key:
// in pre-order every subtree is a contiguous token range, so key j (in node c)
// is visible exactly to the rows [j, end of c's subtree).
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <vector>

#include "../../include/tree_training_b200.h"

extern "C" const char* tt_status_string(int s) {
  switch (s) {
    case TT_OK: return "ok";
    case TT_ERR_INVALID_ARG: return "invalid argument";
    case TT_ERR_UNSUPPORTED: return "unsupported dtype/head_dim/layout";
    case TT_ERR_CUDA: return "CUDA error";
    case TT_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case TT_ERR_NOT_INTERVAL: return "mask is not a per-key row interval (not a tree mask)";
    case TT_ERR_WORKSPACE: return "workspace too small";
    case TT_ERR_CAPACITY: return "output list capacity too small";
    default: return "unknown status";
  }
}

extern "C" int tt_abi_version(void) { return 3; }

extern "C" int tt_pack_forest(int32_t n_nodes, const int32_t* node_len,
                              const int32_t* node_parent, int32_t pos_offset, int32_t* pos_ids,
                              int32_t* chunk_bounds, int32_t* subtree_end, int32_t* leaf_ids,
                              int32_t* n_leaves, int32_t* token_node, int32_t* kv_lo,
                              int32_t* kv_hi) {
  if (n_nodes < 0 || (n_nodes > 0 && (!node_len || !node_parent))) return TT_ERR_INVALID_ARG;
  std::vector<int64_t> start(n_nodes), depth(n_nodes), sub_end(n_nodes);
  std::vector<char> has_child(n_nodes, 0);
  std::vector<int32_t> path;  // current root-to-node path of the pre-order walk
  path.reserve(64);
  int64_t tok = 0;
  for (int32_t i = 0; i < n_nodes; ++i) {
    const int32_t L = node_len[i], p = node_parent[i];
    if (L < 0 || p < -1 || p >= i) return TT_ERR_INVALID_ARG;
    // pre-order: the parent must be on the path to the previous node
    while (!path.empty() && path.back() != p) path.pop_back();
    if (p >= 0 && path.empty()) return TT_ERR_INVALID_ARG;
    path.push_back(i);
    start[i] = tok;
    depth[i] = (p < 0) ? 0 : depth[p] + node_len[p];
    tok += L;
    if (tok > INT32_MAX) return TT_ERR_INVALID_ARG;
    if (p >= 0) has_child[p] = 1;
  }
  for (int32_t i = 0; i < n_nodes; ++i) sub_end[i] = start[i] + node_len[i];
  for (int32_t i = n_nodes - 1; i > 0; --i) {
    const int32_t p = node_parent[i];
    if (p >= 0 && sub_end[i] > sub_end[p]) sub_end[p] = sub_end[i];
  }
  int32_t nl = 0;
  for (int32_t i = 0; i < n_nodes; ++i) {
    const int64_t s = start[i], e = s + node_len[i];
    if (chunk_bounds) {
      chunk_bounds[2 * i] = (int32_t)s;
      chunk_bounds[2 * i + 1] = (int32_t)e;
    }
    if (subtree_end) subtree_end[i] = (int32_t)sub_end[i];
    if (!has_child[i]) {
      if (leaf_ids) leaf_ids[nl] = i;
      ++nl;
    }
    for (int64_t t = s; t < e; ++t) {
      if (pos_ids) pos_ids[t] = (int32_t)(pos_offset + depth[i] + (t - s));
      if (token_node) token_node[t] = i;
      if (kv_lo) kv_lo[t] = (int32_t)t;
      if (kv_hi) kv_hi[t] = (int32_t)sub_end[i];
    }
  }
  if (n_leaves) *n_leaves = nl;
  return TT_OK;
}

extern "C" int tt_gateway_intervals_from_bias(int32_t past_len, const float* bias, int32_t n_q,
                                              int32_t* kv_lo, int32_t* kv_hi) {
  if (past_len < 0 || n_q < 0 || (past_len > 0 && (!bias || !kv_lo || !kv_hi)))
    return TT_ERR_INVALID_ARG;
  for (int32_t j = 0; j < past_len; ++j) {
    const float b = bias[j];
    if (b == 0.0f) {
      kv_lo[j] = 0;
      kv_hi[j] = n_q;
    } else if (b < -1e30f) {  // -inf, or a dtype-min "masked" value
      kv_lo[j] = 0;
      kv_hi[j] = 0;
    } else {
      return TT_ERR_NOT_INTERVAL;
    }
  }
  return TT_OK;
}

extern "C" int tt_build_tiles(int32_t n_q, int32_t n_kv, const int32_t* kv_lo,
                              const int32_t* kv_hi, int32_t tile_q, int32_t tile_kv,
                              int32_t* fwd_ptr, int32_t* fwd_list, int32_t* bwd_ptr,
                              int32_t* bwd_list, int64_t list_cap, int64_t* visible_pairs) {
  if (n_q < 0 || n_kv < 0 || tile_q <= 0 || tile_kv <= 0) return TT_ERR_INVALID_ARG;
  if (n_kv > 0 && (!kv_lo || !kv_hi)) return TT_ERR_INVALID_ARG;
  const int32_t nqt = (n_q + tile_q - 1) / tile_q;
  const int32_t nkt = (n_kv + tile_kv - 1) / tile_kv;
  if ((fwd_list || bwd_list) && list_cap < (int64_t)nqt * nkt) return TT_ERR_CAPACITY;
  int64_t pairs = 0;
  std::vector<int32_t> diff(nqt + 1);
  // per kv tile: visible q tiles with flag; kept to emit both list orders
  std::vector<std::vector<int32_t>> per_q(nqt);
  if (bwd_ptr) bwd_ptr[0] = 0;
  int64_t bwd_n = 0;
  for (int32_t kt = 0; kt < nkt; ++kt) {
    std::fill(diff.begin(), diff.end(), 0);
    const int32_t j0 = kt * tile_kv, j1 = std::min(n_kv, j0 + tile_kv);
    const bool complete = (j1 - j0) == tile_kv;
    int32_t max_lo = INT32_MIN, min_hi = INT32_MAX;
    for (int32_t j = j0; j < j1; ++j) {
      int32_t lo = std::max(kv_lo[j], 0), hi = std::min(kv_hi[j], n_q);
      max_lo = std::max(max_lo, kv_lo[j]);
      min_hi = std::min(min_hi, kv_hi[j]);
      if (lo >= hi) continue;
      pairs += hi - lo;
      diff[lo / tile_q] += 1;
      diff[(hi - 1) / tile_q + 1] -= 1;
    }
    int32_t run = 0;
    for (int32_t qt = 0; qt < nqt; ++qt) {
      run += diff[qt];
      if (run <= 0) continue;
      const int32_t q0 = qt * tile_q, q1 = std::min(n_q, q0 + tile_q);
      const bool full = complete && max_lo <= q0 && min_hi >= q1;
      const int32_t e_kv = kt * 2 + (full ? 0 : 1);
      const int32_t e_q = qt * 2 + (full ? 0 : 1);
      per_q[qt].push_back(e_kv);
      if (bwd_list) bwd_list[bwd_n] = e_q;
      ++bwd_n;
    }
    if (bwd_ptr) bwd_ptr[kt + 1] = (int32_t)bwd_n;
  }
  if (fwd_ptr) {
    int64_t n = 0;
    fwd_ptr[0] = 0;
    for (int32_t qt = 0; qt < nqt; ++qt) {
      for (int32_t e : per_q[qt]) {
        if (fwd_list) fwd_list[n] = e;
        ++n;
      }
      fwd_ptr[qt + 1] = (int32_t)n;
    }
  }
  if (visible_pairs) *visible_pairs = pairs;
  return TT_OK;
}
