// Tree-correct depthwise causal conv + SiLU (forward and backward).
//
// Restates _tree_correct_conv_varlen (tree_dfs_ssm.py:285-348; same
// semantics at dfs_tree_forward.py:191-246): every node convolves
// [parent's last K-1 effective inputs, own tokens] and saves its own last K-1
// effective inputs for its children (:338-346), roots see zero padding.  So
// token t's window is the K-1 tokens before it on its root-to-node path.  The
// host turns the tree into pred[t][m-1] (token m steps back, or -1) once;
// the kernels are then plain gathers, and the backward gathers over the
// inverse map (successor CSR) so dx needs no atomics.
#include <type_traits>
#include <vector>

#include "tt_common.cuh"

extern "C" int tt_conv_predecessors(int32_t n_nodes, const int32_t* bounds,
                                    const int32_t* parents, int32_t K, int32_t* pred) {
  if (n_nodes < 0 || K < 1 || K > 8 || (n_nodes > 0 && (!bounds || !parents))) return TT_ERR_INVALID_ARG;
  if (n_nodes == 0) return TT_OK;
  const int S = bounds[2 * (n_nodes - 1) + 1];
  std::vector<int> prev(S, -1), last(n_nodes, -1);
  int expect = 0;
  for (int c = 0; c < n_nodes; ++c) {
    const int s = bounds[2 * c], e = bounds[2 * c + 1], p = parents[c];
    if (s != expect || e < s || p < -1 || p >= c) return TT_ERR_INVALID_ARG;
    expect = e;
    int before = p >= 0 ? last[p] : -1;
    for (int t = s; t < e; ++t) {
      prev[t] = before;
      before = t;
    }
    last[c] = before;   // a 0-token node hands its parent's context on
  }
  if (!pred) return TT_OK;
  for (int t = 0; t < S; ++t) {
    int cur = t;
    for (int m = 0; m < K - 1; ++m) {
      cur = cur >= 0 ? prev[cur] : -1;
      pred[(int64_t)t * (K - 1) + m] = cur;
    }
  }
  return TT_OK;
}

extern "C" int tt_conv_successors(int32_t S, int32_t K, const int32_t* pred, int32_t* succ_ptr,
                                  int32_t* succ_tok, int32_t* succ_lag, int64_t cap) {
  if (S < 0 || K < 1 || K > 8 || (S > 0 && (!pred || !succ_ptr))) return TT_ERR_INVALID_ARG;
  std::vector<int> cnt(S + 1, 0);
  for (int t = 0; t < S; ++t)
    for (int m = 0; m < K - 1; ++m) {
      const int p = pred[(int64_t)t * (K - 1) + m];
      if (p >= 0) cnt[p + 1]++;
    }
  for (int t = 0; t < S; ++t) cnt[t + 1] += cnt[t];
  for (int t = 0; t <= S; ++t) succ_ptr[t] = cnt[t];
  if ((int64_t)cnt[S] > cap) return TT_ERR_CAPACITY;
  std::vector<int> fill(cnt.begin(), cnt.end() - 1);
  for (int t = 0; t < S; ++t)
    for (int m = 0; m < K - 1; ++m) {
      const int p = pred[(int64_t)t * (K - 1) + m];
      if (p >= 0) {
        succ_tok[fill[p]] = t;
        succ_lag[fill[p]] = m + 1;
        ++fill[p];
      }
    }
  return TT_OK;
}

namespace tt {
namespace {

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

constexpr int kConvTok = 256;   // tokens per block (one per thread)
constexpr int kConvCh = 8;      // channels per thread: the token's predecessor and
                                // successor indices are read once for all of them
constexpr int kPartW = 9;       // per (channel, block): dw[0..K-1], db at [8]
constexpr int kSuccAhead = 8;   // successors whose indices conv_bwd_dx fetches up front

// The window of token t in channel c: xs[m] = x[c][pred_m(t)] for m < K
// (pred_0 = t, 0 where the path is shorter).  Every channel's loads are issued
// before any arithmetic, so a thread keeps kConvCh * K gathers in flight; rows
// past C read row C - 1 and are never used.
template <typename T, int K>
__device__ __forceinline__ void load_windows(const T* __restrict__ x, int C, int S, int c0, int t,
                                             bool live, const int (&pr)[K > 1 ? K - 1 : 1],
                                             float (&xs)[kConvCh][K]) {
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc) {
    const T* xc = x + (int64_t)min(c0 + cc, C - 1) * S;
    xs[cc][0] = live ? to_f32(xc[t]) : 0.f;
#pragma unroll
    for (int m = 1; m < K; ++m) xs[cc][m] = (live && pr[m - 1] >= 0) ? to_f32(xc[pr[m - 1]]) : 0.f;
  }
}

template <int K>
__device__ __forceinline__ void load_pred(const int32_t* __restrict__ pred, int t, bool live,
                                          int (&pr)[K > 1 ? K - 1 : 1]) {
  pr[0] = -1;
#pragma unroll
  for (int m = 0; m < K - 1; ++m) pr[m] = live ? pred[(int64_t)t * (K - 1) + m] : -1;
}

// pre[c][t] = bias + sum_{m=0}^{K-1} w[c][K-1-m] x[c][pred_m(t)],  out = silu(pre)
template <typename T, int K>
__global__ void __launch_bounds__(kConvTok)
conv_fwd(int C, int S, const T* __restrict__ x, const float* __restrict__ w,
         const float* __restrict__ bias, const int32_t* __restrict__ pred, T* __restrict__ out) {
  const int t = blockIdx.x * kConvTok + threadIdx.x;
  const int c0 = blockIdx.y * kConvCh;
  if (t >= S) return;
  int pr[K > 1 ? K - 1 : 1];
  load_pred<K>(pred, t, true, pr);
  float xs[kConvCh][K];
  load_windows<T, K>(x, C, S, c0, t, true, pr, xs);
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc) {
    const int c = c0 + cc;
    if (c >= C) break;
    const float* wc = w + (int64_t)c * K;
    float pre = bias ? bias[c] : 0.f;
#pragma unroll
    for (int m = 0; m < K; ++m) pre = fmaf(wc[K - 1 - m], xs[cc][m], pre);
    out[(int64_t)c * S + t] = from_f32<T>(silu(pre));
  }
}

// dpre[c][t] = dy * d silu(pre)/d pre at every (channel, token), and per block
// of 256 tokens the partial sums of dw[c][j] = sum_t dpre x[pred_{K-1-j}(t)]
// and db[c] = sum_t dpre (reduced in a fixed order by conv_bwd_dw_reduce).
template <typename T, int K>
__global__ void __launch_bounds__(kConvTok)
conv_bwd_dpre(int C, int S, const T* __restrict__ x, const float* __restrict__ w,
              const float* __restrict__ bias, const int32_t* __restrict__ pred,
              const T* __restrict__ dy, float* __restrict__ dpre, float* __restrict__ part,
              int nb) {
  const int t = blockIdx.x * kConvTok + threadIdx.x;
  const int c0 = blockIdx.y * kConvCh;
  const bool live = t < S;
  int pr[K > 1 ? K - 1 : 1];
  load_pred<K>(pred, t, live, pr);
  float xs[kConvCh][K], g[kConvCh];
  load_windows<T, K>(x, C, S, c0, t, live, pr, xs);
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc)
    g[cc] = live ? to_f32(dy[(int64_t)min(c0 + cc, C - 1) * S + t]) : 0.f;
  __shared__ float red[kConvCh][kPartW][kConvTok / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc) {
    const int c = c0 + cc;
    if (c >= C) break;                       // the same for the whole block
    const float* wc = w + (int64_t)c * K;
    float pre = bias ? bias[c] : 0.f;
#pragma unroll
    for (int m = 0; m < K; ++m) pre = fmaf(wc[K - 1 - m], xs[cc][m], pre);
    const float sg = 1.f / (1.f + __expf(-pre));
    const float d = live ? g[cc] * sg * (1.f + pre * (1.f - sg)) : 0.f;
    if (live) dpre[(int64_t)c * S + t] = d;
#pragma unroll
    for (int j = 0; j < kPartW; ++j) {
      // j < K: weight index j, i.e. predecessor m = K-1-j; j = 8: bias; the
      // slots K..7 are never read and hold 0
      if (j >= K && j != 8) {
        if (lane == 0) red[cc][j][wid] = 0.f;
        continue;
      }
      float v = j == 8 ? d : d * xs[cc][j < K ? K - 1 - j : 0];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[cc][j][wid] = v;
    }
  }
  __syncthreads();
  const int n_ch = min(kConvCh, C - c0);
  for (int i = threadIdx.x; i < n_ch * kPartW; i += kConvTok) {
    const int cc = i / kPartW, j = i % kPartW;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < kConvTok / 32; ++q) v += red[cc][j][q];
    part[((int64_t)(c0 + cc) * nb + blockIdx.x) * kPartW + j] = v;
  }
}

__global__ void conv_bwd_dw_reduce(int C, int K, int nb, const float* __restrict__ part,
                                   float* __restrict__ dw, float* __restrict__ db) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C * kPartW) return;
  const int c = i / kPartW, j = i % kPartW;
  if (j >= K && j != 8) return;
  if (j == 8 && !db) return;
  float v = 0.f;
  for (int b = 0; b < nb; ++b) v += part[((int64_t)c * nb + b) * kPartW + j];
  if (j == 8) db[c] = v;
  else dw[(int64_t)c * K + j] = v;
}

// dx[c][t] = w[c][K-1] dpre[c][t] + sum over the tokens u that have t as their
// lag-l predecessor of w[c][K-1-l] dpre[c][u]  (successor CSR, fixed order).
// The first kSuccAhead successors' indices are fetched together, then all
// their dpre loads; longer lists (the last tokens of a node with many
// children) continue one successor at a time.
template <typename T, int K>
__global__ void __launch_bounds__(kConvTok)
conv_bwd_dx(int C, int S, const float* __restrict__ w, const float* __restrict__ dpre,
            const int32_t* __restrict__ sp, const int32_t* __restrict__ stok,
            const int32_t* __restrict__ slag, T* __restrict__ dx) {
  const int t = blockIdx.x * kConvTok + threadIdx.x;
  if (t >= S) return;
  const int c0 = blockIdx.y * kConvCh;
  const int n_ch = min(kConvCh, C - c0);
  const int e0 = sp[t], e1 = sp[t + 1];
  int us[kSuccAhead], ls[kSuccAhead];
#pragma unroll
  for (int i = 0; i < kSuccAhead; ++i) {
    const bool has = e0 + i < e1;
    us[i] = has ? stok[e0 + i] : -1;
    ls[i] = has ? slag[e0 + i] : 0;
  }
  float acc[kConvCh];
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc) {
    const int64_t c = min(c0 + cc, C - 1);
    acc[cc] = w[c * K + K - 1] * dpre[c * S + t];
  }
#pragma unroll
  for (int i = 0; i < kSuccAhead; ++i) {
    if (us[i] < 0) break;
#pragma unroll
    for (int cc = 0; cc < kConvCh; ++cc) {
      const int64_t c = min(c0 + cc, C - 1);
      acc[cc] = fmaf(w[c * K + K - 1 - ls[i]], dpre[c * S + us[i]], acc[cc]);
    }
  }
  for (int e = e0 + kSuccAhead; e < e1; ++e) {
    const int u = stok[e], l = slag[e];
#pragma unroll
    for (int cc = 0; cc < kConvCh; ++cc) {
      const int64_t c = min(c0 + cc, C - 1);
      acc[cc] = fmaf(w[c * K + K - 1 - l], dpre[c * S + u], acc[cc]);
    }
  }
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc)
    if (cc < n_ch) dx[(int64_t)(c0 + cc) * S + t] = from_f32<T>(acc[cc]);
}

// f(std::integral_constant<int, K>()) for the runtime window length K in 1..8
template <typename Fn>
int by_k(int K, Fn fn) {
  switch (K) {
    case 1: return fn(std::integral_constant<int, 1>());
    case 2: return fn(std::integral_constant<int, 2>());
    case 3: return fn(std::integral_constant<int, 3>());
    case 4: return fn(std::integral_constant<int, 4>());
    case 5: return fn(std::integral_constant<int, 5>());
    case 6: return fn(std::integral_constant<int, 6>());
    case 7: return fn(std::integral_constant<int, 7>());
    case 8: return fn(std::integral_constant<int, 8>());
    default: return TT_ERR_INVALID_ARG;
  }
}

template <typename Fn>
int by_dtype(int dtype, Fn fn) {
  switch (dtype) {
    case TT_F32: return fn(float());
    case TT_BF16: return fn(__nv_bfloat16());
    case TT_F16: return fn(__half());
    default: return TT_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace tt

extern "C" int tt_tree_conv_fwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                const float* weight, const float* bias, const int32_t* pred,
                                void* out, void* stream) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return TT_ERR_INVALID_ARG;
  if (C == 0 || S == 0) return TT_OK;
  if (!x || !weight || !out || (K > 1 && !pred)) return TT_ERR_INVALID_ARG;
  return tt::by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return tt::by_k(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      dim3 g((S + tt::kConvTok - 1) / tt::kConvTok, (C + tt::kConvCh - 1) / tt::kConvCh);
      tt::conv_fwd<T, KK><<<g, tt::kConvTok, 0, (cudaStream_t)stream>>>(
          C, S, (const T*)x, weight, bias, pred, (T*)out);
      tt_count_launches(1);
      return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
    });
  });
}

extern "C" int64_t tt_tree_conv_bwd_workspace_size(int32_t C, int32_t S, int32_t K) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return -1;
  const int64_t nb = ((int64_t)S + tt::kConvTok - 1) / tt::kConvTok;
  return (int64_t)C * S * 4 + (int64_t)C * nb * tt::kPartW * 4 + 256;
}

extern "C" int tt_tree_conv_bwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                const float* weight, const float* bias, const int32_t* pred,
                                const int32_t* succ_ptr, const int32_t* succ_tok,
                                const int32_t* succ_lag, const void* dout, void* dx,
                                float* dweight, float* dbias, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return TT_ERR_INVALID_ARG;
  if (C == 0 || S == 0) return TT_OK;
  if (!x || !weight || !dout || !dx || !dweight || !succ_ptr || (K > 1 && !pred))
    return TT_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < tt_tree_conv_bwd_workspace_size(C, S, K))
    return TT_ERR_WORKSPACE;
  return tt::by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    cudaStream_t st = (cudaStream_t)stream;
    const int nb = (S + tt::kConvTok - 1) / tt::kConvTok;
    float* dpre = static_cast<float*>(workspace);
    float* part = dpre + (int64_t)C * S;
    dim3 g(nb, (C + tt::kConvCh - 1) / tt::kConvCh);
    return tt::by_k(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      tt::conv_bwd_dpre<T, KK><<<g, tt::kConvTok, 0, st>>>(C, S, (const T*)x, weight, bias, pred,
                                                           (const T*)dout, dpre, part, nb);
      tt::conv_bwd_dw_reduce<<<(C * tt::kPartW + 255) / 256, 256, 0, st>>>(C, K, nb, part,
                                                                         dweight, dbias);
      tt::conv_bwd_dx<T, KK><<<g, tt::kConvTok, 0, st>>>(C, S, weight, dpre, succ_ptr, succ_tok,
                                                         succ_lag, (T*)dx);
      tt_count_launches(3);
      return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
    });
  });
}
