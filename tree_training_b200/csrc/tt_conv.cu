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

// pre[c][t] = bias + sum_{m=0}^{K-1} w[c][K-1-m] x[c][pred_m(t)]   (pred_0 = t)
template <typename T>
__device__ __forceinline__ float conv_pre(const T* __restrict__ xc, const float* __restrict__ wc,
                                          float b, const int32_t* __restrict__ pr, int t, int K) {
  float acc = b + wc[K - 1] * to_f32(xc[t]);
  for (int m = 1; m < K; ++m) {
    const int p = pr[(int64_t)t * (K - 1) + m - 1];
    if (p >= 0) acc = fmaf(wc[K - 1 - m], to_f32(xc[p]), acc);
  }
  return acc;
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

template <typename T>
__global__ void conv_fwd(int C, int S, int K, const T* __restrict__ x, const float* __restrict__ w,
                         const float* __restrict__ bias, const int32_t* __restrict__ pred, T* out) {
  const int c = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= S) return;
  const float pre = conv_pre(x + (int64_t)c * S, w + (int64_t)c * K, bias ? bias[c] : 0.f, pred, t, K);
  out[(int64_t)c * S + t] = from_f32<T>(silu(pre));
}

template <typename T>
__device__ __forceinline__ float dpre_at(const T* xc, const T* dyc, const float* wc, float b,
                                         const int32_t* pred, int t, int K) {
  const float pre = conv_pre(xc, wc, b, pred, t, K);
  const float sg = 1.f / (1.f + __expf(-pre));
  return to_f32(dyc[t]) * sg * (1.f + pre * (1.f - sg));
}

template <typename T>
__global__ void conv_bwd_dx(int C, int S, int K, const T* __restrict__ x,
                            const float* __restrict__ w, const float* __restrict__ bias,
                            const int32_t* __restrict__ pred, const int32_t* __restrict__ sp,
                            const int32_t* __restrict__ stok, const int32_t* __restrict__ slag,
                            const T* __restrict__ dy, T* dx) {
  const int c = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= S) return;
  const T* xc = x + (int64_t)c * S;
  const T* dyc = dy + (int64_t)c * S;
  const float* wc = w + (int64_t)c * K;
  const float b = bias ? bias[c] : 0.f;
  float acc = wc[K - 1] * dpre_at(xc, dyc, wc, b, pred, t, K);
  for (int e = sp[t]; e < sp[t + 1]; ++e)
    acc = fmaf(wc[K - 1 - slag[e]], dpre_at(xc, dyc, wc, b, pred, stok[e], K), acc);
  dx[(int64_t)c * S + t] = from_f32<T>(acc);
}

template <typename T>
__global__ void conv_bwd_dw(int C, int S, int K, const T* __restrict__ x,
                            const float* __restrict__ w, const float* __restrict__ bias,
                            const int32_t* __restrict__ pred, const T* __restrict__ dy, float* dw,
                            float* db) {
  const int c = blockIdx.x;
  const T* xc = x + (int64_t)c * S;
  const T* dyc = dy + (int64_t)c * S;
  const float* wc = w + (int64_t)c * K;
  const float b = bias ? bias[c] : 0.f;
  float acc[9] = {};
  for (int t = threadIdx.x; t < S; t += blockDim.x) {
    const float d = dpre_at(xc, dyc, wc, b, pred, t, K);
    acc[K - 1] += d * to_f32(xc[t]);
    for (int m = 1; m < K; ++m) {
      const int p = pred[(int64_t)t * (K - 1) + m - 1];
      if (p >= 0) acc[K - 1 - m] += d * to_f32(xc[p]);
    }
    acc[8] += d;
  }
  __shared__ float red[9][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int i = 0; i < 9; ++i) {
    float v = acc[i];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[i][wid] = v;
  }
  __syncthreads();
  if (threadIdx.x < 9) {
    float v = 0.f;
    for (int i = 0; i < nw; ++i) v += red[threadIdx.x][i];
    if (threadIdx.x < K) dw[(int64_t)c * K + threadIdx.x] = v;
    if (threadIdx.x == 8 && db) db[c] = v;
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
    dim3 g((S + 255) / 256, C);
    tt::conv_fwd<T><<<g, 256, 0, (cudaStream_t)stream>>>(C, S, K, (const T*)x, weight, bias, pred,
                                                          (T*)out);
    tt_count_launches(1);
    return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
  });
}

extern "C" int tt_tree_conv_bwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                const float* weight, const float* bias, const int32_t* pred,
                                const int32_t* succ_ptr, const int32_t* succ_tok,
                                const int32_t* succ_lag, const void* dout, void* dx,
                                float* dweight, float* dbias, void* stream) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return TT_ERR_INVALID_ARG;
  if (C == 0 || S == 0) return TT_OK;
  if (!x || !weight || !dout || !dx || !dweight || !succ_ptr || (K > 1 && !pred))
    return TT_ERR_INVALID_ARG;
  return tt::by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    cudaStream_t st = (cudaStream_t)stream;
    dim3 g((S + 255) / 256, C);
    tt::conv_bwd_dx<T><<<g, 256, 0, st>>>(C, S, K, (const T*)x, weight, bias, pred, succ_ptr,
                                          succ_tok, succ_lag, (const T*)dout, (T*)dx);
    tt::conv_bwd_dw<T><<<C, 256, 0, st>>>(C, S, K, (const T*)x, weight, bias, pred,
                                          (const T*)dout, dweight, dbias);
    tt_count_launches(2);
    return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
  });
}
