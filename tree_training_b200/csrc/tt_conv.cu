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

// SiLU and the logistic sigmoid with the fast exponential and divide (a few
// ulp; the conv's outputs carry them into 16-bit or fp32 values checked at
// 1e-5 against the float64 oracle)
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }
// d silu(pre) / d pre times the output gradient g (every backward kernel
// computes dpre through this one expression, so their dpre agree bit for bit)
__device__ __forceinline__ float silu_grad(float g, float pre) {
  const float sg = sigm(pre);
  return g * sg * (1.f + pre * (1.f - sg));
}

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
    const float d = live ? silu_grad(g[cc], pre) : 0.f;
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

// ---- four tokens per thread --------------------------------------------------
// The two backward kernels with each thread on 4 consecutive tokens (one 8- or
// 16-byte access per channel row instead of four 2- or 4-byte ones) for
// S % 4 == 0 and 16-byte aligned rows.  (The forward keeps one token per
// thread: on the config-4 tree its 4-token form measured 0.56 ms against
// 0.37 ms.)  A group whose 4 tokens all have the
// plain window pred_m(t) = t - m (the inside of a node, K <= 5) reads its
// whole window as two quads x[t0-4 .. t0+3]; other groups gather per token as
// above.  Per output the arithmetic and its order are those of the kernels
// above; the dw partials add each thread's 4 tokens before the warp sum.
constexpr int kConvThr4 = kConvTok / 4;     // threads per block: still 256 tokens

template <typename T>
struct alignas(4 * sizeof(T)) Quad {
  T v[4];
};

template <typename T>
__device__ __forceinline__ void ld_quad(const T* p, float* out) {
  const Quad<T> q = *reinterpret_cast<const Quad<T>*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = to_f32(q.v[i]);
}

template <typename T>
__device__ __forceinline__ void st_quad(T* p, const float* in) {
  Quad<T> q;
#pragma unroll
  for (int i = 0; i < 4; ++i) q.v[i] = from_f32<T>(in[i]);
  *reinterpret_cast<Quad<T>*>(p) = q;
}

// pr[i][m] = pred_{m+1}(t0 + i); returns whether all four windows are plain.
template <int K>
__device__ __forceinline__ bool load_pred4(const int32_t* __restrict__ pred, int t0,
                                           int (&pr)[4][K > 1 ? K - 1 : 1]) {
  bool plain = K <= 5 && t0 >= 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    pr[i][0] = -1;
#pragma unroll
    for (int m = 0; m < K - 1; ++m) {
      pr[i][m] = pred[(int64_t)(t0 + i) * (K - 1) + m];
      plain &= pr[i][m] == t0 + i - 1 - m;
    }
  }
  return plain;
}

// The 4-token kernels hold the windows of half their channels at a time
// (registers: 4 channels x 4 tokens x K floats).
constexpr int kHalfCh = kConvCh / 2;

// xs[cc][i][m] = x[c0 + cc][pred_m(t0 + i)] (0 where the path is shorter)
template <typename T, int K>
__device__ __forceinline__ void load_windows4(const T* __restrict__ x, int C, int S, int c0,
                                              int t0, bool plain,
                                              const int (&pr)[4][K > 1 ? K - 1 : 1],
                                              float (&xs)[kHalfCh][4][K]) {
#pragma unroll
  for (int cc = 0; cc < kHalfCh; ++cc) {
    const T* xc = x + (int64_t)min(c0 + cc, C - 1) * S;
    if (plain) {
      float q[8];
      ld_quad(xc + t0 - 4, q);
      ld_quad(xc + t0, q + 4);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int m = 0; m < K; ++m) xs[cc][i][m] = q[4 + i - m];
    } else {
      float q[4];
      ld_quad(xc + t0, q);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xs[cc][i][0] = q[i];
#pragma unroll
        for (int m = 1; m < K; ++m)
          xs[cc][i][m] = pr[i][m - 1] >= 0 ? to_f32(xc[pr[i][m - 1]]) : 0.f;
      }
    }
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(kConvThr4)
conv_bwd_dpre4(int C, int S, const T* __restrict__ x, const float* __restrict__ w,
               const float* __restrict__ bias, const int32_t* __restrict__ pred,
               const T* __restrict__ dy, float* __restrict__ dpre, float* __restrict__ part,
               int nb) {
  const int t0 = (blockIdx.x * kConvThr4 + threadIdx.x) * 4;
  const int c0 = blockIdx.y * kConvCh;
  const bool live = t0 < S;                 // S % 4 == 0: a live group is whole
  const int tl = live ? t0 : 0;
  int pr[4][K > 1 ? K - 1 : 1];
  const bool plain = load_pred4<K>(pred, tl, pr);
  __shared__ float red[kConvCh][kPartW][kConvThr4 / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll 1
  for (int hc = 0; hc < kConvCh; hc += kHalfCh) {
    float xs[kHalfCh][4][K], g[kHalfCh][4];
    load_windows4<T, K>(x, C, S, c0 + hc, tl, plain, pr, xs);
#pragma unroll
    for (int cc = 0; cc < kHalfCh; ++cc)
      ld_quad(dy + (int64_t)min(c0 + hc + cc, C - 1) * S + tl, g[cc]);
#pragma unroll
    for (int cc = 0; cc < kHalfCh; ++cc) {
      const int c = c0 + hc + cc;
      if (c >= C) break;                     // the same for the whole block
      const float* wc = w + (int64_t)c * K;
      float d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float pre = bias ? bias[c] : 0.f;
#pragma unroll
        for (int m = 0; m < K; ++m) pre = fmaf(wc[K - 1 - m], xs[cc][i][m], pre);
        d[i] = live ? silu_grad(g[cc][i], pre) : 0.f;
      }
      if (live)
        *reinterpret_cast<float4*>(dpre + (int64_t)c * S + t0) = make_float4(d[0], d[1], d[2], d[3]);
#pragma unroll
      for (int j = 0; j < kPartW; ++j) {
        if (j >= K && j != 8) {
          if (lane == 0) red[hc + cc][j][wid] = 0.f;
          continue;
        }
        float v = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) v += j == 8 ? d[i] : d[i] * xs[cc][i][j < K ? K - 1 - j : 0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[hc + cc][j][wid] = v;
      }
    }
  }
  __syncthreads();
  const int n_ch = min(kConvCh, C - c0);
  for (int i = threadIdx.x; i < n_ch * kPartW; i += kConvThr4) {
    const int cc = i / kPartW, j = i % kPartW;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < kConvThr4 / 32; ++q) v += red[cc][j][q];
    part[((int64_t)(c0 + cc) * nb + blockIdx.x) * kPartW + j] = v;
  }
}

// dx of 4 tokens: a group whose tokens' successors are exactly t+1 .. t+K-1
// (lags 1 .. K-1, in that order: the inside of a node) reads dpre[t0 .. t0+7]
// as two quads; other groups walk each token's successor list as conv_bwd_dx.
template <typename T, int K>
__global__ void __launch_bounds__(kConvThr4)
conv_bwd_dx4(int C, int S, const float* __restrict__ w, const float* __restrict__ dpre,
             const int32_t* __restrict__ sp, const int32_t* __restrict__ stok,
             const int32_t* __restrict__ slag, T* __restrict__ dx) {
  const int t0 = (blockIdx.x * kConvThr4 + threadIdx.x) * 4;
  if (t0 >= S) return;
  const int c0 = blockIdx.y * kConvCh;
  const int n_ch = min(kConvCh, C - c0);
  int e[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) e[i] = sp[t0 + i];
  bool plain = K <= 5 && t0 + 8 <= S;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    plain &= e[i + 1] - e[i] == K - 1;
#pragma unroll
    for (int m = 0; m < K - 1; ++m)
      if (plain) plain &= stok[e[i] + m] == t0 + i + 1 + m && slag[e[i] + m] == m + 1;
  }
  float acc[kConvCh][4];
  if (plain) {
#pragma unroll
    for (int cc = 0; cc < kConvCh; ++cc) {
      const int64_t c = min(c0 + cc, C - 1);
      const float4 a = *reinterpret_cast<const float4*>(dpre + c * S + t0);
      const float4 b = *reinterpret_cast<const float4*>(dpre + c * S + t0 + 4);
      const float q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s = w[c * K + K - 1] * q[i];
#pragma unroll
        for (int l = 1; l < K; ++l) s = fmaf(w[c * K + K - 1 - l], q[i + l], s);
        acc[cc][i] = s;
      }
    }
  } else {
#pragma unroll
    for (int cc = 0; cc < kConvCh; ++cc) {
      const int64_t c = min(c0 + cc, C - 1);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[cc][i] = w[c * K + K - 1] * dpre[c * S + t0 + i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      for (int ee = e[i]; ee < e[i + 1]; ++ee) {
        const int u = stok[ee], l = slag[ee];
#pragma unroll
        for (int cc = 0; cc < kConvCh; ++cc) {
          const int64_t c = min(c0 + cc, C - 1);
          acc[cc][i] = fmaf(w[c * K + K - 1 - l], dpre[c * S + u], acc[cc][i]);
        }
      }
  }
#pragma unroll
  for (int cc = 0; cc < kConvCh; ++cc)
    if (cc < n_ch) st_quad(dx + (int64_t)(c0 + cc) * S + t0, acc[cc]);
}

// ---- token-major side ----------------------------------------------------------
// The conv output and its gradient in token-major memory ([S, C], channel rows
// contiguous: what the layer's transpose + split into q / k / v reads without a
// transposing copy).  One block per 64 channels x 128 tokens, 256 threads:
//   1. 16-byte cp.async copies stage the tile's x rows (channel-major, tokens
//      [t0 - 8, t0 + 128), the backward 8 more) in shared memory, the
//      backward also the dy rows (token-major, 64 channels); one ballot per
//      32 tokens marks the tokens whose window is t, t - 1, .., t - K + 1
//      (the inside of a node);
//   2. thread (r, q) = (lane + 32 (warp % 2), warp / 2) owns tile channel r
//      over tokens 32 q .. 32 q + 31: it holds the channel's weights in
//      registers and slides along the row, reading each x value once from
//      shared memory (16 bytes at a time) into a register window; a token
//      whose window leaves the node gathers its window from the predecessor
//      table instead (shared memory inside the staged range, global memory
//      outside).  The arithmetic per output is that of the channel-major
//      kernels, in the same order, so the results match them bit for bit;
//   3. the forward writes its output tile into shared memory (one 64-byte
//      token row per warp store) and then to global memory as whole 16-byte
//      row chunks; the backward keeps dpre in registers (see conv_bwd_tm).
// Needs S * sizeof(T) % 16 == 0, C % 8 == 0 and 16-byte aligned bases.
constexpr int kTmCh = 64;                    // channels per tile
constexpr int kTmTok = 128;                  // tokens per tile
constexpr int kTmThreads = 256;
constexpr int kTmHalo = 8;                   // staged tokens before the tile (K - 1 <= 7)
constexpr int kTmRun = 32;                   // tokens per thread

// x row stride (elements) for n staged tokens (a multiple of 16 bytes): the
// smallest with 4 words mod 8 per row, so the 8 lanes of a quarter warp reading
// 16 bytes each from 8 consecutive rows hit disjoint banks
template <typename T>
constexpr int x_row_stride(int n) {
  const int per_word = 4 / static_cast<int>(sizeof(T));
  const int words = n / per_word;
  return (words + (12 - words % 8) % 8) * per_word;
}

// kRight: tokens staged past the tile's end (x and the token-major rows)
template <typename T, int kRight>
struct TmTileR {
  static constexpr int kEl = 16 / static_cast<int>(sizeof(T));   // elements per 16 bytes
  static constexpr int kXS = kTmHalo + kTmTok + kRight;            // staged tokens per x row
  static constexpr int kXW = x_row_stride<T>(kXS);                 // x row stride
  static constexpr int kRows = kTmTok + kRight;                    // token-major rows
  static constexpr int kTW = kTmCh + kEl;                          // token row (+ one chunk pad)
  static constexpr int kBits = (kRows + 31) / 32;                  // plain-window words
  T x[kTmCh][kXW];                       // x[c0 + r][t0 - 8 + i]
  T tm[kRows][kTW];                      // token-major rows: out (fwd) or dy (bwd)
  float w[kTmCh * 8];                    // the tile's weights, [r][K]
  float b[kTmCh];                        // and biases (0 without)
  uint32_t plain[kBits];                 // bit j of word i: token t0 + 32 i + j
  alignas(16) int32_t pred[kRows * 7];   // the rows' predecessor table, [t][K - 1]
};
template <typename T>
using TmTile = TmTileR<T, 0>;

// Stage the tile's weights and biases.
template <int K, typename Tile>
__device__ __forceinline__ void stage_w(Tile& sm, const float* w, const float* bias, int C,
                                        int c0) {
  for (int i = threadIdx.x; i < kTmCh * K; i += kTmThreads) {
    const int c = c0 + i / K;
    sm.w[i] = c < C ? w[(int64_t)c0 * K + i] : 0.f;
  }
  for (int i = threadIdx.x; i < kTmCh; i += kTmThreads)
    sm.b[i] = (bias && c0 + i < C) ? bias[c0 + i] : 0.f;
}

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(ok ? 16u : 0u)
               : "memory");
}

// Stage x[c0 .. c0 + 63][t0 - 8 .. t0 + kXS - 9] (zero outside [0, S) and
// past C).
template <typename Tile, typename T>
__device__ __forceinline__ void stage_x(Tile& sm, const T* x, int C, int S, int c0, int t0) {
  constexpr int kEl = Tile::kEl, kXC = Tile::kXS / kEl;
  for (int q = threadIdx.x; q < kTmCh * kXC; q += kTmThreads) {
    const int r = q / kXC, k = q % kXC;
    const int c = c0 + r, t = t0 - kTmHalo + k * kEl;   // chunks are whole: S % kEl == 0
    const bool ok = c < C && t >= 0 && t < S;
    cp_async16_zfill(&sm.x[r][k * kEl], ok ? x + (int64_t)c * S + t : x, ok);
  }
}

// Stage the predecessor rows of tile tokens 0 .. kRows - 1 (16-byte chunks:
// t0 (K - 1) and S (K - 1) are multiples of 4; rows past S read as 0 and are
// never used).
template <int K, typename Tile>
__device__ __forceinline__ void stage_pred(Tile& sm, const int32_t* pred, int S, int t0) {
  if (K == 1) return;
  constexpr int kChunks = Tile::kRows * (K - 1) / 4;
  const int64_t end = (int64_t)S * (K - 1), base = (int64_t)t0 * (K - 1);
  for (int q = threadIdx.x; q < kChunks; q += kTmThreads) {
    const bool ok = base + 4 * q < end;
    cp_async16_zfill(&sm.pred[4 * q], ok ? pred + base + 4 * q : pred, ok);
  }
}

// The plain-window bits of tile tokens 0 .. 32 kBits - 1 (whole warps per word).
template <int K, typename Tile>
__device__ __forceinline__ void stage_plain(Tile& sm, const int32_t* __restrict__ pred, int S,
                                            int t0) {
  for (int base = (threadIdx.x >> 5) * 32; base < Tile::kBits * 32; base += kTmThreads) {
    const int t = t0 + base + (threadIdx.x & 31);
    bool pl = t < S;
    if (pl) {
      int pv[K > 1 ? K - 1 : 1];             // independent loads, then the compares
#pragma unroll
      for (int m = 0; m < K - 1; ++m) pv[m] = pred[(int64_t)t * (K - 1) + m];
#pragma unroll
      for (int m = 0; m < K - 1; ++m) pl = pl && pv[m] == t - 1 - m;
    }
    const uint32_t bits = __ballot_sync(0xffffffffu, pl);
    if ((threadIdx.x & 31) == 0) sm.plain[base >> 5] = bits;
  }
}

// The window of token t = t0 + tt in tile channel r (c = c0 + r) through the
// predecessor table: xs[m] = x[c][pred_m(t)], from shared memory inside the
// staged range, else from global memory (0 for t >= S or where the path is
// shorter).
template <int K, typename Tile, typename T>
__device__ __forceinline__ void window_gather(const Tile& sm, const T* __restrict__ x,
                                           const int32_t* __restrict__ pred, int S, int c, int r,
                                           int t0, int tt, float* xs) {
  const int t = t0 + tt;
  if (t >= S) {
    for (int m = 0; m < K; ++m) xs[m] = 0.f;
    return;
  }
  auto at = [&](int p) {
    return p < 0 ? 0.f
           : (p >= t0 - kTmHalo && p < t0 - kTmHalo + Tile::kXS)
               ? to_f32(sm.x[r][p - t0 + kTmHalo])
               : to_f32(x[(int64_t)c * S + p]);
  };
  xs[0] = at(t);
  const bool staged = tt < Tile::kRows;      // (tt >= 0: t >= t0 always)
  for (int m = 1; m < K; ++m)
    xs[m] = at(staged ? sm.pred[tt * (K - 1) + m - 1] : pred[(int64_t)t * (K - 1) + m - 1]);
}

// n consecutive x values of tile row r starting at staged index i0 (a
// multiple of kEl) into xr[0 .. n)
template <typename Tile, typename T>
__device__ __forceinline__ void ld_chunk(const Tile& sm, int r, int i0, float* xr) {
  const uint4 v = *reinterpret_cast<const uint4*>(&sm.x[r][i0]);
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < Tile::kEl; ++i) xr[i] = to_f32(e[i]);
}

template <typename T, int K>
__global__ void __launch_bounds__(kTmThreads, 4)
conv_fwd_tm(int C, int S, const T* __restrict__ x, const float* __restrict__ w,
            const float* __restrict__ bias, const int32_t* __restrict__ pred,
            T* __restrict__ out_tm) {
  extern __shared__ __align__(16) uint8_t tm_smem[];
  using Tile = TmTile<T>;
  Tile& sm = *reinterpret_cast<Tile*>(tm_smem);
  constexpr int kEl = Tile::kEl;
  const int c0 = blockIdx.y * kTmCh, t0 = blockIdx.x * kTmTok;
  stage_x(sm, x, C, S, c0, t0);
  stage_pred<K>(sm, pred, S, t0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  stage_w<K>(sm, w, bias, C, c0);
  stage_plain<K>(sm, pred, S, t0);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = (warp & 1) * 32 + lane, tq = (warp >> 1) * kTmRun;
  const uint32_t bits = sm.plain[warp >> 1];
  float wr[K];
#pragma unroll
  for (int m = 0; m < K; ++m) wr[m] = sm.w[r * K + m];
  const float b0 = sm.b[r];
  // clean: every window of the run is plain (a run inside one node), no
  // per-token branch
  auto run = [&](auto clean) {
    constexpr bool kClean = decltype(clean)::value;
    // xr[kTmHalo + j] = x at tile token tq + j
    float xr[kTmHalo + kTmRun];
    ld_chunk<Tile, T>(sm, r, tq, xr);
    if (kEl == 4) ld_chunk<Tile, T>(sm, r, tq + 4, xr + 4);
#pragma unroll
    for (int j = 0; j < kTmRun; ++j) {
      if (j % kEl == 0) ld_chunk<Tile, T>(sm, r, kTmHalo + tq + j, xr + kTmHalo + j);
      float xs[K];
      if (kClean || (bits >> j & 1)) {
#pragma unroll
        for (int m = 0; m < K; ++m) xs[m] = xr[kTmHalo + j - m];
      } else {
        window_gather<K>(sm, x, pred, S, min(c0 + r, C - 1), r, t0, tq + j, xs);
      }
      float pre = b0;
#pragma unroll
      for (int m = 0; m < K; ++m) pre = fmaf(wr[K - 1 - m], xs[m], pre);
      sm.tm[tq + j][r] = from_f32<T>(silu(pre));
    }
  };
  if (bits == 0xffffffffu)
    run(std::true_type());
  else
    run(std::false_type());
  __syncthreads();
  constexpr int kTC = kTmCh / kEl;               // 16-byte chunks per token row
  for (int q = threadIdx.x; q < kTmTok * kTC; q += kTmThreads) {
    const int rr = q / kTC, k = q % kTC;
    const int t = t0 + rr, c = c0 + k * kEl;
    if (t < S && c < C)
      *reinterpret_cast<uint4*>(out_tm + (int64_t)t * C + c) =
          *reinterpret_cast<const uint4*>(&sm.tm[rr][k * kEl]);
  }
}

// The backward from token-major dy in one pass: dx (channel-major) and the
// dw / db partials per (channel, 128-token block), without dpre in global
// memory.  The tile stages x over [t0 - 8, t0 + 136) and dy rows t0 .. t0 +
// 135, and marks the tokens whose successor list is exactly t + 1 .. t + K - 1
// with lags 1 .. K - 1 in CSR order (the inside of a node).  Thread (r, q)
// then slides over tokens 32 q .. 32 q + 31 + K - 1 of channel r: dpre of
// each (the K - 1 past its run are the next run's first tokens, computed
// again here) into a register window, its tokens' dw / db terms, and
// dx[t] = w[K-1] dpre[t] + sum_l w[K-1-l] dpre[t + l] once dpre[t + K - 1] is
// known.  A token with another successor list (a node's last tokens) adds
// the successors of its near chain (t + 1 .. t + near, inside its path) from
// the same registers, then walks the rest of its CSR list, recomputing each
// far successor's dpre from x and dy (a node's later children, far away in
// DFS order).  Per output the arithmetic and
// its order are those of conv_bwd_dpre4 + conv_bwd_dx4, so dx matches the
// channel-major kernels bit for bit; the four runs' dw / db terms are added in
// run order.
template <typename T>
struct TmBwdTile {
  TmTileR<T, kTmHalo> s;                 // x [t0 - 8, t0 + 136), dy rows t0 .. t0 + 135
  float red[kTmTok / kTmRun][kTmCh][kPartW];   // per run: dw / db terms
  uint32_t succ_plain[kTmTok / 32];      // bit j of word i: token t0 + 32 i + j
  uint8_t succ_info[kTmTok];             // per token: near chain length | 8 if far successors
};

// dpre of token u in tile channel r (c = c0 + r): the window through the
// predecessor table, dy from the staged rows or global memory.
template <int K, typename Tile, typename T>
__device__ __forceinline__ float dpre_any(const Tile& sm, const T* __restrict__ x,
                                          const T* __restrict__ dy_tm,
                                          const int32_t* __restrict__ pred, int C, int S, int c,
                                          int r, int t0, int u) {
  float xs[K];
  window_gather<K>(sm, x, pred, S, c, r, t0, u - t0, xs);
  float pre = sm.b[r];
#pragma unroll
  for (int m = 0; m < K; ++m) pre = fmaf(sm.w[r * K + K - 1 - m], xs[m], pre);
  const float g = u - t0 < Tile::kRows ? to_f32(sm.tm[u - t0][r])
                                       : to_f32(dy_tm[(int64_t)u * C + c]);
  return silu_grad(g, pre);
}

// The far part of dx[t]: the successor CSR entries after the first `near`
// (its near chain t + 1 .. t + near, whose terms the caller has added),
// each successor's dpre recomputed from x and dy.
template <int K, typename Tile, typename T>
__device__ __forceinline__ float dx_far(const Tile& sm, const T* __restrict__ x,
                                        const T* __restrict__ dy_tm,
                                        const int32_t* __restrict__ pred,
                                        const int32_t* __restrict__ sp,
                                        const int32_t* __restrict__ stok,
                                        const int32_t* __restrict__ slag, int C, int S, int c,
                                        int r, int t0, int t, int near, float s) {
  const float* wc = sm.w + r * K;
  const int e1 = sp[t + 1];
  for (int e = sp[t] + near; e < e1; ++e) {
    const int u = stok[e], l = slag[e];
    s = fmaf(wc[K - 1 - l], dpre_any<K>(sm, x, dy_tm, pred, C, S, c, r, t0, u), s);
  }
  return s;
}

template <typename T, int K>
__global__ void __launch_bounds__(kTmThreads)
conv_bwd_tm(int C, int S, const T* __restrict__ x, const float* __restrict__ w,
            const float* __restrict__ bias, const int32_t* __restrict__ pred,
            const int32_t* __restrict__ sp, const int32_t* __restrict__ stok,
            const int32_t* __restrict__ slag, const T* __restrict__ dy_tm, T* __restrict__ dx,
            float* __restrict__ part, int nb) {
  extern __shared__ __align__(16) uint8_t tm_smem[];
  using Tile = TmTileR<T, kTmHalo>;
  TmBwdTile<T>& bt = *reinterpret_cast<TmBwdTile<T>*>(tm_smem);
  Tile& sm = bt.s;
  constexpr int kEl = Tile::kEl, kTC = kTmCh / kEl;
  const int c0 = blockIdx.y * kTmCh, t0 = blockIdx.x * kTmTok;
  stage_x(sm, x, C, S, c0, t0);
  for (int q = threadIdx.x; q < Tile::kRows * kTC; q += kTmThreads) {
    const int rr = q / kTC, k = q % kTC;
    const int t = t0 + rr, c = c0 + k * kEl;
    const bool ok = t < S && c < C;
    cp_async16_zfill(&sm.tm[rr][k * kEl], ok ? dy_tm + (int64_t)t * C + c : dy_tm, ok);
  }
  stage_pred<K>(sm, pred, S, t0);
  asm volatile("cp.async.commit_group;" ::: "memory");
  stage_w<K>(sm, w, bias, C, c0);
  stage_plain<K>(sm, pred, S, t0);
  if (threadIdx.x < kTmTok) {
    // successor lists: the near chain (the leading entries (t + 1 + m, m + 1),
    // the tokens that follow t inside its path) and whether others follow.
    // A successor u of lag l is at least l tokens after t in DFS order, and
    // u = t + l only on the chain, so the chain's entries come first in the
    // CSR's token order.
    const int t = t0 + threadIdx.x;
    int near = 0;
    bool far = false;
    if (t < S) {
      const int e0 = sp[t], e1 = sp[t + 1];
      int su[K > 1 ? K - 1 : 1], sl[K > 1 ? K - 1 : 1];   // independent loads
#pragma unroll
      for (int m = 0; m < K - 1; ++m) {
        const bool in = e0 + m < e1;
        su[m] = in ? stok[e0 + m] : -1;
        sl[m] = in ? slag[e0 + m] : 0;
      }
      bool chain = true;
#pragma unroll
      for (int m = 0; m < K - 1; ++m) {
        chain = chain && su[m] == t + 1 + m && sl[m] == m + 1;
        near += chain;
      }
      far = e1 - e0 > near;
    }
    bt.succ_info[threadIdx.x] = (uint8_t)(near | (far ? 8 : 0));
    const bool pl = t < S && near == K - 1 && !far;
    const uint32_t bits = __ballot_sync(0xffffffffu, pl);
    if ((threadIdx.x & 31) == 0) bt.succ_plain[threadIdx.x >> 5] = bits;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int run = warp >> 1, r = (warp & 1) * 32 + lane, tq = run * kTmRun;
  const int c = min(c0 + r, C - 1);          // rows past C compute on row C - 1, never stored
  const uint32_t pb0 = sm.plain[run], pb1 = sm.plain[run + 1], sb = bt.succ_plain[run];
  float wr[K];
#pragma unroll
  for (int m = 0; m < K; ++m) wr[m] = sm.w[r * K + m];
  const float b0 = sm.b[r];
  float acc[kPartW];
#pragma unroll
  for (int j = 0; j < kPartW; ++j) acc[j] = 0.f;
  T* dxr = dx + (int64_t)(c0 + r) * S + t0 + tq;
  const bool row_live = c0 + r < C;
  const uint64_t pbits = pb0 | (uint64_t)pb1 << 32;
  // The run in chunks of 8 tokens (a loop that is not unrolled, so the state
  // carried across chunks bounds the registers): chunk ci computes dpre of
  // run tokens 8 ci .. 8 ci + 7 (chunk 4: only the K - 1 tokens past the
  // run), then dx of chunk ci - 1, whose successors' dpre are now known.
  // clean: every window and successor list of the run is plain (a run inside
  // one node, all tokens < S), no per-token branch.
  auto body = [&](auto clean) {
    constexpr bool kClean = decltype(clean)::value;
    float xp[8], dp[8];                      // the previous chunk's x and dpre
    ld_chunk<Tile, T>(sm, r, tq, xp);
    if (kEl == 4) ld_chunk<Tile, T>(sm, r, tq + 4, xp + 4);
#pragma unroll
    for (int i = 0; i < 8; ++i) dp[i] = 0.f;
#pragma unroll 1
    for (int ci = 0; ci <= kTmRun / 8; ++ci) {
      const int base = 8 * ci;
      float xc[8], dc[8];
      ld_chunk<Tile, T>(sm, r, kTmHalo + tq + base, xc);
      if (kEl == 4) ld_chunk<Tile, T>(sm, r, kTmHalo + tq + base + 4, xc + 4);
      const uint32_t cb = (uint32_t)(pbits >> base) & 0xffu;
      const bool last = ci == kTmRun / 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int tt = tq + base + i;
        if (last && i >= K - 1) {
          dc[i] = 0.f;
          continue;
        }
        float xs[K];
        if (kClean || (cb >> i & 1)) {
#pragma unroll
          for (int m = 0; m < K; ++m) xs[m] = i >= m ? xc[i - m] : xp[8 + i - m];
        } else {
          window_gather<K>(sm, x, pred, S, c, r, t0, tt, xs);
        }
        float pre = b0;
#pragma unroll
        for (int m = 0; m < K; ++m) pre = fmaf(wr[K - 1 - m], xs[m], pre);
        dc[i] = (kClean || t0 + tt < S) ? silu_grad(to_f32(sm.tm[tt][r]), pre) : 0.f;
        if (!last) {
#pragma unroll
          for (int jj = 0; jj < K; ++jj) acc[jj] += dc[i] * xs[K - 1 - jj];
          acc[8] += dc[i];
        }
      }
      if (ci > 0) {                          // dx of chunk ci - 1
        const int pbase = base - 8;
        const uint32_t sc = (sb >> pbase) & 0xffu;
        float dxv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (kClean || (sc >> i & 1)) {
            float sacc = wr[K - 1] * dp[i];
#pragma unroll
            for (int l = 1; l < K; ++l) sacc = fmaf(wr[K - 1 - l], i + l < 8 ? dp[i + l] : dc[i + l - 8], sacc);
            dxv[i] = sacc;
          } else if (t0 + tq + pbase + i < S) {
            // the near chain from registers, then the far successors
            const int info = bt.succ_info[tq + pbase + i], near = info & 7;
            float sacc = wr[K - 1] * dp[i];
#pragma unroll
            for (int l = 1; l < K; ++l)
              if (l <= near) sacc = fmaf(wr[K - 1 - l], i + l < 8 ? dp[i + l] : dc[i + l - 8], sacc);
            if (info & 8)
              sacc = dx_far<K>(sm, x, dy_tm, pred, sp, stok, slag, C, S, c, r, t0,
                               t0 + tq + pbase + i, near, sacc);
            dxv[i] = sacc;
          }
        }
        // whole 16-byte chunks (S % kEl == 0: live or dead as a whole)
#pragma unroll
        for (int h = 0; h < 8 / kEl; ++h) {
          if (row_live && (kClean || t0 + tq + pbase + h * kEl < S)) {
            uint4 v;
            T* e = reinterpret_cast<T*>(&v);
#pragma unroll
            for (int i = 0; i < kEl; ++i) e[i] = from_f32<T>(dxv[h * kEl + i]);
            *reinterpret_cast<uint4*>(dxr + pbase + h * kEl) = v;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xp[i] = xc[i];
        dp[i] = dc[i];
      }
    }
  };
  constexpr uint32_t kTail = (1u << (K - 1)) - 1u;
  if (pb0 == 0xffffffffu && (pb1 & kTail) == kTail && sb == 0xffffffffu)
    body(std::true_type());
  else
    body(std::false_type());
  // the run's dw / db terms, added over the four runs in order
#pragma unroll
  for (int j = 0; j < kPartW; ++j) bt.red[run][r][j] = acc[j];
  __syncthreads();
  for (int i = threadIdx.x; i < kTmCh * kPartW; i += kTmThreads) {
    const int rr = i / kPartW, j = i % kPartW;
    if (c0 + rr >= C) continue;
    float v = 0.f;
    if (j < K || j == 8) {
#pragma unroll
      for (int q = 0; q < kTmTok / kTmRun; ++q) v += bt.red[q][rr][j];
    }
    part[((int64_t)(c0 + rr) * nb + blockIdx.x) * kPartW + j] = v;
  }
}

inline bool quad_ok(int S, const void* a, const void* b, const void* c) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return S % 4 == 0 && al(a) && al(b) && al(c);
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

namespace {
bool tm_ok(int dtype, int C, int S, const void* a, const void* b, const void* c) {
  const int el = dtype == TT_F32 ? 4 : 8;   // elements per 16 bytes
  return C % 8 == 0 && S % el == 0 && tt::quad_ok(S, a, b, c);
}

// Launch a token-major tile kernel with its dynamic shared memory (Tile).
template <typename Tile, typename Kern, typename... Args>
int launch_tm(Kern kern, dim3 grid, cudaStream_t st, Args... args) {
  const int bytes = (int)sizeof(Tile);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return TT_ERR_CUDA;
  kern<<<grid, tt::kTmThreads, bytes, st>>>(args...);
  return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
}
}  // namespace

extern "C" int tt_tree_conv_fwd_ex(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                   const float* weight, const float* bias, const int32_t* pred,
                                   void* out, int32_t out_token_major, void* stream) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return TT_ERR_INVALID_ARG;
  if (C == 0 || S == 0) return TT_OK;
  if (!x || !weight || !out || (K > 1 && !pred)) return TT_ERR_INVALID_ARG;
  if (out_token_major && !tm_ok(dtype, C, S, x, out, out)) return TT_ERR_UNSUPPORTED;
  return tt::by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return tt::by_k(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      if (out_token_major) {
        dim3 g((S + tt::kTmTok - 1) / tt::kTmTok, (C + tt::kTmCh - 1) / tt::kTmCh);
        tt_count_launches(1);
        return launch_tm<tt::TmTile<T>>(tt::conv_fwd_tm<T, KK>, g, (cudaStream_t)stream, C, S, (const T*)x,
                            weight, bias, pred, (T*)out);
      }
      dim3 g((S + tt::kConvTok - 1) / tt::kConvTok, (C + tt::kConvCh - 1) / tt::kConvCh);
      tt::conv_fwd<T, KK><<<g, tt::kConvTok, 0, (cudaStream_t)stream>>>(
          C, S, (const T*)x, weight, bias, pred, (T*)out);
      tt_count_launches(1);
      return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
    });
  });
}

extern "C" int tt_tree_conv_fwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                const float* weight, const float* bias, const int32_t* pred,
                                void* out, void* stream) {
  return tt_tree_conv_fwd_ex(dtype, C, S, K, x, weight, bias, pred, out, 0, stream);
}

extern "C" int64_t tt_tree_conv_bwd_workspace_size(int32_t C, int32_t S, int32_t K) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return -1;
  // dpre, then the dw / db partials per (channel, block of 128 tokens: the
  // token-major kernels' blocks; the channel-major ones use 256-token blocks)
  const int64_t nb = ((int64_t)S + tt::kTmTok - 1) / tt::kTmTok;
  return (int64_t)C * S * 4 + (int64_t)C * nb * tt::kPartW * 4 + 256;
}

extern "C" int tt_tree_conv_bwd_ex(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                   const float* weight, const float* bias, const int32_t* pred,
                                   const int32_t* succ_ptr, const int32_t* succ_tok,
                                   const int32_t* succ_lag, const void* dout,
                                   int32_t dout_token_major, void* dx, float* dweight,
                                   float* dbias, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  if (C < 0 || S < 0 || K < 1 || K > 8) return TT_ERR_INVALID_ARG;
  if (C == 0 || S == 0) return TT_OK;
  if (!x || !weight || !dout || !dx || !dweight || !succ_ptr || (K > 1 && !pred))
    return TT_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < tt_tree_conv_bwd_workspace_size(C, S, K))
    return TT_ERR_WORKSPACE;
  if (dout_token_major && !(tm_ok(dtype, C, S, x, dout, dx) &&
                            (reinterpret_cast<uintptr_t>(workspace) & 15) == 0))
    return TT_ERR_UNSUPPORTED;
  return tt::by_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    cudaStream_t st = (cudaStream_t)stream;
    const int tok = dout_token_major ? tt::kTmTok : tt::kConvTok;
    const int nb = (S + tok - 1) / tok;
    float* dpre = static_cast<float*>(workspace);
    float* part = dpre + (int64_t)C * S;
    dim3 g(nb, (C + tt::kConvCh - 1) / tt::kConvCh);
    return tt::by_k(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      // the 4-token kernels also move dpre by 16 bytes
      const bool q4 = tt::quad_ok(S, x, dout, dx) &&
                      (reinterpret_cast<uintptr_t>(workspace) & 15) == 0;
      if (dout_token_major) {
        // dpre stays in shared memory: one pass to dx and the partials
        const int rc = launch_tm<tt::TmBwdTile<T>>(
            tt::conv_bwd_tm<T, KK>, dim3(nb, (C + tt::kTmCh - 1) / tt::kTmCh), st, C, S,
            (const T*)x, weight, bias, pred, succ_ptr, succ_tok, succ_lag, (const T*)dout, (T*)dx,
            part, nb);
        if (rc != TT_OK) return rc;
        tt::conv_bwd_dw_reduce<<<(C * tt::kPartW + 255) / 256, 256, 0, st>>>(C, K, nb, part,
                                                                           dweight, dbias);
        tt_count_launches(2);
        return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
      }
      if (q4)
        tt::conv_bwd_dpre4<T, KK><<<g, tt::kConvThr4, 0, st>>>(
            C, S, (const T*)x, weight, bias, pred, (const T*)dout, dpre, part, nb);
      else
        tt::conv_bwd_dpre<T, KK><<<g, tt::kConvTok, 0, st>>>(
            C, S, (const T*)x, weight, bias, pred, (const T*)dout, dpre, part, nb);
      tt::conv_bwd_dw_reduce<<<(C * tt::kPartW + 255) / 256, 256, 0, st>>>(C, K, nb, part,
                                                                         dweight, dbias);
      const dim3 gx((S + tt::kConvTok - 1) / tt::kConvTok, (C + tt::kConvCh - 1) / tt::kConvCh);
      if (q4)
        tt::conv_bwd_dx4<T, KK><<<gx, tt::kConvThr4, 0, st>>>(C, S, weight, dpre, succ_ptr,
                                                              succ_tok, succ_lag, (T*)dx);
      else
        tt::conv_bwd_dx<T, KK><<<gx, tt::kConvTok, 0, st>>>(C, S, weight, dpre, succ_ptr,
                                                            succ_tok, succ_lag, (T*)dx);
      tt_count_launches(3);
      return cudaGetLastError() == cudaSuccess ? (int)TT_OK : (int)TT_ERR_CUDA;
    });
  });
}

extern "C" int tt_tree_conv_bwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                                const float* weight, const float* bias, const int32_t* pred,
                                const int32_t* succ_ptr, const int32_t* succ_tok,
                                const int32_t* succ_lag, const void* dout, void* dx,
                                float* dweight, float* dbias, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  return tt_tree_conv_bwd_ex(dtype, C, S, K, x, weight, bias, pred, succ_ptr, succ_tok, succ_lag,
                             dout, 0, dx, dweight, dbias, workspace, workspace_bytes, stream);
}
