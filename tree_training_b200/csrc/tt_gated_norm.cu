// Fused gated RMSNorm of the GDN output (the per-node norm + gate of
// dfs_tree_forward.py:420-433, which runs the layer's Qwen3.5 gated norm,
// transformers models/qwen3_5_moe/modeling_qwen3_5_moe.py Qwen3_5MoeRMSNormGated):
//
//   y = x * rsqrt(mean(x^2) + eps) * w * silu(z),   silu(z) = z * sigmoid(z)
//
// over rows of D values (tokens x value heads, D = head_v_dim), in one pass
// each way instead of the module's five elementwise kernels.  Arithmetic is
// fp32 with one rounding at the end (the module rounds the normed value to
// the input type before the weight).  One warp per row: lane l holds the E =
// D / 32 values [E l, E l + E).  The backward recomputes the norm:
//   n = r x,  s = silu(z),  g = dy * w * s            (gradient of n)
//   dx = r g - x r^3 mean(x g)
//   dz = dy * n * w * sigmoid(z) * (1 + z (1 - sigmoid(z)))
//   dw = sum over rows of dy * n * s     (per-block partials [blocks, D], no atomics)
#include <algorithm>
#include <type_traits>

#include "tt_common.cuh"

namespace tt {
namespace gated_norm {
namespace {

constexpr int kWarps = 8;

template <typename T, int E>
__device__ __forceinline__ void load_e(const T* p, float (&v)[E]) {
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = to_f32(p[i]);
}

__device__ __forceinline__ float sigmoid(float z) { return 1.f / (1.f + expf(-z)); }

__device__ __forceinline__ float warp_sum(float a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  return a;
}

template <typename T, int E>
__global__ void __launch_bounds__(32 * kWarps)
gated_norm_fwd(int64_t rows, const T* __restrict__ x, const T* __restrict__ z,
               const float* __restrict__ w, float eps, T* __restrict__ y) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t o = row * D + E * lane;
  float v[E], g[E];
  load_e<T, E>(x + o, v);
  load_e<T, E>(z + o, g);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss = fmaf(v[i], v[i], ss);
  const float r = rsqrtf(warp_sum(ss) / D + eps);
  T out[E];
#pragma unroll
  for (int i = 0; i < E; ++i)
    out[i] = from_f32<T>(v[i] * r * w[E * lane + i] * (g[i] * sigmoid(g[i])));
#pragma unroll
  for (int i = 0; i < E; ++i) y[o + i] = out[i];
}

template <typename T, int E>
__global__ void __launch_bounds__(32 * kWarps)
gated_norm_bwd(int64_t rows, const T* __restrict__ x, const T* __restrict__ z,
               const float* __restrict__ w, float eps, const T* __restrict__ dy,
               T* __restrict__ dx, T* __restrict__ dz, float* __restrict__ dw_part) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float wt[E], dw[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    wt[i] = w[E * lane + i];
    dw[i] = 0.f;
  }
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const int64_t o = row * D + E * lane;
    float v[E], g[E], d[E];
    load_e<T, E>(x + o, v);
    load_e<T, E>(z + o, g);
    load_e<T, E>(dy + o, d);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss = fmaf(v[i], v[i], ss);
    const float r = rsqrtf(warp_sum(ss) / D + eps);
    float xg = 0.f;
    T dzo[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float sg = sigmoid(g[i]);
      const float s = g[i] * sg;
      const float n = v[i] * r;
      dw[i] = fmaf(d[i] * n, s, dw[i]);
      dzo[i] = from_f32<T>(d[i] * n * wt[i] * sg * (1.f + g[i] * (1.f - sg)));
      d[i] = d[i] * wt[i] * s;                 // now the gradient of n
      xg = fmaf(v[i], d[i], xg);
    }
    const float k = r * r * r * warp_sum(xg) / D;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      dz[o + i] = dzo[i];
      dx[o + i] = from_f32<T>(r * d[i] - v[i] * k);
    }
  }
  __shared__ float red[kWarps][D];
#pragma unroll
  for (int i = 0; i < E; ++i) red[warp][E * lane + i] = dw[i];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float a = 0.f;
    for (int q = 0; q < kWarps; ++q) a += red[q][c];
    dw_part[(int64_t)blockIdx.x * D + c] = a;
  }
}

template <typename F>
int dispatch(int dtype, int D, F f) {
  auto by_e = [&](auto tag) -> int {
    using T = decltype(tag);
    switch (D) {
      case 32: return f(T(), std::integral_constant<int, 1>());
      case 64: return f(T(), std::integral_constant<int, 2>());
      case 128: return f(T(), std::integral_constant<int, 4>());
      case 256: return f(T(), std::integral_constant<int, 8>());
      default: return TT_ERR_UNSUPPORTED;
    }
  };
  switch (dtype) {
    case TT_BF16: return by_e(__nv_bfloat16());
    case TT_F16: return by_e(__half());
    case TT_F32: return by_e(float());
    default: return TT_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace gated_norm
}  // namespace tt

extern "C" int tt_gated_rmsnorm_bwd_blocks(int64_t rows) {
  const int64_t want = (rows + tt::gated_norm::kWarps - 1) / tt::gated_norm::kWarps;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, 148 * 8));
}

extern "C" int tt_gated_rmsnorm_fwd(int dtype, int64_t rows, int32_t D, const void* x,
                                    const void* z, const float* weight, float eps, void* y,
                                    void* stream) {
  using namespace tt::gated_norm;
  if (rows < 0 || (rows > 0 && (!x || !z || !weight || !y))) return TT_ERR_INVALID_ARG;
  if (rows == 0) return TT_OK;
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  const int rc = dispatch(dtype, D, [&](auto tag, auto e) {
    using T = decltype(tag);
    constexpr int E = decltype(e)::value;
    gated_norm_fwd<T, E><<<grid, 32 * kWarps, 0, (cudaStream_t)stream>>>(
        rows, (const T*)x, (const T*)z, weight, eps, (T*)y);
    return (int)TT_OK;
  });
  if (rc != TT_OK) return rc;
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

extern "C" int tt_gated_rmsnorm_bwd(int dtype, int64_t rows, int32_t D, const void* x,
                                    const void* z, const float* weight, float eps,
                                    const void* dy, void* dx, void* dz, float* dw_part,
                                    int32_t blocks, void* stream) {
  using namespace tt::gated_norm;
  if (rows < 0 || blocks <= 0 ||
      (rows > 0 && (!x || !z || !weight || !dy || !dx || !dz || !dw_part)))
    return TT_ERR_INVALID_ARG;
  if (rows == 0) return TT_OK;
  const int rc = dispatch(dtype, D, [&](auto tag, auto e) {
    using T = decltype(tag);
    constexpr int E = decltype(e)::value;
    gated_norm_bwd<T, E><<<blocks, 32 * kWarps, 0, (cudaStream_t)stream>>>(
        rows, (const T*)x, (const T*)z, weight, eps, (const T*)dy, (T*)dx, (T*)dz, dw_part);
    return (int)TT_OK;
  });
  if (rc != TT_OK) return rc;
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
