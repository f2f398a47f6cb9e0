// Fused attention prologue: per-head RMSNorm of q / k followed by the rotary
// embedding, in one pass (transformers' Qwen3 attention, models/qwen3/
// modeling_qwen3.py lines 263-268: q_norm / k_norm then apply_rotary_pos_emb,
// with the tree's depth-based position ids already folded into cos / sin).
//
//   n = x * rsqrt(mean(x^2) + eps) * w
//   y = n * cos + rotate_half(n) * sin,   rotate_half(n) = [-n2, n1]
//
// Arithmetic is fp32 throughout (the unfused torch path rounds n to the input
// type before the weight and the rotation).  One warp per (token, head) row of
// D = 32 E values: lane l holds [E l, E l + E), so the rotation partner
// (d +- D/2) sits in lane l ^ 16.  The backward recomputes n from x:
//   dn = dy * cos + rotate_half^T(dy * sin),  rotate_half^T(z) = [z2, -z1]
//   g = dn * w ;  dx = r g - x r^3 mean(x g) ;  dw = sum over rows of dn x r
// with dw summed per block into a [blocks, D] array (no atomics; the caller
// adds the rows).
#include <algorithm>
#include <type_traits>

#include "tt_common.cuh"

namespace tt {
namespace prologue {
namespace {

constexpr int kWarps = 8;

template <typename T, int E>
__device__ __forceinline__ void load_row(const T* p, float (&v)[E]) {
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = to_f32(p[i]);
}

template <typename T, int E>
__global__ void __launch_bounds__(32 * kWarps)
qk_norm_rope_fwd(int64_t rows, int H, const T* __restrict__ x, const float* __restrict__ w,
                 const T* __restrict__ cos_, const T* __restrict__ sin_, float eps,
                 T* __restrict__ y) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t tok = row / H;
  float v[E], c[E], s[E], wt[E];
  load_row<T, E>(x + row * D + E * lane, v);
  load_row<T, E>(cos_ + tok * D + E * lane, c);
  load_row<T, E>(sin_ + tok * D + E * lane, s);
#pragma unroll
  for (int i = 0; i < E; ++i) wt[i] = w[E * lane + i];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / D + eps);
  const float sign = lane < 16 ? -1.f : 1.f;   // rotate_half: first half takes -n2
  T out[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const float n = v[i] * r * wt[i];
    const float partner = __shfl_xor_sync(0xffffffffu, n, 16);
    out[i] = from_f32<T>(n * c[i] + sign * partner * s[i]);
  }
#pragma unroll
  for (int i = 0; i < E; ++i) y[row * D + E * lane + i] = out[i];
}

template <typename T, int E>
__global__ void __launch_bounds__(32 * kWarps)
qk_norm_rope_bwd(int64_t rows, int H, const T* __restrict__ x, const float* __restrict__ w,
                 const T* __restrict__ cos_, const T* __restrict__ sin_, float eps,
                 const T* __restrict__ dy, T* __restrict__ dx, float* __restrict__ dw_part) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float dw[E];
#pragma unroll
  for (int i = 0; i < E; ++i) dw[i] = 0.f;
  float wt[E];
#pragma unroll
  for (int i = 0; i < E; ++i) wt[i] = w[E * lane + i];
  const float sign = lane < 16 ? 1.f : -1.f;   // rotate_half^T: first half takes +z2
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const int64_t tok = row / H;
    float v[E], c[E], s[E], g[E];
    load_row<T, E>(x + row * D + E * lane, v);
    load_row<T, E>(cos_ + tok * D + E * lane, c);
    load_row<T, E>(sin_ + tok * D + E * lane, s);
    load_row<T, E>(dy + row * D + E * lane, g);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / D + eps);
    float xg = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float zs = g[i] * s[i];
      const float partner = __shfl_xor_sync(0xffffffffu, zs, 16);
      const float dn = g[i] * c[i] + sign * partner;     // gradient of the normed value
      dw[i] = fmaf(dn, v[i] * r, dw[i]);
      g[i] = dn * wt[i];
      xg = fmaf(v[i], g[i], xg);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) xg += __shfl_xor_sync(0xffffffffu, xg, o);
    const float k = r * r * r * xg / D;
#pragma unroll
    for (int i = 0; i < E; ++i) dx[row * D + E * lane + i] = from_f32<T>(r * g[i] - v[i] * k);
  }
  // per-block dw partial: warps summed in a fixed order
  __shared__ float red[kWarps][D];
#pragma unroll
  for (int i = 0; i < E; ++i) red[warp][E * lane + i] = dw[i];
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int q = 0; q < kWarps; ++q) a += red[q][d];
    dw_part[(int64_t)blockIdx.x * D + d] = a;
  }
}

template <typename T, typename F>
int dispatch_e(int D, F f) {
  switch (D) {
    case 64: return f(std::integral_constant<int, 2>());
    case 128: return f(std::integral_constant<int, 4>());
    case 256: return f(std::integral_constant<int, 8>());
    default: return TT_ERR_UNSUPPORTED;
  }
}

template <typename F>
int dispatch_t(int dtype, F f) {
  switch (dtype) {
    case TT_BF16: return f(__nv_bfloat16());
    case TT_F16: return f(__half());
    case TT_F32: return f(float());
    default: return TT_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace prologue
}  // namespace tt

extern "C" int tt_qk_norm_rope_bwd_blocks(int64_t rows) {
  const int64_t want = (rows + tt::prologue::kWarps - 1) / tt::prologue::kWarps;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, 148 * 8));
}

extern "C" int tt_qk_norm_rope_fwd(int dtype, int64_t n_tok, int32_t H, int32_t D, const void* x,
                                   const float* weight, const void* cos_, const void* sin_,
                                   float eps, void* y, void* stream) {
  using namespace tt::prologue;
  if (n_tok < 0 || H <= 0 || (n_tok > 0 && (!x || !weight || !cos_ || !sin_ || !y)))
    return TT_ERR_INVALID_ARG;
  const int64_t rows = n_tok * H;
  if (rows == 0) return TT_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((rows + kWarps - 1) / kWarps);
  int rc = dispatch_t(dtype, [&](auto tag) {
    using T = decltype(tag);
    return dispatch_e<T>(D, [&](auto e) {
      constexpr int E = decltype(e)::value;
      qk_norm_rope_fwd<T, E><<<grid, 32 * kWarps, 0, st>>>(rows, H, (const T*)x, weight,
                                                            (const T*)cos_, (const T*)sin_, eps,
                                                            (T*)y);
      return (int)TT_OK;
    });
  });
  if (rc != TT_OK) return rc;
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

extern "C" int tt_qk_norm_rope_bwd(int dtype, int64_t n_tok, int32_t H, int32_t D, const void* x,
                                   const float* weight, const void* cos_, const void* sin_,
                                   float eps, const void* dy, void* dx, float* dw_part,
                                   int32_t blocks, void* stream) {
  using namespace tt::prologue;
  if (n_tok < 0 || H <= 0 || blocks <= 0 ||
      (n_tok > 0 && (!x || !weight || !cos_ || !sin_ || !dy || !dx || !dw_part)))
    return TT_ERR_INVALID_ARG;
  const int64_t rows = n_tok * H;
  if (rows == 0) return TT_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = dispatch_t(dtype, [&](auto tag) {
    using T = decltype(tag);
    return dispatch_e<T>(D, [&](auto e) {
      constexpr int E = decltype(e)::value;
      qk_norm_rope_bwd<T, E><<<blocks, 32 * kWarps, 0, st>>>(
          rows, H, (const T*)x, weight, (const T*)cos_, (const T*)sin_, eps, (const T*)dy,
          (T*)dx, dw_part);
      return (int)TT_OK;
    });
  });
  if (rc != TT_OK) return rc;
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
