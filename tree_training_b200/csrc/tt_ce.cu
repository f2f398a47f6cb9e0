// Cross-entropy over LM-head logits, fused with its gradient: one pass per row
// computes the log-sum-exp and the label's logit; with write_grad a second
// overwrites the row with  w * (softmax - onehot(label)),  the gradient of
// w * CE  with respect to the logits.  The caller's chunked linear + CE (the
// leaf-token loss of tree_grad_hybrid.py:533-535 / make_tree_loss_fn
// :546-558, without ever holding all [tokens, vocab] logits) runs the loss-only
// form in the forward and the gradient form on recomputed logits in the
// backward.
//
// One CTA per row, 512 threads.  The row is read twice (HBM- or L2-bound:
// 2 reads + 1 write of vocab x 2 bytes per token); the log-sum-exp uses a
// per-thread online max / rescaled sum, merged across the block.
#include <cfloat>

#include "tt_common.cuh"

namespace tt {
namespace ce {
namespace {

constexpr int kThreads = 512;

struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum merge(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
ce_fwd_grad(int V, T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels,
            const float* __restrict__ weights, int64_t ignore_index, float* __restrict__ loss,
            int write_grad) {
  const int row = blockIdx.x;
  T* x = logits + row * ld;
  const int64_t lab = labels[row];
  const bool ignored = lab == ignore_index || lab < 0 || lab >= V;
  const float w = ignored ? 0.f : weights[row];
  // pass 1: online max and rescaled sum of exponentials
  MaxSum a{-INFINITY, 0.f};
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = to_f32(x[i]);
    if (v > a.m) {
      a.s = a.s * __expf(a.m - v) + 1.f;
      a.m = v;
    } else {
      a.s += __expf(v - a.m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum b{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s, o)};
    a = merge(a, b);
  }
  __shared__ MaxSum red[kThreads / 32];
  __shared__ float s_lse, s_xl;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    MaxSum t = red[0];
    for (int i = 1; i < kThreads / 32; ++i) t = merge(t, red[i]);
    s_lse = t.m + logf(t.s);
    s_xl = ignored ? 0.f : to_f32(x[lab]);
    loss[row] = ignored ? 0.f : w * (s_lse - s_xl);
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = s_lse;
  // pass 2: the gradient, in place (every thread has read what it overwrites)
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float p = __expf(to_f32(x[i]) - lse);
    x[i] = from_f32<T>(w * (p - (i == lab ? 1.f : 0.f)));
  }
}

}  // namespace
}  // namespace ce
}  // namespace tt

extern "C" int tt_ce_fwd_grad(int dtype, int32_t n_rows, int32_t vocab, void* logits,
                              int64_t ld, const int64_t* labels, const float* weights,
                              int64_t ignore_index, float* loss, int write_grad, void* stream) {
  if (n_rows < 0 || vocab <= 0 || ld < vocab || (n_rows > 0 && (!logits || !labels ||
      !weights || !loss)))
    return TT_ERR_INVALID_ARG;
  if (n_rows == 0) return TT_OK;
  cudaStream_t st = (cudaStream_t)stream;
  using namespace tt::ce;
  switch (dtype) {
    case TT_BF16:
      ce_fwd_grad<__nv_bfloat16><<<n_rows, kThreads, 0, st>>>(
          vocab, (__nv_bfloat16*)logits, ld, labels, weights, ignore_index, loss, write_grad);
      break;
    case TT_F16:
      ce_fwd_grad<__half><<<n_rows, kThreads, 0, st>>>(vocab, (__half*)logits, ld, labels,
                                                       weights, ignore_index, loss, write_grad);
      break;
    case TT_F32:
      ce_fwd_grad<float><<<n_rows, kThreads, 0, st>>>(vocab, (float*)logits, ld, labels, weights,
                                                      ignore_index, loss, write_grad);
      break;
    default:
      return TT_ERR_UNSUPPORTED;
  }
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
