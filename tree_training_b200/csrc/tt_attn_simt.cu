// Exact tree attention on CUDA cores (fp32 FMA, fp32 softmax).
//
// This is the fp32 path (the reference's config-1 dtype, max_rel 1e-4) and
// the in-library cross-check of the tcgen05 path.  Same math as the SDPA call
// the reference makes (TF/integrations/sdpa_attention.py:92-101) with the
// dense mask of dfs_tree_forward.py:548-550 replaced by key intervals.
//
// Layout: 64-row query tiles x 64-key tiles; 4 threads per row (or key), each
// owning head dims d = slice + 4*i so the 4 threads of a row read consecutive
// shared-memory words.  No atomics: dK/dV and dQ are separate passes driven
// by the per-kv-tile and per-q-tile work lists.
#include <cfloat>
#include <climits>

#include "tt_common.cuh"

namespace tt {
namespace {

constexpr int kBQ = 64;
constexpr int kBK = 64;
constexpr int kTPR = 4;
constexpr int kThreads = kBQ * kTPR;

__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
attn_fwd_simt(int n_q, int n_kv, int rep, const T* __restrict__ q, int64_t q_st, int64_t q_sh,
              const T* __restrict__ k, int64_t k_st, int64_t k_sh, const T* __restrict__ v,
              int64_t v_st, int64_t v_sh, const int32_t* __restrict__ kv_lo,
              const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ fwd_ptr,
              const int32_t* __restrict__ fwd_list, float scale, T* __restrict__ out,
              float* __restrict__ lse) {
  constexpr int DPT = D / kTPR;
  extern __shared__ float smem[];
  float* sK = smem;
  float* sV = sK + kBK * D;
  int32_t* sLo = reinterpret_cast<int32_t*>(sV + kBK * D);
  int32_t* sHi = sLo + kBK;

  const int qt = blockIdx.x, h = blockIdx.y, hq = gridDim.y;
  const int hk = h / rep;
  const int tid = threadIdx.x, r = tid / kTPR, sl = tid % kTPR;
  const int row = qt * kBQ + r;

  float qr[DPT], o[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    qr[i] = row < n_q ? to_f32(q[row * q_st + h * q_sh + sl + kTPR * i]) * scale : 0.f;
    o[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int e0 = fwd_ptr[qt], e1 = fwd_ptr[qt + 1];
  for (int e = e0; e < e1; ++e) {
    const int kt = fwd_list[e] >> 1;
    __syncthreads();
    for (int idx = tid; idx < kBK * D; idx += kThreads) {
      const int jj = idx / D, d = idx % D, j = kt * kBK + jj;
      sK[idx] = j < n_kv ? to_f32(k[j * k_st + hk * k_sh + d]) : 0.f;
      sV[idx] = j < n_kv ? to_f32(v[j * v_st + hk * v_sh + d]) : 0.f;
    }
    for (int jj = tid; jj < kBK; jj += kThreads) {
      const int j = kt * kBK + jj;
      sLo[jj] = j < n_kv ? kv_lo[j] : 0;
      sHi[jj] = j < n_kv ? kv_hi[j] : 0;
    }
    __syncthreads();
    float s[kBK];
    float mt = -INFINITY;
#pragma unroll 8
    for (int jj = 0; jj < kBK; ++jj) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < DPT; ++i) acc = fmaf(qr[i], sK[jj * D + sl + kTPR * i], acc);
      acc = quad_sum(acc);
      s[jj] = visible(sLo[jj], sHi[jj], row) ? acc : -INFINITY;
      mt = fmaxf(mt, s[jj]);
    }
    const float mn = fmaxf(m, mt);
    if (mn == -INFINITY) continue;
    const float alpha = expf(m - mn);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < DPT; ++i) o[i] *= alpha;
#pragma unroll 4
    for (int jj = 0; jj < kBK; ++jj) {
      const float p = expf(s[jj] - mn);
      l += p;
#pragma unroll
      for (int i = 0; i < DPT; ++i) o[i] = fmaf(p, sV[jj * D + sl + kTPR * i], o[i]);
    }
    m = mn;
  }
  if (row < n_q) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < DPT; ++i)
      out[(int64_t)row * hq * D + h * D + sl + kTPR * i] = from_f32<T>(o[i] * inv);
    if (sl == 0) lse[(int64_t)h * lse_ld(n_q) + row] = l > 0.f ? m + logf(l) : INFINITY;
  }
}

// delta[h, i] = sum_d O[i,h,d] * dO[i,h,d]   (one warp per (row, head))
template <typename T>
__global__ void attn_bwd_delta(int n_q, int hq, int D, const T* __restrict__ out,
                               const T* __restrict__ dout, int64_t do_st, int64_t do_sh,
                               float* __restrict__ delta) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int ld = lse_ld(n_q);
  if (w >= ld * hq) return;
  const int i = w / hq, h = w % hq;
  float acc = 0.f;
  if (i < n_q)
    for (int d = lane; d < D; d += 32)
    acc = fmaf(to_f32(out[(int64_t)i * hq * D + h * D + d]), to_f32(dout[i * do_st + h * do_sh + d]),
               acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[(int64_t)h * ld + i] = acc;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dkdv_simt(int n_q, int n_kv, int hq, int rep, const T* __restrict__ q, int64_t q_st,
                   int64_t q_sh, const T* __restrict__ k, int64_t k_st, int64_t k_sh,
                   const T* __restrict__ v, int64_t v_st, int64_t v_sh, const T* __restrict__ dout,
                   int64_t do_st, int64_t do_sh, const float* __restrict__ lse,
                   const float* __restrict__ delta, const int32_t* __restrict__ kv_lo,
                   const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ bwd_ptr,
                   const int32_t* __restrict__ bwd_list, float scale, T* __restrict__ dk,
                   int64_t dk_st, int64_t dk_sh, T* __restrict__ dv, int64_t dv_st,
                   int64_t dv_sh) {
  constexpr int DPT = D / kTPR;
  extern __shared__ float smem[];
  float* sQ = smem;
  float* sDO = sQ + kBQ * D;
  float* sLse = sDO + kBQ * D;
  float* sDel = sLse + kBQ;

  const int kt = blockIdx.x, hk = blockIdx.y;
  const int tid = threadIdx.x, jj = tid / kTPR, sl = tid % kTPR;
  const int j = kt * kBK + jj;
  const bool jv = j < n_kv;
  const int lo = jv ? kv_lo[j] : 0, hi = jv ? kv_hi[j] : 0;
  float kr[DPT], vr[DPT], gk[DPT], gv[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    kr[i] = jv ? to_f32(k[j * k_st + hk * k_sh + sl + kTPR * i]) : 0.f;
    vr[i] = jv ? to_f32(v[j * v_st + hk * v_sh + sl + kTPR * i]) : 0.f;
    gk[i] = 0.f;
    gv[i] = 0.f;
  }
  const int e0 = bwd_ptr[kt], e1 = bwd_ptr[kt + 1];
  for (int hh = 0; hh < rep; ++hh) {
    const int h = hk * rep + hh;
    for (int e = e0; e < e1; ++e) {
      const int qt = bwd_list[e] >> 1;
      __syncthreads();
      for (int idx = tid; idx < kBQ * D; idx += kThreads) {
        const int rr = idx / D, d = idx % D, row = qt * kBQ + rr;
        sQ[idx] = row < n_q ? to_f32(q[row * q_st + h * q_sh + d]) : 0.f;
        sDO[idx] = row < n_q ? to_f32(dout[row * do_st + h * do_sh + d]) : 0.f;
      }
      for (int rr = tid; rr < kBQ; rr += kThreads) {
        const int row = qt * kBQ + rr;
        sLse[rr] = row < n_q ? lse[(int64_t)h * lse_ld(n_q) + row] : INFINITY;
        sDel[rr] = row < n_q ? delta[(int64_t)h * lse_ld(n_q) + row] : 0.f;
      }
      __syncthreads();
#pragma unroll 2
      for (int rr = 0; rr < kBQ; ++rr) {
        const int row = qt * kBQ + rr;
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int i = 0; i < DPT; ++i) {
          s = fmaf(sQ[rr * D + sl + kTPR * i], kr[i], s);
          dp = fmaf(sDO[rr * D + sl + kTPR * i], vr[i], dp);
        }
        s = quad_sum(s);
        dp = quad_sum(dp);
        const float p = visible(lo, hi, row) ? expf(s * scale - sLse[rr]) : 0.f;
        const float ds = p * (dp - sDel[rr]);
#pragma unroll
        for (int i = 0; i < DPT; ++i) {
          gv[i] = fmaf(p, sDO[rr * D + sl + kTPR * i], gv[i]);
          gk[i] = fmaf(ds, sQ[rr * D + sl + kTPR * i], gk[i]);
        }
      }
    }
  }
  if (jv) {
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      dk[j * dk_st + hk * dk_sh + sl + kTPR * i] = from_f32<T>(gk[i] * scale);
      dv[j * dv_st + hk * dv_sh + sl + kTPR * i] = from_f32<T>(gv[i]);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
attn_bwd_dq_simt(int n_q, int n_kv, int rep, const T* __restrict__ q, int64_t q_st, int64_t q_sh,
                 const T* __restrict__ k, int64_t k_st, int64_t k_sh, const T* __restrict__ v,
                 int64_t v_st, int64_t v_sh, const T* __restrict__ dout, int64_t do_st,
                 int64_t do_sh, const float* __restrict__ lse, const float* __restrict__ delta,
                 const int32_t* __restrict__ kv_lo, const int32_t* __restrict__ kv_hi,
                 const int32_t* __restrict__ fwd_ptr, const int32_t* __restrict__ fwd_list,
                 float scale, T* __restrict__ dq, int64_t dq_st, int64_t dq_sh) {
  constexpr int DPT = D / kTPR;
  extern __shared__ float smem[];
  float* sK = smem;
  float* sV = sK + kBK * D;
  int32_t* sLo = reinterpret_cast<int32_t*>(sV + kBK * D);
  int32_t* sHi = sLo + kBK;

  const int qt = blockIdx.x, h = blockIdx.y;
  const int hk = h / rep;
  const int tid = threadIdx.x, r = tid / kTPR, sl = tid % kTPR;
  const int row = qt * kBQ + r;
  const bool rv = row < n_q;
  float qr[DPT], dor[DPT], g[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    qr[i] = rv ? to_f32(q[row * q_st + h * q_sh + sl + kTPR * i]) : 0.f;
    dor[i] = rv ? to_f32(dout[row * do_st + h * do_sh + sl + kTPR * i]) : 0.f;
    g[i] = 0.f;
  }
  const float lrow = rv ? lse[(int64_t)h * lse_ld(n_q) + row] : INFINITY;
  const float drow = rv ? delta[(int64_t)h * lse_ld(n_q) + row] : 0.f;
  const int e0 = fwd_ptr[qt], e1 = fwd_ptr[qt + 1];
  for (int e = e0; e < e1; ++e) {
    const int kt = fwd_list[e] >> 1;
    __syncthreads();
    for (int idx = tid; idx < kBK * D; idx += kThreads) {
      const int jj = idx / D, d = idx % D, j = kt * kBK + jj;
      sK[idx] = j < n_kv ? to_f32(k[j * k_st + hk * k_sh + d]) : 0.f;
      sV[idx] = j < n_kv ? to_f32(v[j * v_st + hk * v_sh + d]) : 0.f;
    }
    for (int jj = tid; jj < kBK; jj += kThreads) {
      const int j = kt * kBK + jj;
      sLo[jj] = j < n_kv ? kv_lo[j] : 0;
      sHi[jj] = j < n_kv ? kv_hi[j] : 0;
    }
    __syncthreads();
#pragma unroll 2
    for (int jj = 0; jj < kBK; ++jj) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int i = 0; i < DPT; ++i) {
        s = fmaf(qr[i], sK[jj * D + sl + kTPR * i], s);
        dp = fmaf(dor[i], sV[jj * D + sl + kTPR * i], dp);
      }
      s = quad_sum(s);
      dp = quad_sum(dp);
      const float p = visible(sLo[jj], sHi[jj], row) ? expf(s * scale - lrow) : 0.f;
      const float ds = p * (dp - drow);
#pragma unroll
      for (int i = 0; i < DPT; ++i) g[i] = fmaf(ds, sK[jj * D + sl + kTPR * i], g[i]);
    }
  }
  if (rv) {
#pragma unroll
    for (int i = 0; i < DPT; ++i) dq[row * dq_st + h * dq_sh + sl + kTPR * i] = from_f32<T>(g[i] * scale);
  }
}

// ---- dense mask -> key intervals -------------------------------------------
constexpr int kMaskCols = 256;
constexpr int kMaskRows = 256;

template <typename M>
__device__ __forceinline__ int mask_class(M x);  // 1 visible, 0 masked, -1 not a tree mask value
template <>
__device__ __forceinline__ int mask_class<uint8_t>(uint8_t x) { return x != 0; }
template <>
__device__ __forceinline__ int mask_class<float>(float x) {
  return x == 0.f ? 1 : (x < -1e30f ? 0 : -1);
}
template <>
__device__ __forceinline__ int mask_class<__nv_bfloat16>(__nv_bfloat16 x) {
  return mask_class<float>(__bfloat162float(x));
}
template <>
__device__ __forceinline__ int mask_class<__half>(__half x) {
  const float f = __half2float(x);
  return f == 0.f ? 1 : (f <= -65504.f ? 0 : -1);
}

__global__ void mask_init(int n_kv, int32_t* lo, int32_t* hi) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n_kv) {
    lo[j] = INT_MAX;
    hi[j] = INT_MIN;
  }
}

template <typename M>
__global__ void mask_span(int n_q, int n_kv, const M* __restrict__ mask, int64_t sq, int64_t skv,
                          int32_t* lo, int32_t* hi, int32_t* status) {
  const int j = blockIdx.x * kMaskCols + threadIdx.x;
  if (j >= n_kv) return;
  const int i0 = blockIdx.y * kMaskRows, i1 = min(n_q, i0 + kMaskRows);
  int first = INT_MAX, last = INT_MIN;
  for (int i = i0; i < i1; ++i) {
    const int c = mask_class<M>(mask[i * sq + j * skv]);
    if (c < 0) set_status(status, TT_ERR_NOT_INTERVAL);
    if (c > 0) {
      first = min(first, i);
      last = i;
    }
  }
  if (first != INT_MAX) {
    atomicMin(lo + j, first);
    atomicMax(hi + j, last + 1);
  }
}

template <typename M>
__global__ void mask_verify(int n_q, int n_kv, const M* __restrict__ mask, int64_t sq,
                            int64_t skv, const int32_t* lo, const int32_t* hi,
                            int32_t* status) {
  const int j = blockIdx.x * kMaskCols + threadIdx.x;
  if (j >= n_kv) return;
  const int a = max(lo[j], blockIdx.y * kMaskRows);
  const int b = min(hi[j], min(n_q, (int)(blockIdx.y + 1) * kMaskRows));
  for (int i = a; i < b; ++i)
    if (mask_class<M>(mask[i * sq + j * skv]) != 1) set_status(status, TT_ERR_NOT_INTERVAL);
}

__global__ void mask_finalize(int n_kv, int32_t* lo, int32_t* hi) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n_kv && lo[j] == INT_MAX) {
    lo[j] = 0;
    hi[j] = 0;
  }
}

template <typename M>
int launch_mask(int n_q, int n_kv, const void* mask, int64_t sq, int64_t skv, int32_t* lo,
                int32_t* hi, int32_t* status, cudaStream_t st) {
  const int b1 = (n_kv + 255) / 256;
  mask_init<<<b1, 256, 0, st>>>(n_kv, lo, hi);
  dim3 g((n_kv + kMaskCols - 1) / kMaskCols, (n_q + kMaskRows - 1) / kMaskRows);
  mask_span<M><<<g, kMaskCols, 0, st>>>(n_q, n_kv, (const M*)mask, sq, skv, lo, hi, status);
  mask_verify<M><<<g, kMaskCols, 0, st>>>(n_q, n_kv, (const M*)mask, sq, skv, lo, hi, status);
  mask_finalize<<<b1, 256, 0, st>>>(n_kv, lo, hi);
  tt_count_launches(4);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

__global__ void lse_fill_pad(int n_q, int hq, float* lse) {
  const int ld = lse_ld(n_q), pad = ld - n_q;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx < pad * hq) lse[(int64_t)(idx / pad) * ld + n_q + idx % pad] = INFINITY;
}

template <typename T, int D>
int launch_fwd(int n_q, int n_kv, int hq, int hkv, const void* q, int64_t q_st, int64_t q_sh,
               const void* k, int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
               int64_t v_sh, const int32_t* lo, const int32_t* hi, const int32_t* fp,
               const int32_t* fl, float scale, void* out, float* lse, cudaStream_t st) {
  const size_t smem = 2 * kBK * D * sizeof(float) + 2 * kBK * sizeof(int32_t);
  auto kern = attn_fwd_simt<T, D>;
  TT_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((n_q + kBQ - 1) / kBQ, hq);
  kern<<<grid, kThreads, smem, st>>>(n_q, n_kv, hq / hkv, (const T*)q, q_st, q_sh, (const T*)k,
                                     k_st, k_sh, (const T*)v, v_st, v_sh, lo, hi, fp, fl, scale,
                                     (T*)out, lse);
  const int pad = lse_ld(n_q) - n_q;
  if (pad > 0) lse_fill_pad<<<(pad * hq + 255) / 256, 256, 0, st>>>(n_q, hq, lse);
  tt_count_launches(pad > 0 ? 2 : 1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

template <typename T, int D>
int launch_bwd(int n_q, int n_kv, int hq, int hkv, const void* q, int64_t q_st, int64_t q_sh,
               const void* k, int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
               int64_t v_sh, const void* out, const void* dout, int64_t do_st, int64_t do_sh,
               const float* lse, const int32_t* lo, const int32_t* hi, const int32_t* fp,
               const int32_t* fl, const int32_t* bp, const int32_t* bl, float scale, void* dq,
               int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
               int64_t dv_st, int64_t dv_sh, float* delta, int phases, cudaStream_t st) {
  const int rep = hq / hkv;
  const int warps = lse_ld(n_q) * hq;
  int launches = 0;
  if (warps > 0 && (phases & TT_BWD_PREP)) {
    ++launches;
    attn_bwd_delta<T><<<(warps + 7) / 8, 256, 0, st>>>(n_q, hq, D, (const T*)out, (const T*)dout,
                                                        do_st, do_sh, delta);
  }
  const size_t smem_kv = 2 * kBQ * D * sizeof(float) + 2 * kBQ * sizeof(float);
  auto kkv = attn_bwd_dkdv_simt<T, D>;
  TT_CUDA_OK(cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv));
  dim3 gkv((n_kv + kBK - 1) / kBK, hkv);
  if (n_kv > 0 && (phases & TT_BWD_DKDV)) {
    ++launches;
    kkv<<<gkv, kThreads, smem_kv, st>>>(n_q, n_kv, hq, rep, (const T*)q, q_st, q_sh, (const T*)k,
                                        k_st, k_sh, (const T*)v, v_st, v_sh, (const T*)dout, do_st,
                                        do_sh, lse, delta, lo, hi, bp, bl, scale, (T*)dk, dk_st,
                                        dk_sh, (T*)dv, dv_st, dv_sh);
  }
  const size_t smem_q = 2 * kBK * D * sizeof(float) + 2 * kBK * sizeof(int32_t);
  auto kq = attn_bwd_dq_simt<T, D>;
  TT_CUDA_OK(cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q));
  dim3 gq((n_q + kBQ - 1) / kBQ, hq);
  if (n_q > 0 && (phases & TT_BWD_DQ)) {
    ++launches;
    kq<<<gq, kThreads, smem_q, st>>>(n_q, n_kv, rep, (const T*)q, q_st, q_sh, (const T*)k, k_st,
                                     k_sh, (const T*)v, v_st, v_sh, (const T*)dout, do_st, do_sh,
                                     lse, delta, lo, hi, fp, fl, scale, (T*)dq, dq_st, dq_sh);
  }
  tt_count_launches(launches);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

template <int D>
int dispatch_fwd_dtype(int dtype, int n_q, int n_kv, int hq, int hkv, const void* q, int64_t a,
                       int64_t b, const void* k, int64_t c, int64_t d, const void* v, int64_t e,
                       int64_t f, const int32_t* lo, const int32_t* hi, const int32_t* fp,
                       const int32_t* fl, float scale, void* out, float* lse, cudaStream_t st) {
  switch (dtype) {
    case TT_F32:
      return launch_fwd<float, D>(n_q, n_kv, hq, hkv, q, a, b, k, c, d, v, e, f, lo, hi, fp, fl,
                                  scale, out, lse, st);
    case TT_BF16:
      return launch_fwd<__nv_bfloat16, D>(n_q, n_kv, hq, hkv, q, a, b, k, c, d, v, e, f, lo, hi,
                                          fp, fl, scale, out, lse, st);
    case TT_F16:
      return launch_fwd<__half, D>(n_q, n_kv, hq, hkv, q, a, b, k, c, d, v, e, f, lo, hi, fp, fl,
                                   scale, out, lse, st);
    default:
      return TT_ERR_UNSUPPORTED;
  }
}

template <int D, typename... Args>
int dispatch_bwd_dtype(int dtype, Args... args) {
  switch (dtype) {
    case TT_F32: return launch_bwd<float, D>(args...);
    case TT_BF16: return launch_bwd<__nv_bfloat16, D>(args...);
    case TT_F16: return launch_bwd<__half, D>(args...);
    default: return TT_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace tt

int tt_launch_attn_fwd_simt(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                            int32_t D, const void* q, int64_t q_st, int64_t q_sh, const void* k,
                            int64_t k_st, int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                            const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                            const int32_t* fwd_list, float scale, void* out, float* lse,
                            cudaStream_t st) {
  if (n_q == 0) return TT_OK;
  switch (D) {
    case 32: return tt::dispatch_fwd_dtype<32>(dtype, n_q, n_kv, hq, hkv, q, q_st, q_sh, k, k_st, k_sh, v, v_st, v_sh, kv_lo, kv_hi, fwd_ptr, fwd_list, scale, out, lse, st);
    case 64: return tt::dispatch_fwd_dtype<64>(dtype, n_q, n_kv, hq, hkv, q, q_st, q_sh, k, k_st, k_sh, v, v_st, v_sh, kv_lo, kv_hi, fwd_ptr, fwd_list, scale, out, lse, st);
    case 128: return tt::dispatch_fwd_dtype<128>(dtype, n_q, n_kv, hq, hkv, q, q_st, q_sh, k, k_st, k_sh, v, v_st, v_sh, kv_lo, kv_hi, fwd_ptr, fwd_list, scale, out, lse, st);
    default: return TT_ERR_UNSUPPORTED;
  }
}

int tt_launch_attn_bwd_simt(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                            int32_t D, const void* q, int64_t q_st, int64_t q_sh, const void* k,
                            int64_t k_st, int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                            const void* out, const void* dout, int64_t do_st, int64_t do_sh,
                            const float* lse, const int32_t* kv_lo, const int32_t* kv_hi,
                            const int32_t* fwd_ptr, const int32_t* fwd_list,
                            const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
                            void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st,
                            int64_t dk_sh, void* dv, int64_t dv_st, int64_t dv_sh, float* delta,
                            int phases, cudaStream_t st) {
#define TT_BWD_ARGS                                                                          \
  n_q, n_kv, hq, hkv, q, q_st, q_sh, k, k_st, k_sh, v, v_st, v_sh, out, dout, do_st, do_sh, lse, \
      kv_lo, kv_hi, fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh, dk, dk_st,    \
      dk_sh, dv, dv_st, dv_sh, delta, phases, st
  switch (D) {
    case 32: return tt::dispatch_bwd_dtype<32>(dtype, TT_BWD_ARGS);
    case 64: return tt::dispatch_bwd_dtype<64>(dtype, TT_BWD_ARGS);
    case 128: return tt::dispatch_bwd_dtype<128>(dtype, TT_BWD_ARGS);
    default: return TT_ERR_UNSUPPORTED;
  }
#undef TT_BWD_ARGS
}

int tt_launch_mask_to_intervals(int mask_dtype, int32_t n_q, int32_t n_kv, const void* mask,
                                int64_t sq, int64_t skv, int32_t* lo, int32_t* hi,
                                int32_t* status, cudaStream_t st) {
  if (n_kv == 0) return TT_OK;
  switch (mask_dtype) {
    case TT_U8: return tt::launch_mask<uint8_t>(n_q, n_kv, mask, sq, skv, lo, hi, status, st);
    case TT_F32: return tt::launch_mask<float>(n_q, n_kv, mask, sq, skv, lo, hi, status, st);
    case TT_BF16: return tt::launch_mask<__nv_bfloat16>(n_q, n_kv, mask, sq, skv, lo, hi, status, st);
    case TT_F16: return tt::launch_mask<__half>(n_q, n_kv, mask, sq, skv, lo, hi, status, st);
    default: return TT_ERR_UNSUPPORTED;
  }
}
