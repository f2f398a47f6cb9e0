// Tree gated delta rule (GDN), forward and backward, fp32 internally.
//
// Restates torch_chunk_gated_delta_rule_tree_varlen (tree_dfs_ssm.py:38-156):
// one chunk per tree node c (tokens [s, e), L = e - s), per v-head:
//   gam = cumsum(g)                                   (:106)
//   D[j,m] = exp(gam_j - gam_m) for j >= m            (:109)
//   A = -(beta_j k_j . k_m) D   strictly lower        (:116)
//   T = I + A + A^2   (the row loop at :119-126)      applied as x + Ax + A(Ax)
//   U = T (v beta),  W = T (k beta e^gam)             (:127-128)
//   S_in = state after the PARENT node                (:131-132)
//   Vn = U - W S_in                                   (:134-135)
//   O = (q e^gam) S_in + (q k^T * D, lower incl.) Vn  (:137-140)
//   S_out = e^{gam_L} S_in + (k e^{gam_L - gam})^T Vn (:144-148)
// and the exact gradient of that function (what torch autograd computes
// through the reference's Python loop).
//
// Everything is expressed as per-node segmented GEMMs (one descriptor per
// node, any strides per operand) plus elementwise kernels; node states only
// depend on the parent, so the recurrence runs one launch set per tree depth
// level (all nodes of a level in parallel) and the backward runs the levels in
// reverse, summing each node's state gradient over its children without
// atomics.  Internal layout: per-token vectors [H][S][D] fp32, per-node LxL
// matrices packed per node ([H][sum L^2]), states [n_nodes+1][H][Dk][Dv].
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "tt_gdn_gemm.cuh"

namespace tt {
namespace gdn {
namespace {

#ifndef TT_GDN_BK
#define TT_GDN_BK 16
#endif
constexpr int kBM = 64, kBN = 64, kBK = TT_GDN_BK;   // K slice depth: 16 or 32
constexpr int kGemmThreads = 128;           // 16 x 8 threads, 8 x 4 outputs each
constexpr int kRowPad = 4;                  // keeps 16-byte rows, spreads banks

// Two fp32 FMAs in one instruction (IEEE, no flush to zero): d = a * b + c.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// 4-byte asynchronous global -> shared copy; `valid` false writes a zero.
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))), "l"(gmem),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kGemmStages = 3;              // K slices in flight

// C[i,j] = alpha * sum_k A[i,k] B[k,j] + beta * Cin[i,j] over a list of 64 x 64
// output tiles (tile = {segment, tm << 16 | tn}) and heads (blockIdx.z);
// operand element (r, c) of segment s lives at
// base + head * h_stride + off_s + r * rs_s + c * cs_s.
// Register-blocked: each of the 128 threads owns rows {4ty..4ty+3,
// 32+4ty..} and columns {4tx..4tx+3} of the tile, reads them as float4 from
// shared memory and accumulates with paired FMAs.  K slices stream into a
// 3-stage shared-memory ring with asynchronous 4-byte copies (any stride,
// zero-filled outside the segment), two slices ahead of the multiply.
__global__ void __launch_bounds__(kGemmThreads)
seg_gemm(const SegDesc* __restrict__ segs, const int2* __restrict__ tiles,
         const float* __restrict__ A, long long a_hs, const float* __restrict__ B, long long b_hs,
         float* C, long long c_hs, float alpha, float beta, const float* Cin) {
  const int2 tl = tiles[blockIdx.x];
  const SegDesc sd = segs[tl.x];
  const int tm = tl.y >> 16, tn = tl.y & 0xFFFF;
  const int h = blockIdx.z;
  const float* a = A + h * a_hs + sd.a_off;
  const float* b = B + h * b_hs + sd.b_off;
  float* c = C + h * c_hs + sd.c_off;
  const float* cin = (Cin ? Cin : C) + h * c_hs + sd.c_off;   // Cin: C's layout
  __shared__ __align__(16) float sa[kGemmStages][kBK][kBM + kRowPad];
  __shared__ __align__(16) float sb[kGemmStages][kBK][kBN + kRowPad];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int i0 = tm * kBM, j0 = tn * kBN;
  // consecutive threads walk the operand's unit-stride dimension: element i
  // (of kBK/2) of this thread sits at (row ar0 + i*adr, k ak0 + i*adk) of the A
  // slice and (k bk0 + i*bdk, column bc0 + i*bdc) of the B slice
  const bool a_kfast = sd.a_cs == 1, b_nfast = sd.b_cs == 1;
  const int ar0 = a_kfast ? (tid / kBK) : (tid & 63), ak0 = a_kfast ? (tid % kBK) : (tid >> 6);
  const int adr = a_kfast ? kGemmThreads / kBK : 0, adk = a_kfast ? 0 : 2;
  const int bc0 = b_nfast ? (tid & 63) : (tid / kBK), bk0 = b_nfast ? (tid >> 6) : (tid % kBK);
  const int bdc = b_nfast ? 0 : kGemmThreads / kBK, bdk = b_nfast ? 2 : 0;
  const int astep = adr * (int)sd.a_rs + adk * (int)sd.a_cs;
  const int bstep = bdk * (int)sd.b_rs + bdc * (int)sd.b_cs;
  constexpr int kPer = kBM * kBK / kGemmThreads;   // staged elements per operand per thread
  auto issue = [&](int k0, int st) {
    const float* pa = a + (long long)(i0 + ar0) * sd.a_rs + (long long)(k0 + ak0) * sd.a_cs;
    const float* pb = b + (long long)(k0 + bk0) * sd.b_rs + (long long)(j0 + bc0) * sd.b_cs;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const bool in_a = i0 + ar0 + i * adr < sd.M && k0 + ak0 + i * adk < sd.K;
      cp_async4(&sa[st][ak0 + i * adk][ar0 + i * adr], in_a ? pa + i * astep : a, in_a);
      const bool in_b = k0 + bk0 + i * bdk < sd.K && j0 + bc0 + i * bdc < sd.N;
      cp_async4(&sb[st][bk0 + i * bdk][bc0 + i * bdc], in_b ? pb + i * bstep : b, in_b);
    }
  };
  // acc[p][w]: rows 2p and 2p+1 of the thread's 8 rows, column w of its 4
  float2 acc[4][4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int w = 0; w < 4; ++w) acc[p][w] = make_float2(0.f, 0.f);
  const int nk = (sd.K + kBK - 1) / kBK;
  // one commit group per slice (empty past the end), so wait_group counts slices
#pragma unroll
  for (int t = 0; t < kGemmStages - 1; ++t) {
    if (t < nk) issue(t * kBK, t);
    cp_async_commit();
  }
  for (int t = 0; t < nk; ++t) {
    cp_async_wait<kGemmStages - 2>();   // slice t has landed (this thread's copies)
    __syncthreads();                    // ... and everyone's; slice t-1 is consumed
    if (t + kGemmStages - 1 < nk)
      issue((t + kGemmStages - 1) * kBK, (t + kGemmStages - 1) % kGemmStages);
    cp_async_commit();
    const int buf = t % kGemmStages;
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sa[buf][kk][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sa[buf][kk][32 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sb[buf][kk][4 * tx]);
      // row pairs come straight from the float4s; one broadcast per column
      const float2 ap[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w),
                            make_float2(a1.x, a1.y), make_float2(a1.z, a1.w)};
      const float bw[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float2 bb = make_float2(bw[w], bw[w]);
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[p][w] = fma2(ap[p], bb, acc[p][w]);
      }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int gi = i0 + (u < 4 ? 4 * ty + u : 32 + 4 * ty + (u - 4));
    if (gi >= sd.M) continue;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int gj = j0 + 4 * tx + w;
      if (gj >= sd.N) continue;
      const float v = (u & 1) ? acc[u >> 1][w].y : acc[u >> 1][w].x;
      const long long o = gi * sd.c_rs + gj * sd.c_cs;
      c[o] = alpha * v + (beta != 0.f ? beta * cin[o] : 0.f);
    }
  }
}

// Row stride of a node's L x L matrices: L rounded up to 4 floats, so that
// every row starts on a 16-byte boundary (the tensor-core GEMM stages rows
// with 16-byte copies).  Columns [L, Lp) are padding that no kernel reads.
__host__ __device__ __forceinline__ int row_stride(int L) { return (L + 3) & ~3; }

// ---- elementwise kernels ---------------------------------------------------------

constexpr int kTokWarps = 8;   // per-(token, head) kernels: one warp each, 8 per block

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Per (head, token): normalised/scaled q and k, v, beta, and the scaled copies
// used as GEMM operands.  gam must already hold the per-node cumsum.
template <typename T>
__global__ void __launch_bounds__(32 * kTokWarps)
prep_tokens(int S, int Hk, int H, int Dk, int Dv, const T* __restrict__ q,
            const T* __restrict__ k, const T* __restrict__ v, long long q_ts, long long k_ts,
            long long v_ts,
            const float* __restrict__ beta, const float* __restrict__ gam,
            const float* __restrict__ gl_tok, int l2norm, float q_scale,
            float* Q, float* K, float* Vb, float* Kb, float* Kbg, float* Qg, float* Kd) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), h = blockIdx.y;
  const int lane = threadIdx.x & 31;
  if (t >= S) return;                        // whole warps: no block-wide syncs below
  const int hk = h / (H / Hk);
  const T* qr = q + (long long)t * q_ts + (long long)hk * Dk;
  const T* kr = k + (long long)t * k_ts + (long long)hk * Dk;
  float sq = 0.f, sk = 0.f;
  for (int d = lane; d < Dk; d += 32) {
    const float a = to_f32(qr[d]), b = to_f32(kr[d]);
    sq += a * a;
    sk += b * b;
  }
  sq = warp_sum(sq);
  sk = warp_sum(sk);
  const float rq = l2norm ? rsqrtf(sq + 1e-6f) : 1.f;
  const float rk = l2norm ? rsqrtf(sk + 1e-6f) : 1.f;
  const long long ht = (long long)h * S + t;
  const float bt = beta[(long long)t * H + h];
  const float gm = gam[ht];
  const float eg = expf(gm), ed = expf(gl_tok[ht] - gm);
  for (int d = lane; d < Dk; d += 32) {
    const float qs = to_f32(qr[d]) * rq * q_scale;
    const float ks = to_f32(kr[d]) * rk;
    Q[ht * Dk + d] = qs;
    K[ht * Dk + d] = ks;
    Kb[ht * Dk + d] = ks * bt;
    Kbg[ht * Dk + d] = ks * bt * eg;
    Qg[ht * Dk + d] = qs * eg;
    Kd[ht * Dk + d] = ks * ed;
  }
  const T* vr = v + (long long)t * v_ts + (long long)h * Dv;
  for (int d = lane; d < Dv; d += 32) Vb[ht * Dv + d] = to_f32(vr[d]) * bt;
}

// Per (node, head): gam = cumsum(g) over the node's tokens, gl_tok = gam at the
// node's last token (written for every token of the node), gl[c] too.
__global__ void node_cumsum(int S, int H, int n_nodes, const int* __restrict__ nstart,
                            const int* __restrict__ nlen, const float* __restrict__ g,
                            float* gam, float* gl_tok, float* gl) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = blockIdx.y;
  if (c >= n_nodes) return;
  const int s = nstart[c], L = nlen[c];
  float acc = 0.f;
  for (int j = 0; j < L; ++j) {
    acc += g[(long long)(s + j) * H + h];
    gam[(long long)h * S + s + j] = acc;
  }
  for (int j = 0; j < L; ++j) gl_tok[(long long)h * S + s + j] = acc;
  gl[(long long)h * n_nodes + c] = acc;
}

// In place on the packed LxL matrices of every node: A = -KK * D (strict
// lower), Aqk = QK * D (lower incl.).  Raw products are kept in KK/QK.  One
// block per (token, head): row j of the token's node.
__global__ void decay_masks(int S, const int* __restrict__ nstart, const int* __restrict__ nlen,
                            const int* __restrict__ tok_node,
                            const long long* __restrict__ loff, long long l_hs,
                            const float* __restrict__ gam, const float* __restrict__ KK,
                            const float* __restrict__ QK, float* Am, float* Aqk) {
  const int t = blockIdx.x, h = blockIdx.y, c = tok_node[t], j = t - nstart[c];
  const int L = nlen[c];
  const long long base = h * l_hs + loff[c] + (long long)j * row_stride(L);
  const float gj = gam[(long long)h * S + nstart[c] + j];
  for (int m = threadIdx.x; m < L; m += blockDim.x) {
    const float d = m <= j ? expf(gj - gam[(long long)h * S + nstart[c] + m]) : 0.f;
    Am[base + m] = m < j ? -KK[base + m] * d : 0.f;
    Aqk[base + m] = m <= j ? QK[base + m] * d : 0.f;
  }
}

// Exact-inverse mode, first step: each 64 x 64 diagonal block of a node's A
// (the trailing block may be smaller) is replaced in place by
// T_ii = (I - A_ii)^-1, by forward substitution T = I + A T.  Column c of
// T_ii depends only on column c of the rows above it, so thread c owns it.
constexpr int kInvB = 64;
__global__ void __launch_bounds__(kInvB)
tri_inv_diag(const int2* __restrict__ blocks, const int* __restrict__ nlen,
             const long long* __restrict__ loff, long long l_hs, float* Am) {
  const int2 bl = blocks[blockIdx.x];
  const int c = bl.x, i0 = bl.y * kInvB, h = blockIdx.y;
  const int L = nlen[c], Lp = row_stride(L);
  const int bs = min(kInvB, L - i0);
  float* base = Am + h * l_hs + loff[c] + (long long)i0 * Lp + i0;
  __shared__ float sA[kInvB][kInvB + 1];
  __shared__ float sT[kInvB][kInvB + 1];
  for (int idx = threadIdx.x; idx < bs * bs; idx += blockDim.x)
    sA[idx / bs][idx % bs] = base[(long long)(idx / bs) * Lp + idx % bs];
  __syncthreads();
  const int col = threadIdx.x;
  if (col < bs) {
    for (int r = 0; r < bs; ++r) {
      float t = r == col ? 1.f : 0.f;
      for (int j = col; j < r; ++j) t = fmaf(sA[r][j], sT[j][col], t);
      sT[r][col] = r >= col ? t : 0.f;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < bs * bs; idx += blockDim.x)
    base[(long long)(idx / bs) * Lp + idx % bs] = sT[idx / bs][idx % bs];
}

// states[c+1][h] += exp(gl[h][c]) * states[parent+1][h]   for the level's nodes
__global__ void state_decay_add(int H, int DkDv, int n_nodes, const int* __restrict__ nodes,
                                const int* __restrict__ parent, const float* __restrict__ gl,
                                float* states) {
  const int c = nodes[blockIdx.y], h = blockIdx.z;
  const long long hs = (long long)H * DkDv;
  const float f = expf(gl[(long long)h * n_nodes + c]);
  const float* src = states + (long long)(parent[c] + 1) * hs + (long long)h * DkDv;
  float* dst = states + (long long)(c + 1) * hs + (long long)h * DkDv;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < DkDv; i += gridDim.x * blockDim.x)
    dst[i] += f * src[i];
}

// Fill states[0] (initial state or zeros).
__global__ void init_state(long long n, const float* __restrict__ init, float* s0) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) s0[i] = init ? init[i] : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(32 * kTokWarps)
store_out(int S, int H, int Dv, const float* __restrict__ O, T* out) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), h = blockIdx.y;
  if (t >= S) return;
  for (int d = threadIdx.x & 31; d < Dv; d += 32)
    out[((long long)t * H + h) * Dv + d] = from_f32<T>(O[((long long)h * S + t) * Dv + d]);
}

template <typename T>
__global__ void __launch_bounds__(32 * kTokWarps)
load_dout(int S, int H, int Dv, const T* __restrict__ dout, float* dO) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), h = blockIdx.y;
  if (t >= S) return;
  for (int d = threadIdx.x & 31; d < Dv; d += 32)
    dO[((long long)h * S + t) * Dv + d] = to_f32(dout[((long long)t * H + h) * Dv + d]);
}

// dSo[c] = sum over children dSi[ch] (+ dlast for the last DFS node) for the
// level's nodes; children in CSR (child_ptr, child_idx).
__global__ void gather_dstate(int H, int DkDv, int n_nodes, const int* __restrict__ nodes,
                              const int* __restrict__ child_ptr, const int* __restrict__ child_idx,
                              const float* __restrict__ dSi, const float* __restrict__ dlast,
                              const int* __restrict__ cap_slot, const float* __restrict__ dcap,
                              float* dSo) {
  const int c = nodes[blockIdx.y], h = blockIdx.z;
  const long long hs = (long long)H * DkDv;
  const int slot = dcap ? cap_slot[c] : -1;   // gradient of a captured state, if any
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < DkDv; i += gridDim.x * blockDim.x) {
    float a = (dlast && c == n_nodes - 1) ? dlast[(long long)h * DkDv + i] : 0.f;
    if (slot >= 0) a += dcap[(long long)slot * hs + (long long)h * DkDv + i];
    for (int e = child_ptr[c]; e < child_ptr[c + 1]; ++e)
      a += dSi[(long long)child_idx[e] * hs + (long long)h * DkDv + i];
    dSo[(long long)c * hs + (long long)h * DkDv + i] = a;
  }
}

// dSi[c] += exp(gl[c]) dSo[c]  and  dgl[h][c] = exp(gl[c]) <S_in, dSo>  (the
// gradient of the state decay factor) for the level's nodes.
__global__ void dstate_decay(int H, int DkDv, int n_nodes, const int* __restrict__ nodes,
                             const int* __restrict__ parent, const float* __restrict__ gl,
                             const float* __restrict__ states, const float* __restrict__ dSo,
                             float* dSi, float* dgl) {
  const int c = nodes[blockIdx.x], h = blockIdx.y;
  const long long hs = (long long)H * DkDv;
  const float f = expf(gl[(long long)h * n_nodes + c]);
  const float* sin = states + (long long)(parent[c] + 1) * hs + (long long)h * DkDv;
  const float* so = dSo + (long long)c * hs + (long long)h * DkDv;
  float* si = dSi + (long long)c * hs + (long long)h * DkDv;
  float acc = 0.f;
  for (int i = threadIdx.x; i < DkDv; i += blockDim.x) {
    si[i] += f * so[i];
    acc += sin[i] * so[i];
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a += red[w];
    dgl[(long long)h * n_nodes + c] = f * a;
  }
}

// On every node's LxL matrices:
//   dA  = (dT + dT A^T + A^T dT) on the strict lower part (inputs combined by
//         the caller into dA = dT + X, X = dT A^T + A^T dT), masked here;
//   G   = -dA * D (-> dKb += G K, dK += G^T Kb)
//   F   = dAqk * D (lower incl.; -> dQ += F K, dK += F^T Q)
//   dDD = (-dA * KK + dAqk * QK) * D, whose row/col sums give dgam.
// KK / QK: the raw products (premasked = 0) or the masked A and Aqk
// (premasked = 1, A = -KK D below the diagonal, Aqk = QK D on and below it):
// either way dDD = (-dA KK + dAqk QK) D = dA A + dAqk Aqk.
__global__ void grad_masks(int S, const int* __restrict__ nstart, const int* __restrict__ nlen,
                           const int* __restrict__ tok_node,
                           const long long* __restrict__ loff, long long l_hs,
                           const float* __restrict__ gam, const float* __restrict__ KK,
                           const float* __restrict__ QK, int premasked, float* dA, float* dAqk,
                           float* dDD) {
  const int t = blockIdx.x, h = blockIdx.y, c = tok_node[t], j = t - nstart[c];
  const int L = nlen[c];
  const long long base = h * l_hs + loff[c] + (long long)j * row_stride(L);
  const float gj = gam[(long long)h * S + nstart[c] + j];
  for (int m = threadIdx.x; m < L; m += blockDim.x) {
    const float d = m <= j ? expf(gj - gam[(long long)h * S + nstart[c] + m]) : 0.f;
    const float da = m < j ? dA[base + m] : 0.f;
    const float dq = m <= j ? dAqk[base + m] : 0.f;
    dDD[base + m] = premasked ? da * KK[base + m] + dq * QK[base + m]
                              : (-da * KK[base + m] + dq * QK[base + m]) * d;
    dA[base + m] = -da * d;      // G
    dAqk[base + m] = dq * d;     // F
  }
}

// dgam_j += sum_m dDD[j, m] - sum_i dDD[i, j]  (per node, per head; dDD is
// lower triangular).  One block per (node, head): warps take rows (coalesced
// row sums into `rowsum`), then threads take columns and walk down the rows,
// so every read of the node's matrix is a coalesced row segment.  The two
// sums cancel to a small difference: both accumulate in fp64.
constexpr int kRowColThreads = 256;
// grad_masks and ddd_rowcol in one pass per (node, head), without writing
// dDD: warp w takes rows j = w, w + 8, ...; for each element of its row it
// forms G, F (written back over dA, dAqk, the whole row as grad_masks does)
// and dDD[j, m] in registers, sums the row (fp64, lanes then shuffles, as
// ddd_rowcol) and adds the value to its own fp64 column partial in shared
// memory.  After all rows the 8 warps' partials of each column are added in
// warp order and dgam_m += rowsum_m - colsum_m.  Shared memory: 9 x L doubles
// (the launch takes nodes up to kFusedMaskMaxL tokens).
constexpr int kFusedMaskMaxL = 2048;
__global__ void __launch_bounds__(kRowColThreads)
grad_masks_rowcol(int S, const int* __restrict__ nstart, const int* __restrict__ nlen,
                  const long long* __restrict__ loff, long long l_hs,
                  const float* __restrict__ gam, const float* __restrict__ KK,
                  const float* __restrict__ QK, int premasked, float* dA, float* dAqk,
                  float* dgam) {
  extern __shared__ double gm_smem[];
  constexpr int kW = kRowColThreads / 32;
  const int c = blockIdx.x, h = blockIdx.y;
  const int L = nlen[c], Lp = row_stride(L), s0 = nstart[c];
  double* colp = gm_smem;               // [kW][L]
  double* rs = gm_smem + kW * L;        // [L]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kW * L; i += kRowColThreads) colp[i] = 0.0;
  __syncthreads();
  const float* g = gam + (long long)h * S + s0;
  const long long nb = h * l_hs + loff[c];
  for (int j = warp; j < L; j += kW) {
    const long long base = nb + (long long)j * Lp;
    const float gj = g[j];
    double a = 0.0;
    for (int m = lane; m < L; m += 32) {
      const float d = m <= j ? expf(gj - g[m]) : 0.f;
      const float da = m < j ? dA[base + m] : 0.f;
      const float dq = m <= j ? dAqk[base + m] : 0.f;
      const float v = premasked ? da * KK[base + m] + dq * QK[base + m]
                                : (-da * KK[base + m] + dq * QK[base + m]) * d;
      dA[base + m] = -da * d;      // G
      dAqk[base + m] = dq * d;     // F
      if (m <= j) {
        a += (double)v;
        colp[warp * L + m] += (double)v;
      }
    }
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) rs[j] = a;
  }
  __syncthreads();
  for (int m = threadIdx.x; m < L; m += kRowColThreads) {
    double col = 0.0;
#pragma unroll
    for (int w = 0; w < kW; ++w) col += colp[w * L + m];
    dgam[(long long)h * S + s0 + m] += (float)(rs[m] - col);
  }
}

__global__ void __launch_bounds__(kRowColThreads)
ddd_rowcol(int S, const int* __restrict__ nstart, const int* __restrict__ nlen,
           const long long* __restrict__ loff, long long l_hs, const float* __restrict__ dDD,
           double* rowsum, float* dgam) {
  const int c = blockIdx.x, h = blockIdx.y;
  const int L = nlen[c], Lp = row_stride(L), s0 = nstart[c];
  const float* base = dDD + h * l_hs + loff[c];
  double* rs = rowsum + (long long)h * S + s0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < L; j += kRowColThreads / 32) {
    const float* row = base + (long long)j * Lp;
    double a = 0.0;
    for (int m = lane; m <= j; m += 32) a += (double)row[m];
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) rs[j] = a;
  }
  __syncthreads();
  for (int m = threadIdx.x; m < L; m += kRowColThreads) {
    double col = 0.0;
    const float* p = base + (long long)m * Lp + m;
#pragma unroll 4
    for (int j = m; j < L; ++j, p += Lp) col += (double)*p;
    dgam[(long long)h * S + s0 + m] += (float)(rs[m] - col);
  }
}

// Per (head, token): assemble the input gradients.  Inputs (fp32 [H][S][D]):
// dQs (grad of the scaled q, incl. the e^gam part via dQg), dKt (grad of k
// from all k-terms except the beta-scaled ones), dKb (grad of k*beta incl.
// dKbg*e^gam), dVb; plus gam, gl, and the Qg/Kbg/Kd-dependent dgam parts.
// kIt > 0: Dk == 32 kIt, every lane's q / k values and gradients held in
// registers (all loads issued up front, dq / dk written once); kIt == 0: any
// Dk, the gradients stored and finished in a second pass.  Same arithmetic
// and order either way.
template <typename T, int kIt>
__global__ void __launch_bounds__(32 * kTokWarps)
assemble_token_grads(int S, int Hk, int H, int Dk, int Dv, const T* __restrict__ q,
                                     const T* __restrict__ k, const T* __restrict__ v,
                                     long long q_ts, long long k_ts, long long v_ts,
                                     const float* __restrict__ beta, const float* __restrict__ gam,
                                     const float* __restrict__ gl_tok, int l2norm, float q_scale,
                                     const float* __restrict__ dQ, const float* __restrict__ dQg,
                                     const float* __restrict__ dK, const float* __restrict__ dKd,
                                     const float* __restrict__ dKb, const float* __restrict__ dKbg,
                                     const float* __restrict__ dVb, float* dgam, float* dq_h,
                                     float* dk_h, float* dbeta_out, T* dv_out) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), h = blockIdx.y;
  const int lane = threadIdx.x & 31;
  if (t >= S) return;                        // whole warps: no block-wide syncs below
  const int hk = h / (H / Hk);
  const long long ht = (long long)h * S + t;
  const T* qr = q + (long long)t * q_ts + (long long)hk * Dk;
  const T* kr = k + (long long)t * k_ts + (long long)hk * Dk;
  const float bt = beta[(long long)t * H + h];
  const float gm = gam[ht];
  const float eg = expf(gm), ed = expf(gl_tok[ht] - gm);
  constexpr int kR = kIt > 0 ? kIt : 1;
  float qv[kR], kv[kR], gq[kR], gkk[kR];
  // norms again (cheap) for the normalised q/k and the l2norm backward
  float sq = 0.f, sk = 0.f;
  if (kIt > 0) {
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      qv[i] = to_f32(qr[lane + 32 * i]);
      kv[i] = to_f32(kr[lane + 32 * i]);
      sq += qv[i] * qv[i];
      sk += kv[i] * kv[i];
    }
  } else {
    for (int d = lane; d < Dk; d += 32) {
      const float a = to_f32(qr[d]), b = to_f32(kr[d]);
      sq += a * a;
      sk += b * b;
    }
  }
  sq = warp_sum(sq);
  sk = warp_sum(sk);
  const float rq = l2norm ? rsqrtf(sq + 1e-6f) : 1.f;
  const float rk = l2norm ? rsqrtf(sk + 1e-6f) : 1.f;
  // d(scaled q) = dQ + dQg e^gam ; d(k) = dK + dKd e^{gl-gam} + beta (dKb + dKbg e^gam)
  float p_qg = 0.f, p_kbg = 0.f, p_kd = 0.f, p_kb = 0.f, xdq = 0.f, xdk = 0.f;
  auto term = [&](int d, float qx, float kx, float& gqn_out, float& gk_out) {
    const float qn = qx * rq, kn = kx * rk;
    const float qs = qn * q_scale;
    const float gqs = dQ[ht * Dk + d] + dQg[ht * Dk + d] * eg;
    const float gkb = dKb[ht * Dk + d] + dKbg[ht * Dk + d] * eg;
    const float gk = dK[ht * Dk + d] + dKd[ht * Dk + d] * ed + bt * gkb;
    p_qg += qs * eg * dQg[ht * Dk + d];
    p_kbg += kn * bt * eg * dKbg[ht * Dk + d];
    p_kd += kn * ed * dKd[ht * Dk + d];
    p_kb += kn * gkb;
    const float gqn = gqs * q_scale;          // grad wrt normalised q
    xdq += qn * gqn;
    xdk += kn * gk;
    gqn_out = gqn;
    gk_out = gk;
  };
  if (kIt > 0) {
#pragma unroll
    for (int i = 0; i < kR; ++i) term(lane + 32 * i, qv[i], kv[i], gq[i], gkk[i]);
  } else {
    for (int d = lane; d < Dk; d += 32) {
      float gqn, gk;
      term(d, to_f32(qr[d]), to_f32(kr[d]), gqn, gk);
      dq_h[ht * Dk + d] = gqn;                // finished below with the l2norm backward
      dk_h[ht * Dk + d] = gk;
    }
  }
  p_qg = warp_sum(p_qg);
  p_kbg = warp_sum(p_kbg);
  p_kd = warp_sum(p_kd);
  p_kb = warp_sum(p_kb);
  xdq = warp_sum(xdq);
  xdk = warp_sum(xdk);
  // y = x r (r = (|x|^2+eps)^-1/2): dx = r dy - r^3 (x.dy) x = r (dy - (y.dy) y)
  if (kIt > 0) {
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      const int d = lane + 32 * i;
      if (l2norm) {
        dq_h[ht * Dk + d] = rq * (gq[i] - xdq * (qv[i] * rq));
        dk_h[ht * Dk + d] = rk * (gkk[i] - xdk * (kv[i] * rk));
      } else {
        dq_h[ht * Dk + d] = gq[i];
        dk_h[ht * Dk + d] = gkk[i];
      }
    }
  } else {
    for (int d = lane; d < Dk; d += 32) {
      if (l2norm) {
        const float qn = to_f32(qr[d]) * rq, kn = to_f32(kr[d]) * rk;
        dq_h[ht * Dk + d] = rq * (dq_h[ht * Dk + d] - xdq * qn);
        dk_h[ht * Dk + d] = rk * (dk_h[ht * Dk + d] - xdk * kn);
      }
    }
  }
  float p_vb = 0.f;
  const T* vr = v + (long long)t * v_ts + (long long)h * Dv;
#pragma unroll 4
  for (int d = lane; d < Dv; d += 32) {
    const float g = dVb[ht * Dv + d];
    p_vb += to_f32(vr[d]) * g;
    dv_out[((long long)t * H + h) * Dv + d] = from_f32<T>(g * bt);
  }
  p_vb = warp_sum(p_vb);
  if (lane == 0) {
    dbeta_out[(long long)t * H + h] = p_kb + p_vb;
    // e^gam terms of Qg, Kbg and the -gam of Kd (the +gl part goes to the node's last token)
    dgam[ht] += p_qg + p_kbg - p_kd;
  }
}

// dgl per node from the Kd term: sum over the node's tokens of kn e^{gl-gam} . dKd,
// added to dgam at the node's last token together with the state-decay part.
// Then dg = reverse cumsum of dgam within the node.
__global__ void node_dg(int S, int H, int n_nodes, const int* __restrict__ nstart,
                        const int* __restrict__ nlen, const float* __restrict__ kd_dot,
                        const float* __restrict__ dgl, float* dgam, float* dg) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x, h = blockIdx.y;
  if (c >= n_nodes) return;
  const int s = nstart[c], L = nlen[c];
  if (L == 0) return;
  // fp64 sums: dg is a reverse cumulative sum of terms that largely cancel
  double tail = dgl[(long long)h * n_nodes + c];
  for (int j = 0; j < L; ++j) tail += kd_dot[(long long)h * S + s + j];
  double acc = tail;
  for (int j = L - 1; j >= 0; --j) {
    acc += dgam[(long long)h * S + s + j];
    dg[(long long)(s + j) * H + h] = (float)acc;
  }
}

// kd_dot[h][t] = kn_t e^{gl-gam_t} . dKd_t  (per token, reduced over Dk)
__global__ void __launch_bounds__(32 * kTokWarps)
kd_dot_kernel(int S, int Dk, const float* __restrict__ Kd, const float* __restrict__ dKd,
              float* out) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= S) return;
  const long long ht = (long long)blockIdx.y * S + t;
  float acc = 0.f;
  for (int d = lane; d < Dk; d += 32) acc += Kd[ht * Dk + d] * dKd[ht * Dk + d];
  acc = warp_sum(acc);
  if (lane == 0) out[ht] = acc;
}

// dq/dk per k-head: sum the per-v-head gradients of each GQA group, cast.
template <typename T>
__global__ void __launch_bounds__(32 * kTokWarps)
reduce_gqa(int S, int Hk, int H, int Dk, const float* __restrict__ src, T* dst) {
  const int t = blockIdx.x * kTokWarps + (threadIdx.x >> 5), hk = blockIdx.y, rep = H / Hk;
  if (t >= S) return;
  for (int d = threadIdx.x & 31; d < Dk; d += 32) {
    float a = 0.f;
    for (int r = 0; r < rep; ++r) a += src[(((long long)(hk * rep + r)) * S + t) * Dk + d];
    dst[((long long)t * Hk + hk) * Dk + d] = from_f32<T>(a);
  }
}

// The same for dq and dk in one launch (blockIdx.y: 0 = q, 1 = k), one thread
// per 4 consecutive elements of a (token, k-head) row: 16-byte loads of each
// group head, added in head order as above.  Needs Dk % 4 == 0, 16-byte aligned
// sources and destinations aligned to 4 elements.
template <typename T>
__global__ void __launch_bounds__(256)
reduce_gqa4(int S, int Hk, int H, int Dk, const float* __restrict__ src_q, T* dst_q,
            const float* __restrict__ src_k, T* dst_k) {
  const float* src = blockIdx.y ? src_k : src_q;
  T* dst = blockIdx.y ? dst_k : dst_q;
  const int nq = Dk / 4, rep = H / Hk;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)S * Hk * nq) return;
  const int e = (int)(i % nq) * 4;
  const long long th = i / nq;
  const int hk = (int)(th % Hk), t = (int)(th / Hk);
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < rep; ++r) {
    const float4 v =
        *reinterpret_cast<const float4*>(src + (((long long)(hk * rep + r)) * S + t) * Dk + e);
    a[0] += v.x;
    a[1] += v.y;
    a[2] += v.z;
    a[3] += v.w;
  }
  struct alignas(4 * sizeof(T)) Q4 {
    T v[4];
  } o;
#pragma unroll
  for (int j = 0; j < 4; ++j) o.v[j] = from_f32<T>(a[j]);
  *reinterpret_cast<Q4*>(dst + ((long long)t * Hk + hk) * Dk + e) = o;
}

__global__ void dinit_kernel(int H, int DkDv, int n_roots, const int* __restrict__ roots,
                             const float* __restrict__ dSi, float* dinit) {
  const long long hs = (long long)H * DkDv;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= hs) return;
  float a = 0.f;
  for (int r = 0; r < n_roots; ++r) a += dSi[(long long)roots[r] * hs + i];
  dinit[i] = a;
}

// =============================================================================
// host orchestration
// =============================================================================

// A call's metadata (plan arrays, GEMM descriptors and tile lists: one
// contiguous span of the workspace) travels host -> device through a pinned
// staging buffer that a copy kernel reads in stream order.  No pageable copy
// (which can make the host wait for the stream) and no copy-engine queue (in
// which it would wait behind a large upload the caller has in flight on
// another stream).  Two buffers per device alternate; one is refilled only
// after the copy kernel that read it has run.
struct MetaStage {
  char* host = nullptr;
  size_t cap = 0;
  cudaEvent_t read = nullptr;   // recorded after the copy kernel that read `host`
  bool pending = false;
};
constexpr int kStageDevs = 64;
MetaStage g_stage[kStageDevs][2];
int g_stage_next[kStageDevs];
std::mutex g_stage_mu;

__global__ void copy_from_host(const uint4* __restrict__ src, uint4* __restrict__ dst,
                               long long n16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16;
       i += (long long)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

struct MetaPiece {
  void* dst;
  const void* src;
  size_t bytes;
};

// Copies every piece (device destinations inside [span, span + span_bytes),
// span and span_bytes multiples of 16) through a staging buffer.
int upload_meta(char* span, size_t span_bytes, const std::vector<MetaPiece>& pieces,
                cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStageDevs) return TT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_stage_mu);
  MetaStage& m = g_stage[dev][g_stage_next[dev]];
  g_stage_next[dev] ^= 1;
  if (m.pending && cudaEventSynchronize(m.read) != cudaSuccess) return TT_ERR_CUDA;
  m.pending = false;
  if (m.cap < span_bytes) {
    if (m.host) cudaFreeHost(m.host);
    m.host = nullptr;
    m.cap = 0;
    const size_t cap = span_bytes + span_bytes / 2 + 4096;
    if (cudaHostAlloc(reinterpret_cast<void**>(&m.host), cap,
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
      return TT_ERR_CUDA;
    m.cap = cap;
  }
  if (!m.read && cudaEventCreateWithFlags(&m.read, cudaEventDisableTiming) != cudaSuccess)
    return TT_ERR_CUDA;
  for (const MetaPiece& pc : pieces)
    if (pc.bytes) std::memcpy(m.host + (static_cast<char*>(pc.dst) - span), pc.src, pc.bytes);
  void* src_dev = nullptr;
  if (cudaHostGetDevicePointer(&src_dev, m.host, 0) != cudaSuccess) return TT_ERR_CUDA;
  const long long n16 = (long long)(span_bytes / 16);
  const int blocks = (int)std::min<long long>((n16 + 255) / 256, 512);
  copy_from_host<<<std::max(blocks, 1), 256, 0, st>>>(static_cast<const uint4*>(src_dev),
                                                      reinterpret_cast<uint4*>(span), n16);
  if (cudaGetLastError() != cudaSuccess || cudaEventRecord(m.read, st) != cudaSuccess)
    return TT_ERR_CUDA;
  m.pending = true;
  return TT_OK;
}

struct Plan {
  int S, H, Hk, Dk, Dv, n;
  // elements from one token's q / k / v row to the next (0: packed rows of
  // Hk * Dk, Hk * Dk and H * Dv elements)
  long long q_ts = 0, k_ts = 0, v_ts = 0;
  std::vector<int> start, len, parent, depth;
  std::vector<int> tok_node;       // node of each token
  std::vector<long long> loff;     // packed L x Lp offset per node (Lp = row_stride(L))
  std::vector<long long> xoff;     // 64 x Lp scratch block per node (exact inverse)
  long long ll_total = 0;          // sum L * Lp
  long long lp_total = 0;          // sum Lp
  int max_len = 0, max_depth = 0;
  std::vector<std::vector<int>> levels;
  std::vector<int> child_ptr, child_idx, roots;
};

int make_plan(Plan& p, int S, int H, int Hk, int Dk, int Dv, int n, const int32_t* bounds,
              const int32_t* parents) {
  p.S = S; p.H = H; p.Hk = Hk; p.Dk = Dk; p.Dv = Dv; p.n = n;
  p.start.resize(n); p.len.resize(n); p.parent.resize(n); p.depth.resize(n); p.loff.resize(n);
  p.xoff.resize(n);
  int expect = 0;
  for (int c = 0; c < n; ++c) {
    const int s = bounds[2 * c], e = bounds[2 * c + 1], par = parents[c];
    if (s != expect || e < s || par < -1 || par >= c) return TT_ERR_INVALID_ARG;
    expect = e;
    p.start[c] = s; p.len[c] = e - s; p.parent[c] = par;
    p.depth[c] = par < 0 ? 0 : p.depth[par] + 1;
    p.loff[c] = p.ll_total;
    p.ll_total += (long long)(e - s) * row_stride(e - s);
    p.xoff[c] = 64LL * p.lp_total;
    p.lp_total += row_stride(e - s);
    p.max_len = std::max(p.max_len, e - s);
    p.max_depth = std::max(p.max_depth, p.depth[c]);
  }
  if (expect != S) return TT_ERR_INVALID_ARG;
  p.tok_node.resize(S);
  for (int c = 0; c < n; ++c)
    for (int t = p.start[c]; t < p.start[c] + p.len[c]; ++t) p.tok_node[t] = c;
  p.levels.assign(p.max_depth + 1, {});
  for (int c = 0; c < n; ++c) p.levels[p.depth[c]].push_back(c);
  p.child_ptr.assign(n + 1, 0);
  for (int c = 0; c < n; ++c) if (p.parent[c] >= 0) p.child_ptr[p.parent[c] + 1]++;
  for (int c = 0; c < n; ++c) p.child_ptr[c + 1] += p.child_ptr[c];
  p.child_idx.resize(p.child_ptr[n]);
  std::vector<int> fill(p.child_ptr.begin(), p.child_ptr.end() - 1);
  for (int c = 0; c < n; ++c) {
    if (p.parent[c] >= 0) p.child_idx[fill[p.parent[c]]++] = c;
    else p.roots.push_back(c);
  }
  return TT_OK;
}

// Bump allocator over the caller's workspace (256-byte aligned pieces).
struct Arena {
  char* base;
  int64_t cap, used = 0;
  bool sizing;
  template <typename T>
  T* get(long long n) {
    const int64_t bytes = ((int64_t)std::max<long long>(n, 1) * (int64_t)sizeof(T) + 255) / 256 * 256;
    T* r = sizing ? nullptr : reinterpret_cast<T*>(base + used);
    used += bytes;
    return r;
  }
};

// All device buffers of one forward (+ backward) run.
struct Bufs {
  float *gam, *gl_tok, *gl, *Q, *K, *Vb, *Kb, *Kbg, *Qg, *Kd, *U, *W, *T1, *Vn, *O;
  float *KK, *QK, *Am, *Aqk, *states;
  // backward
  float *dO, *dVn, *dQg, *dKd, *dW, *dT, *dA, *dAqk, *dDD, *X, *dVb, *dKbg, *dKb, *dQ, *dK;
  float *dSo, *dSi, *dgl, *dgam, *kd_dot, *dq_h, *dk_h;
  double* rowsum;   // fp64 row sums of dDD per (head, token)
  int *d_tok_node;
  int *d_start, *d_len, *d_parent, *d_child_ptr, *d_child_idx, *d_roots, *d_level_nodes;
  long long* d_loff;
  SegDesc* d_desc;
  int2* d_tiles;
  int2* d_tiles_tc;
  int2* d_inv_blocks;   // (node, diagonal block) pairs of the exact-inverse mode
  int* d_cap_slot;      // per node: index into the captured states, or -1
};

// Descriptor sets: built on the host in one vector, copied once, with the
// exact list of 64 x 64 output tiles of each set (so no block of a launch
// lands outside its segment).
struct DescSet {
  int first, count, tfirst, tcount;
  int tc_first, tc_count;   // the same segments as 128 x 128 tensor-core tiles
  double flops;   // 2 M N K summed over the set's segments, one head
};

struct Builder {
  const Plan& p;
  std::vector<SegDesc> all;
  std::vector<int2> tiles;      // 64 x 64 tiles (CUDA-core GEMM)
  std::vector<int2> tiles_tc;   // kTcTile x kTcTile tiles (tensor-core GEMM)
  explicit Builder(const Plan& pl) : p(pl) {}
  DescSet add(const std::vector<SegDesc>& v) {
    DescSet d{(int)all.size(), (int)v.size(), (int)tiles.size(), 0, (int)tiles_tc.size(), 0, 0.0};
    for (size_t i = 0; i < v.size(); ++i) {
      d.flops += 2.0 * v[i].M * v[i].N * v[i].K;
      const int seg = (int)all.size() + (int)i;
      const int tms = (v[i].M + kBM - 1) / kBM, tns = (v[i].N + kBN - 1) / kBN;
      for (int tm = 0; tm < tms; ++tm)
        for (int tn = 0; tn < tns; ++tn) tiles.push_back(make_int2(seg, (tm << 16) | tn));
      const int ums = (v[i].M + kTcTile - 1) / kTcTile, uns = (v[i].N + kTcTile - 1) / kTcTile;
      for (int tm = 0; tm < ums; ++tm)
        for (int tn = 0; tn < uns; ++tn) tiles_tc.push_back(make_int2(seg, (tm << 16) | tn));
    }
    d.tcount = (int)tiles.size() - d.tfirst;
    d.tc_count = (int)tiles_tc.size() - d.tc_first;
    all.insert(all.end(), v.begin(), v.end());
    return d;
  }
  // Dual pairs (v1[i] then v2[i], the first flagged `dual`) adding both
  // products into v1[i]'s output tiles: tensor-core tiles for the first of
  // each pair only, none for the CUDA-core GEMM (which runs the two single
  // sets instead).
  DescSet add_dual(const std::vector<SegDesc>& v1, const std::vector<SegDesc>& v2) {
    DescSet d{(int)all.size(), 2 * (int)v1.size(), (int)tiles.size(), 0,
              (int)tiles_tc.size(), 0, 0.0};
    for (size_t i = 0; i < v1.size(); ++i) {
      d.flops += 2.0 * v1[i].M * v1[i].N * v1[i].K + 2.0 * v2[i].M * v2[i].N * v2[i].K;
      const int seg = (int)all.size();
      SegDesc first = v1[i];
      first.dual = 1;
      all.push_back(first);
      all.push_back(v2[i]);
      const int ums = (first.M + kTcTile - 1) / kTcTile, uns = (first.N + kTcTile - 1) / kTcTile;
      for (int tm = 0; tm < ums; ++tm)
        for (int tn = 0; tn < uns; ++tn) tiles_tc.push_back(make_int2(seg, (tm << 16) | tn));
    }
    d.tc_count = (int)tiles_tc.size() - d.tc_first;
    return d;
  }
};

SegDesc desc(int M, int N, int K, long long ao, long long ars, long long acs, long long bo,
             long long brs, long long bcs, long long co, long long crs, long long ccs,
             int kmode = kKFull) {
  SegDesc d;
  d.M = M; d.N = N; d.K = K; d.kmode = kmode; d.tok0 = 0; d.dual = 0;
  d.a_off = ao; d.a_rs = ars; d.a_cs = acs;
  d.b_off = bo; d.b_rs = brs; d.b_cs = bcs;
  d.c_off = co; d.c_rs = crs; d.c_cs = ccs;
  return d;
}

std::atomic<int64_t> g_gemm_flops{0};
std::atomic<int64_t> g_gemm_tc_flops{0};

// Which GEMM runs the segments: 0 = automatic (tensor cores: 3xTF32 products
// for fp32 inputs, TF32 products for 16-bit inputs), 1 = tensor cores with
// 3xTF32 products for any input, 2 = the CUDA-core fp32 GEMM; plus 4 = stage
// the tensor cores' operands with cp.async copies instead of TMA.
// Initialised from TT_GDN_GEMM; tt_gdn_set_gemm_mode changes it.
std::atomic<int> g_gemm_mode{-1};

int gemm_mode() {
  int m = g_gemm_mode.load();
  if (m < 0) {
    const char* e = std::getenv("TT_GDN_GEMM");
    m = e ? std::atoi(e) & 7 : 0;
    if ((m & 3) == 3) m = 0;
    g_gemm_mode.store(m);
  }
  return m;
}

// One GEMM launch context: the device descriptor/tile arrays, the host copy
// of the descriptors (for the tensor-core kernel's layout check) and the
// product split the run uses (0 = CUDA cores, 1 = TF32, 3 = 3xTF32).
struct GemmCtx {
  const SegDesc* d_desc;
  const int2* d_tiles;
  const int2* d_tiles_tc;
  const std::vector<SegDesc>* h_desc;
  const std::vector<int2>* h_tiles_tc;
  int split;
  bool tma;
  int rc = TT_OK;
};

// Tiles address segments by their index in the whole descriptor array.
// C = alpha A B + beta Cin (Cin defaults to C; it has C's offsets and strides)
void launch_gemm(GemmCtx& g, DescSet ds, int H, const float* A, long long a_hs, const float* B,
                 long long b_hs, float* C, long long c_hs, float alpha, float beta,
                 cudaStream_t st, const float* Cin = nullptr, EpiMask mask = {}) {
  if (ds.tcount == 0) return;
  const bool tc = g.split != 0 && tt_gdn_tc_gemm_supported(g.h_desc->data(), ds.first, ds.count,
                                                           A, a_hs, B, b_hs, C, c_hs);
  if (mask.mode != kMaskNone && !tc) {   // only the tensor-core epilogue applies masks
    g.rc = TT_ERR_UNSUPPORTED;
    return;
  }
  if (tc) {
    int launches = 0;
    if (g.tma) {
      // chunks of at most kTmaMaxSegs segments (their tensor maps travel as
      // kernel parameters), each with the tiles of exactly its segments
      int t = ds.tc_first;
      const int t_end = ds.tc_first + ds.tc_count;
      for (int c0 = 0; c0 < ds.count; c0 += kTmaMaxSegs) {
        const int c1 = std::min(ds.count, c0 + kTmaMaxSegs);
        const int seg_end = ds.first + c1;
        int t1 = t;
        while (t1 < t_end && (*g.h_tiles_tc)[t1].x < seg_end) ++t1;
        int rc = tt_gdn_seg_gemm_tma(g.h_desc->data() + ds.first + c0, ds.first + c0, c1 - c0,
                                     g.d_desc, g.d_tiles_tc + t, t1 - t, H, A, a_hs, B, b_hs, C,
                                     c_hs, alpha, beta, Cin, g.split, st, mask);
        if (rc == TT_ERR_UNSUPPORTED)
          rc = tt_gdn_seg_gemm_tc(g.d_desc, g.d_tiles_tc + t, t1 - t, H, A, a_hs, B, b_hs, C,
                                  c_hs, alpha, beta, Cin, g.split, st, mask);
        if (rc != TT_OK) g.rc = rc;
        if (t1 > t) ++launches;
        t = t1;
      }
    } else {
      const int rc = tt_gdn_seg_gemm_tc(g.d_desc, g.d_tiles_tc + ds.tc_first, ds.tc_count, H, A,
                                        a_hs, B, b_hs, C, c_hs, alpha, beta, Cin, g.split, st,
                                        mask);
      if (rc != TT_OK) g.rc = rc;
      launches = 1;
    }
    tt_count_launches(launches);
    g_gemm_flops.fetch_add(static_cast<int64_t>(ds.flops * H), std::memory_order_relaxed);
    g_gemm_tc_flops.fetch_add(static_cast<int64_t>(ds.flops * H), std::memory_order_relaxed);
    return;
  }
  dim3 grid(ds.tcount, 1, H);
  seg_gemm<<<grid, kGemmThreads, 0, st>>>(g.d_desc, g.d_tiles + ds.tfirst, A, a_hs, B, b_hs, C,
                                          c_hs, alpha, beta, Cin);
  tt_count_launches(1);
  g_gemm_flops.fetch_add(static_cast<int64_t>(ds.flops * H), std::memory_order_relaxed);
}

// C = A1 B1 + A2 B2 + beta C_in over the dual set `dual_ds` (pairs of ds1's
// and ds2's segments) in one TMA-staged tensor-core launch per chunk, the
// two products accumulating in the same TMEM tile; the CUDA-core GEMM and
// the cp.async staging run the two single sets one after the other instead.
void launch_gemm_dual(GemmCtx& g, DescSet dual_ds, DescSet ds1, DescSet ds2, int H,
                      const float* A1, long long a1_hs, const float* B1, long long b1_hs,
                      const float* A2, long long a2_hs, const float* B2, long long b2_hs,
                      float* C, long long c_hs, float beta, cudaStream_t st,
                      const float* Cin = nullptr) {
  const bool fused = g.split != 0 && g.tma && dual_ds.tc_count > 0 &&
                     tt_gdn_tc_gemm_supported(g.h_desc->data(), ds1.first, ds1.count, A1, a1_hs,
                                              B1, b1_hs, C, c_hs) &&
                     tt_gdn_tc_gemm_supported(g.h_desc->data(), ds2.first, ds2.count, A2, a2_hs,
                                              B2, b2_hs, C, c_hs);
  if (!fused) {
    launch_gemm(g, ds1, H, A1, a1_hs, B1, b1_hs, C, c_hs, 1.f, beta, st, Cin);
    launch_gemm(g, ds2, H, A2, a2_hs, B2, b2_hs, C, c_hs, 1.f, 1.f, st);
    return;
  }
  int launches = 0;
  int t = dual_ds.tc_first;
  const int t_end = dual_ds.tc_first + dual_ds.tc_count;
  // kTmaMaxSegs is even, so no pair straddles two chunks
  static_assert(kTmaMaxSegs % 2 == 0, "dual pairs per launch");
  for (int c0 = 0; c0 < dual_ds.count; c0 += kTmaMaxSegs) {
    const int c1 = std::min(dual_ds.count, c0 + kTmaMaxSegs);
    const int seg_end = dual_ds.first + c1;
    int t1 = t;
    while (t1 < t_end && (*g.h_tiles_tc)[t1].x < seg_end) ++t1;
    const int rc = tt_gdn_seg_gemm_tma(g.h_desc->data() + dual_ds.first + c0,
                                       dual_ds.first + c0, c1 - c0, g.d_desc, g.d_tiles_tc + t,
                                       t1 - t, H, A1, a1_hs, B1, b1_hs, C, c_hs, 1.f, beta, Cin,
                                       g.split, st, EpiMask{},
                                       DualOperands{A2, a2_hs, B2, b2_hs});
    if (rc != TT_OK) g.rc = rc;
    if (t1 > t) ++launches;
    t = t1;
  }
  tt_count_launches(launches);
  g_gemm_flops.fetch_add(static_cast<int64_t>(dual_ds.flops * H), std::memory_order_relaxed);
  g_gemm_tc_flops.fetch_add(static_cast<int64_t>(dual_ds.flops * H), std::memory_order_relaxed);
}

template <typename T>
int run(const Plan& p, bool backward, Arena& ar, const void* q_, const void* k_, const void* v_,
        const float* g, const float* beta, const float* init, int flags, void* out_,
        float* last_state, const void* dout_, const float* dlast, void* dq_, void* dk_,
        void* dv_, float* dg, float* dbeta, float* dinit, cudaStream_t st, int n_cap = 0,
        const int32_t* cap_nodes = nullptr, float* captured = nullptr,
        const float* dcaptured = nullptr) {
  const T* q = (const T*)q_;
  const T* k = (const T*)k_;
  const T* v = (const T*)v_;
  const int l2norm = flags & TT_GDN_QK_L2NORM;
  const bool exact = (flags & TT_GDN_EXACT_INVERSE) != 0;
  const bool reuse = backward && (flags & TT_GDN_SAVED_FORWARD) != 0;
  const int S = p.S, H = p.H, Dk = p.Dk, Dv = p.Dv, n = p.n, Hk = p.Hk;
  const long long q_ts = p.q_ts ? p.q_ts : (long long)Hk * Dk;
  const long long k_ts = p.k_ts ? p.k_ts : (long long)Hk * Dk;
  const long long v_ts = p.v_ts ? p.v_ts : (long long)H * Dv;
  const long long vk = (long long)S * Dk, vv = (long long)S * Dv;   // head strides
  const long long llh = p.ll_total;
  const int DkDv = Dk * Dv;
  const long long sh = (long long)H * DkDv;                           // one state set
  Bufs b{};
  b.gam = ar.get<float>((long long)H * S);
  b.gl_tok = ar.get<float>((long long)H * S);
  b.gl = ar.get<float>((long long)H * n);
  b.Q = ar.get<float>(H * vk); b.K = ar.get<float>(H * vk); b.Vb = ar.get<float>(H * vv);
  b.Kb = ar.get<float>(H * vk); b.Kbg = ar.get<float>(H * vk); b.Qg = ar.get<float>(H * vk);
  b.Kd = ar.get<float>(H * vk); b.U = ar.get<float>(H * vv); b.W = ar.get<float>(H * vk);
  // T1: scratch of the T = I + A + A^2 products, and of the exact inverse's
  // block rows (64 x L per node at offset 64 * start)
  const long long t1_hs = std::max(std::max(vk, vv), 64LL * p.lp_total);
  b.T1 = ar.get<float>(H * t1_hs); b.Vn = ar.get<float>(H * vv);
  b.O = ar.get<float>(H * vv);
  b.KK = ar.get<float>(H * llh); b.QK = ar.get<float>(H * llh);
  b.Am = ar.get<float>(H * llh); b.Aqk = ar.get<float>(H * llh);
  b.states = ar.get<float>((long long)(n + 1) * sh);
  if (backward) {
    b.dO = ar.get<float>(H * vv); b.dVn = ar.get<float>(H * vv); b.dQg = ar.get<float>(H * vk);
    b.dKd = ar.get<float>(H * vk); b.dW = ar.get<float>(H * vk);
    b.dT = ar.get<float>(H * llh); b.dA = ar.get<float>(H * llh); b.dAqk = ar.get<float>(H * llh);
    b.dDD = ar.get<float>(H * llh); b.X = ar.get<float>(H * llh);
    b.dVb = ar.get<float>(H * vv); b.dKbg = ar.get<float>(H * vk); b.dKb = ar.get<float>(H * vk);
    b.dQ = ar.get<float>(H * vk); b.dK = ar.get<float>(H * vk);
    b.dSo = ar.get<float>((long long)n * sh); b.dSi = ar.get<float>((long long)n * sh);
    b.dgl = ar.get<float>((long long)H * n); b.dgam = ar.get<float>((long long)H * S);
    b.kd_dot = ar.get<float>((long long)H * S);
    b.rowsum = ar.get<double>((long long)H * S);
    b.dq_h = ar.get<float>(H * vk); b.dk_h = ar.get<float>(H * vk);
  }
  // metadata + descriptors
  Builder bd(p);
  std::vector<SegDesc> v_kk, v_av, v_ak, v_qs, v_aqv;
  std::vector<std::vector<SegDesc>> lv_ws(p.levels.size()), lv_kdv(p.levels.size());
  for (int c = 0; c < n; ++c) {
    const int L = p.len[c];
    const long long tk = (long long)p.start[c] * Dk, tv = (long long)p.start[c] * Dv;
    const long long lo = p.loff[c];
    const int Lp = row_stride(L);
    // KK = Kb K^T, QK = Q K^T : [L x L], K = Dk (tok0: the decay-mask epilogue)
    v_kk.push_back(desc(L, L, Dk, tk, Dk, 1, tk, 1, Dk, lo, Lp, 1, kKLowerC));
    v_kk.back().tok0 = p.start[c];
    // A * X for X = [L x Dv] (U) / [L x Dk] (W)
    v_av.push_back(desc(L, Dv, L, lo, Lp, 1, tv, Dv, 1, tv, Dv, 1, kKToRow));
    v_ak.push_back(desc(L, Dk, L, lo, Lp, 1, tk, Dk, 1, tk, Dk, 1, kKToRow));
  }
  const long long st_off = sh;   // states[c+1] offset base (per-head stride added by kernel)
  for (size_t d = 0; d < p.levels.size(); ++d) {
    for (int c : p.levels[d]) {
      const int L = p.len[c];
      const long long tk = (long long)p.start[c] * Dk, tv = (long long)p.start[c] * Dv;
      const long long sin = (long long)(p.parent[c] + 1) * st_off;
      const long long sout = (long long)(c + 1) * st_off;
      // Vn -= W S_in : [L x Dv] = [L x Dk][Dk x Dv]
      lv_ws[d].push_back(desc(L, Dv, Dk, tk, Dk, 1, sin, Dv, 1, tv, Dv, 1));
      // O = Qg S_in, then O += Aqk Vn: they read the recurrence's results
      // but feed nothing back into it, so each runs once over every node
      // after the level sweep
      v_qs.push_back(desc(L, Dv, Dk, tk, Dk, 1, sin, Dv, 1, tv, Dv, 1));
      v_aqv.push_back(desc(L, Dv, L, p.loff[c], row_stride(L), 1, tv, Dv, 1, tv, Dv, 1,
                           kKToRow));
      // S_out = Kd^T Vn : [Dk x Dv] = [Dk x L][L x Dv]
      lv_kdv[d].push_back(desc(Dk, Dv, L, tk, 1, Dk, tv, Dv, 1, sout, Dv, 1));
    }
  }
  // exact inverse, block row i >= 1 of each node with more than i blocks:
  //   X = A[i0:i1, 0:i0] T[0:i0, 0:i0] ;  T[i0:i1, 0:i0] = T[i0:i1, i0:i1] X
  // (T's rows above i0 are final by then; X lives in T1 at 64 * start)
  const int max_nb = (p.max_len + kInvB - 1) / kInvB;
  std::vector<int2> inv_blocks;
  std::vector<std::vector<SegDesc>> li_x(std::max(0, max_nb - 1)), li_t(std::max(0, max_nb - 1));
  for (int c = 0; c < n; ++c) {
    const int L = p.len[c];
    const long long lo = p.loff[c], xo = p.xoff[c];
    const int Lp = row_stride(L);
    for (int i = 0; i * kInvB < L; ++i) {
      inv_blocks.push_back(make_int2(c, i));
      if (i == 0) continue;
      const int i0 = i * kInvB, bs = std::min(kInvB, L - i0);
      li_x[i - 1].push_back(desc(bs, i0, i0, lo + (long long)i0 * Lp, Lp, 1, lo, Lp, 1, xo, Lp, 1,
                                 kKFromCol));
      li_t[i - 1].push_back(desc(bs, i0, bs, lo + (long long)i0 * Lp + i0, Lp, 1, xo, Lp, 1,
                                 lo + (long long)i0 * Lp, Lp, 1, kKToRow));
    }
  }
  DescSet ds_kk = bd.add(v_kk), ds_av = bd.add(v_av), ds_ak = bd.add(v_ak);
  std::vector<DescSet> ds_inv_x, ds_inv_t;
  for (int i = 0; i + 1 < max_nb; ++i) {
    ds_inv_x.push_back(bd.add(li_x[i]));
    ds_inv_t.push_back(bd.add(li_t[i]));
  }
  std::vector<DescSet> ds_ws, ds_kdv;
  for (size_t d = 0; d < p.levels.size(); ++d) {
    ds_ws.push_back(bd.add(lv_ws[d]));
    ds_kdv.push_back(bd.add(lv_kdv[d]));
  }
  const DescSet ds_qs = bd.add(v_qs), ds_aqv = bd.add(v_aqv);
  const DescSet dd_o = bd.add_dual(v_qs, v_aqv);   // O = Qg S_in + Aqk Vn in one launch
  // backward descriptors
  std::vector<std::vector<SegDesc>> lb_dvn2(p.levels.size()), lb_dsi2(p.levels.size());
  std::vector<SegDesc> b_dvn1, b_dsi1;
  std::vector<SegDesc> b_dqg, b_dkd, b_dw, b_daqk, b_dt1, b_dt2, b_x1, b_x2, b_tvt, b_tvt2,
      b_tkt, b_tkt2, b_gk, b_gtk, b_fk, b_ftq;
  if (backward) {
    for (size_t d = 0; d < p.levels.size(); ++d) {
      for (int c : p.levels[d]) {
        const int L = p.len[c];
        const long long tk = (long long)p.start[c] * Dk, tv = (long long)p.start[c] * Dv;
        const long long lo = p.loff[c];
        const long long so = (long long)c * st_off;
        // dVn = Aqk^T dO : [L x Dv] = [L x L]^T [L x Dv] (independent of the
        // reverse sweep: once over every node before it)
        b_dvn1.push_back(desc(L, Dv, L, lo, 1, row_stride(L), tv, Dv, 1, tv, Dv, 1, kKFromRow));
        // dVn += Kd dSo : [L x Dv] = [L x Dk][Dk x Dv]
        lb_dvn2[d].push_back(desc(L, Dv, Dk, tk, Dk, 1, so, Dv, 1, tv, Dv, 1));
        // dSi = Qg^T dO : [Dk x Dv] = [Dk x L][L x Dv] (likewise before the sweep)
        b_dsi1.push_back(desc(Dk, Dv, L, tk, 1, Dk, tv, Dv, 1, so, Dv, 1));
        // dSi -= W^T dVn
        lb_dsi2[d].push_back(desc(Dk, Dv, L, tk, 1, Dk, tv, Dv, 1, so, Dv, 1));
      }
    }
    for (int c = 0; c < n; ++c) {
      const int L = p.len[c];
      const long long tk = (long long)p.start[c] * Dk, tv = (long long)p.start[c] * Dv;
      const long long lo = p.loff[c];
      const int Lp = row_stride(L);
      const long long sin = (long long)(p.parent[c] + 1) * st_off;
      const long long so = (long long)c * st_off;
      // dQg = dO S_in^T : [L x Dk] = [L x Dv][Dv x Dk]
      b_dqg.push_back(desc(L, Dk, Dv, tv, Dv, 1, sin, 1, Dv, tk, Dk, 1));
      // dKd = Vn dSo^T
      b_dkd.push_back(desc(L, Dk, Dv, tv, Dv, 1, so, 1, Dv, tk, Dk, 1));
      // dW = -dVn S_in^T
      b_dw.push_back(desc(L, Dk, Dv, tv, Dv, 1, sin, 1, Dv, tk, Dk, 1));
      // dAqk = dO Vn^T : [L x L]
      b_daqk.push_back(desc(L, L, Dv, tv, Dv, 1, tv, 1, Dv, lo, Lp, 1, kKLowerC));
      // dT = dVn Vb^T + dW Kbg^T
      b_dt1.push_back(desc(L, L, Dv, tv, Dv, 1, tv, 1, Dv, lo, Lp, 1, kKLowerC));
      b_dt2.push_back(desc(L, L, Dk, tk, Dk, 1, tk, 1, Dk, lo, Lp, 1, kKLowerC));
      // X = dT A^T : [L x L] = [L x L][L x L]^T ; X += A^T dT
      b_x1.push_back(desc(L, L, L, lo, Lp, 1, lo, 1, Lp, lo, Lp, 1, kKToCol));
      b_x2.push_back(desc(L, L, L, lo, 1, Lp, lo, Lp, 1, lo, Lp, 1, kKFromRow));
      // T^T y = y + A^T y + A^T (A^T y)  for y = dVn [L x Dv] and dW [L x Dk]
      b_tvt.push_back(desc(L, Dv, L, lo, 1, Lp, tv, Dv, 1, tv, Dv, 1, kKFromRow));
      b_tkt.push_back(desc(L, Dk, L, lo, 1, Lp, tk, Dk, 1, tk, Dk, 1, kKFromRow));
      // G K (dKb += G K), G^T Kb (dK += G^T Kb), F K (dQ += F K), F^T Q (dK += F^T Q)
      b_gk.push_back(desc(L, Dk, L, lo, Lp, 1, tk, Dk, 1, tk, Dk, 1, kKToRow));
      b_gtk.push_back(desc(L, Dk, L, lo, 1, Lp, tk, Dk, 1, tk, Dk, 1, kKFromRow));
    }
  }
  DescSet ds_dqg = bd.add(b_dqg), ds_dkd = bd.add(b_dkd), ds_dw = bd.add(b_dw),
          ds_daqk = bd.add(b_daqk), ds_dt1 = bd.add(b_dt1), ds_dt2 = bd.add(b_dt2),
          ds_x1 = bd.add(b_x1), ds_x2 = bd.add(b_x2), ds_tvt = bd.add(b_tvt),
          ds_tkt = bd.add(b_tkt), ds_gk = bd.add(b_gk), ds_gtk = bd.add(b_gtk);
  // products that add into the same output, as dual pairs: dT = dVn Vb^T +
  // dW Kbg^T; dA = dT A^T + A^T dT (+ dT); dK = G^T Kb + F^T Q
  const DescSet dd_dt = bd.add_dual(b_dt1, b_dt2), dd_x = bd.add_dual(b_x1, b_x2),
                dd_gtk = bd.add_dual(b_gtk, b_gtk);
  std::vector<DescSet> ds_dvn2, ds_dsi2;
  for (size_t d = 0; d < p.levels.size(); ++d) {
    ds_dvn2.push_back(bd.add(lb_dvn2[d]));
    ds_dsi2.push_back(bd.add(lb_dsi2[d]));
  }
  const DescSet ds_dvn1 = bd.add(b_dvn1), ds_dsi1 = bd.add(b_dsi1);
  // int metadata
  std::vector<int> level_nodes, level_first;
  for (auto& l : p.levels) {
    level_first.push_back((int)level_nodes.size());
    level_nodes.insert(level_nodes.end(), l.begin(), l.end());
  }
  b.d_tok_node = ar.get<int>(S);
  b.d_start = ar.get<int>(n); b.d_len = ar.get<int>(n); b.d_parent = ar.get<int>(n);
  b.d_child_ptr = ar.get<int>(n + 1); b.d_child_idx = ar.get<int>(std::max<size_t>(1, p.child_idx.size()));
  b.d_roots = ar.get<int>(std::max<size_t>(1, p.roots.size()));
  b.d_level_nodes = ar.get<int>(std::max<size_t>(1, level_nodes.size()));
  b.d_loff = ar.get<long long>(n);
  b.d_desc = ar.get<SegDesc>((long long)bd.all.size());
  b.d_tiles = ar.get<int2>((long long)bd.tiles.size());
  b.d_tiles_tc = ar.get<int2>((long long)bd.tiles_tc.size());
  b.d_inv_blocks = ar.get<int2>(std::max<long long>(1, (long long)inv_blocks.size()));
  b.d_cap_slot = ar.get<int>(n);
  if (ar.sizing) return TT_OK;
  if (ar.used > ar.cap) return TT_ERR_WORKSPACE;
  std::vector<int> cap_slot(n, -1);
  for (int i = 0; i < n_cap; ++i) cap_slot[cap_nodes[i]] = i;
  {
    // the metadata pieces are consecutive arena allocations: one span
    char* span = reinterpret_cast<char*>(b.d_tok_node);
    const size_t span_bytes =
        (size_t)(reinterpret_cast<char*>(b.d_cap_slot) + (((size_t)n * 4 + 255) / 256) * 256 -
                 span);
    const std::vector<MetaPiece> pieces = {
        {b.d_tok_node, p.tok_node.data(), (size_t)S * 4},
        {b.d_start, p.start.data(), (size_t)n * 4},
        {b.d_len, p.len.data(), (size_t)n * 4},
        {b.d_parent, p.parent.data(), (size_t)n * 4},
        {b.d_child_ptr, p.child_ptr.data(), (size_t)(n + 1) * 4},
        {b.d_child_idx, p.child_idx.data(), p.child_idx.size() * 4},
        {b.d_roots, p.roots.data(), p.roots.size() * 4},
        {b.d_level_nodes, level_nodes.data(), level_nodes.size() * 4},
        {b.d_loff, p.loff.data(), (size_t)n * 8},
        {b.d_desc, bd.all.data(), bd.all.size() * sizeof(SegDesc)},
        {b.d_tiles, bd.tiles.data(), bd.tiles.size() * sizeof(int2)},
        {b.d_tiles_tc, bd.tiles_tc.data(), bd.tiles_tc.size() * sizeof(int2)},
        {b.d_inv_blocks, inv_blocks.data(), inv_blocks.size() * sizeof(int2)},
        {b.d_cap_slot, cap_slot.data(), (size_t)n * 4}};
    const int rc = upload_meta(span, span_bytes, pieces, st);
    if (rc != TT_OK) return rc;
  }

  const float q_scale = 1.f / sqrtf((float)Dk);
  const int mode = gemm_mode();
  GemmCtx gc{b.d_desc, b.d_tiles, b.d_tiles_tc, &bd.all, &bd.tiles_tc,
             (mode & 3) == 2 ? 0 : ((mode & 3) == 1 || std::is_same<T, float>::value) ? 3 : 1,
             (mode & 4) == 0};
  // the decay masks ride on the K K^T / Q K^T epilogues when the TMA-staged
  // tensor-core GEMM runs them and A is kept (the exact-inverse mode
  // overwrites it with T)
  const bool fuse_mask = gc.split != 0 && gc.tma && !exact;
  auto blocks = [](long long nel) { return (unsigned)((nel + 255) / 256); };
  int launches = 1;   // the metadata copy
  // ---------------------------------------------------------------- forward
  // (skipped when the workspace still holds this pass from tt_gdn_tree_fwd)
  if (!reuse) {
    node_cumsum<<<dim3((n + 127) / 128, H), 128, 0, st>>>(S, H, n, b.d_start, b.d_len, g, b.gam,
                                                          b.gl_tok, b.gl);
    prep_tokens<T><<<dim3((S + kTokWarps - 1) / kTokWarps, H), 32 * kTokWarps, 0, st>>>(
        S, Hk, H, Dk, Dv, q, k, v, q_ts, k_ts, v_ts, beta, b.gam, b.gl_tok, l2norm, q_scale, b.Q,
        b.K, b.Vb, b.Kb,
        b.Kbg, b.Qg, b.Kd);
    launches += 2;
    if (fuse_mask) {
      // A = -(Kb K^T) * D (strictly lower), Aqk = (Q K^T) * D (lower) straight
      // from the GEMM epilogue
      launch_gemm(gc, ds_kk, H, b.Kb, vk, b.K, vk, b.Am, llh, 1.f, 0.f, st, nullptr,
                  EpiMask{kMaskA, b.gam, (long long)S});
      launch_gemm(gc, ds_kk, H, b.Q, vk, b.K, vk, b.Aqk, llh, 1.f, 0.f, st, nullptr,
                  EpiMask{kMaskAqk, b.gam, (long long)S});
    } else {
      launch_gemm(gc, ds_kk, H, b.Kb, vk, b.K, vk, b.KK, llh, 1.f, 0.f, st);
      launch_gemm(gc, ds_kk, H, b.Q, vk, b.K, vk, b.QK, llh, 1.f, 0.f, st);
      decay_masks<<<dim3(S, H), 128, 0, st>>>(S, b.d_start, b.d_len, b.d_tok_node, b.d_loff, llh,
                                               b.gam, b.KK, b.QK, b.Am, b.Aqk);
      ++launches;
    }
    if (exact) {
      // Am <- T = (I - A)^-1 in place: diagonal blocks, then block rows in order
      tri_inv_diag<<<dim3((unsigned)inv_blocks.size(), H), kInvB, 0, st>>>(
          b.d_inv_blocks, b.d_len, b.d_loff, llh, b.Am);
      ++launches;
      for (size_t i = 0; i < ds_inv_x.size(); ++i) {
        launch_gemm(gc, ds_inv_x[i], H, b.Am, llh, b.Am, llh, b.T1, t1_hs, 1.f,
                    0.f, st);
        launch_gemm(gc, ds_inv_t[i], H, b.Am, llh, b.T1, t1_hs, b.Am, llh, 1.f,
                    0.f, st);
      }
      // U = T Vb;  W = T Kbg
      launch_gemm(gc, ds_av, H, b.Am, llh, b.Vb, vv, b.U, vv, 1.f, 0.f, st);
      launch_gemm(gc, ds_ak, H, b.Am, llh, b.Kbg, vk, b.W, vk, 1.f, 0.f, st);
    } else {
      // U = T Vb = Vb + A (Vb + A Vb);  W = T Kbg likewise (T = I + A + A^2):
      // T1 = X + A X first, then X + A T1, both as GEMMs with X as the
      // epilogue's input (T1 has head stride vv / vk here)
      launch_gemm(gc, ds_av, H, b.Am, llh, b.Vb, vv, b.T1, vv, 1.f, 1.f, st, b.Vb);
      launch_gemm(gc, ds_av, H, b.Am, llh, b.T1, vv, b.U, vv, 1.f, 1.f, st, b.Vb);
      launch_gemm(gc, ds_ak, H, b.Am, llh, b.Kbg, vk, b.T1, vk, 1.f, 1.f, st, b.Kbg);
      launch_gemm(gc, ds_ak, H, b.Am, llh, b.T1, vk, b.W, vk, 1.f, 1.f, st, b.Kbg);
    }
    init_state<<<blocks(sh), 256, 0, st>>>(sh, init, b.states);
    ++launches;
    for (size_t d = 0; d < p.levels.size(); ++d) {
      const int cnt = (int)p.levels[d].size();
      // states are [n+1][H][Dk][Dv]: per-head stride DkDv, segment offsets cover (c+1)*H*DkDv
      // Vn = U - W S_in (every node's rows are written by its own level)
      launch_gemm(gc, ds_ws[d], H, b.W, vk, b.states, DkDv, b.Vn, vv, -1.f, 1.f, st, b.U);
      launch_gemm(gc, ds_kdv[d], H, b.Kd, vk, b.Vn, vv, b.states, DkDv, 1.f, 0.f, st);
      state_decay_add<<<dim3(std::max(1, DkDv / 1024), cnt, H), 256, 0, st>>>(
          H, DkDv, n, b.d_level_nodes + level_first[d], b.d_parent, b.gl, b.states);
      ++launches;
    }
    if (!backward) {   // the output; the backward (which recomputes this pass) never reads it
      launch_gemm_dual(gc, dd_o, ds_qs, ds_aqv, H, b.Qg, vk, b.states, DkDv, b.Aqk, llh, b.Vn,
                       vv, b.O, vv, 0.f, st);
    }
  }
  if (!backward) {
    store_out<T><<<dim3((S + kTokWarps - 1) / kTokWarps, H), 32 * kTokWarps, 0, st>>>(S, H, Dv, b.O, (T*)out_);
    ++launches;
    if (last_state) {
      TT_CUDA_OK(cudaMemcpyAsync(last_state, b.states + (long long)n * sh, sh * 4,
                                 cudaMemcpyDeviceToDevice, st));
    }
    for (int i = 0; i < n_cap && captured; ++i)   // state after each captured node
      TT_CUDA_OK(cudaMemcpyAsync(captured + (long long)i * sh,
                                 b.states + (long long)(cap_nodes[i] + 1) * sh, sh * 4,
                                 cudaMemcpyDeviceToDevice, st));
    tt_count_launches(launches);
    if (gc.rc != TT_OK) return gc.rc;
    return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
  }
  // ---------------------------------------------------------------- backward
  load_dout<T><<<dim3((S + kTokWarps - 1) / kTokWarps, H), 32 * kTokWarps, 0, st>>>(S, H, Dv, (const T*)dout_, b.dO);
  ++launches;
  launch_gemm(gc, ds_dvn1, H, b.Aqk, llh, b.dO, vv, b.dVn, vv, 1.f, 0.f, st);
  launch_gemm(gc, ds_dsi1, H, b.Qg, vk, b.dO, vv, b.dSi, DkDv, 1.f, 0.f, st);
  for (int d = (int)p.levels.size() - 1; d >= 0; --d) {
    const int cnt = (int)p.levels[d].size();
    gather_dstate<<<dim3(std::max(1, DkDv / 1024), cnt, H), 256, 0, st>>>(
        H, DkDv, n, b.d_level_nodes + level_first[d], b.d_child_ptr, b.d_child_idx, b.dSi, dlast,
        b.d_cap_slot, dcaptured, b.dSo);
    launch_gemm(gc, ds_dvn2[d], H, b.Kd, vk, b.dSo, DkDv, b.dVn, vv, 1.f, 1.f, st);
    launch_gemm(gc, ds_dsi2[d], H, b.W, vk, b.dVn, vv, b.dSi, DkDv, -1.f, 1.f, st);
    dstate_decay<<<dim3(cnt, H), 1024, 0, st>>>(H, DkDv, n, b.d_level_nodes + level_first[d],
                                               b.d_parent, b.gl, b.states, b.dSo, b.dSi, b.dgl);
    launches += 2;
  }
  // per-node gradients, no more dependencies between nodes
  launch_gemm(gc, ds_dqg, H, b.dO, vv, b.states, DkDv, b.dQg, vk, 1.f, 0.f, st);
  launch_gemm(gc, ds_dkd, H, b.Vn, vv, b.dSo, DkDv, b.dKd, vk, 1.f, 0.f, st);
  launch_gemm(gc, ds_dw, H, b.dVn, vv, b.states, DkDv, b.dW, vk, -1.f, 0.f, st);
  launch_gemm(gc, ds_daqk, H, b.dO, vv, b.Vn, vv, b.dAqk, llh, 1.f, 0.f, st);
  launch_gemm_dual(gc, dd_dt, ds_dt1, ds_dt2, H, b.dVn, vv, b.Vb, vv, b.dW, vk, b.Kbg, vk, b.dT,
                   llh, 0.f, st);
  if (exact) {
    // Am holds T = (I - A)^-1:  dA = T^T dT T^T (masked in grad_masks);
    // dVb = T^T dVn;  dKbg = T^T dW
    launch_gemm(gc, ds_x2, H, b.Am, llh, b.dT, llh, b.X, llh, 1.f, 0.f, st);
    launch_gemm(gc, ds_x1, H, b.X, llh, b.Am, llh, b.dA, llh, 1.f, 0.f, st);
    launch_gemm(gc, ds_tvt, H, b.Am, llh, b.dVn, vv, b.dVb, vv, 1.f, 0.f, st);
    launch_gemm(gc, ds_tkt, H, b.Am, llh, b.dW, vk, b.dKbg, vk, 1.f, 0.f, st);
  } else {
    // dA = dT + dT A^T + A^T dT  (masked in grad_masks)
    launch_gemm_dual(gc, dd_x, ds_x1, ds_x2, H, b.dT, llh, b.Am, llh, b.Am, llh, b.dT, llh,
                     b.dA, llh, 1.f, st, b.dT);
    // dVb = T^T dVn = dVn + A^T (dVn + A^T dVn);  dKbg = T^T dW likewise
    launch_gemm(gc, ds_tvt, H, b.Am, llh, b.dVn, vv, b.T1, vv, 1.f, 1.f, st, b.dVn);
    launch_gemm(gc, ds_tvt, H, b.Am, llh, b.T1, vv, b.dVb, vv, 1.f, 1.f, st, b.dVn);
    launch_gemm(gc, ds_tkt, H, b.Am, llh, b.dW, vk, b.T1, vk, 1.f, 1.f, st, b.dW);
    launch_gemm(gc, ds_tkt, H, b.Am, llh, b.T1, vk, b.dKbg, vk, 1.f, 1.f, st, b.dW);
  }
  // masks: dA -> G = -dA*D, dAqk -> F = dAqk*D, dDD
  TT_CUDA_OK(cudaMemsetAsync(b.dgam, 0, (size_t)H * S * 4, st));
  if (p.max_len <= kFusedMaskMaxL) {
    // one pass: G, F and the row / column sums of dDD without storing it
    const size_t smem = (size_t)(kRowColThreads / 32 + 1) * std::max(p.max_len, 1) * 8;
    if (smem > 48 * 1024)
      TT_CUDA_OK(cudaFuncSetAttribute(grad_masks_rowcol,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    grad_masks_rowcol<<<dim3(n, H), kRowColThreads, smem, st>>>(
        S, b.d_start, b.d_len, b.d_loff, llh, b.gam, fuse_mask ? b.Am : b.KK,
        fuse_mask ? b.Aqk : b.QK, fuse_mask ? 1 : 0, b.dA, b.dAqk, b.dgam);
    launches += 1;
  } else {
    grad_masks<<<dim3(S, H), 128, 0, st>>>(S, b.d_start, b.d_len, b.d_tok_node, b.d_loff, llh,
                                              b.gam, fuse_mask ? b.Am : b.KK,
                                              fuse_mask ? b.Aqk : b.QK, fuse_mask ? 1 : 0, b.dA,
                                              b.dAqk, b.dDD);
    ddd_rowcol<<<dim3(n, H), kRowColThreads, 0, st>>>(S, b.d_start, b.d_len, b.d_loff, llh,
                                                       b.dDD, b.rowsum, b.dgam);
    launches += 2;
  }
  // dKb = G K ; dK = G^T Kb + F^T Q ; dQ = F K
  launch_gemm(gc, ds_gk, H, b.dA, llh, b.K, vk, b.dKb, vk, 1.f, 0.f, st);
  launch_gemm_dual(gc, dd_gtk, ds_gtk, ds_gtk, H, b.dA, llh, b.Kb, vk, b.dAqk, llh, b.Q, vk,
                   b.dK, vk, 0.f, st);
  launch_gemm(gc, ds_gk, H, b.dAqk, llh, b.K, vk, b.dQ, vk, 1.f, 0.f, st);
  kd_dot_kernel<<<dim3((S + kTokWarps - 1) / kTokWarps, H), 32 * kTokWarps, 0, st>>>(S, Dk, b.Kd, b.dKd, b.kd_dot);
  {
    auto asm_kernel = Dk == 128 ? assemble_token_grads<T, 4> : assemble_token_grads<T, 0>;
    asm_kernel<<<dim3((S + kTokWarps - 1) / kTokWarps, H), 32 * kTokWarps, 0, st>>>(
        S, Hk, H, Dk, Dv, q, k, v, q_ts, k_ts, v_ts, beta, b.gam, b.gl_tok, l2norm, q_scale, b.dQ,
        b.dQg, b.dK, b.dKd, b.dKb, b.dKbg, b.dVb, b.dgam, b.dq_h, b.dk_h, dbeta, (T*)dv_);
  }
  node_dg<<<dim3((n + 127) / 128, H), 128, 0, st>>>(S, H, n, b.d_start, b.d_len, b.kd_dot, b.dgl,
                                                    b.dgam, dg);
  const auto al = [](const void* ptr, int a) { return reinterpret_cast<uintptr_t>(ptr) % a == 0; };
  if (Dk % 4 == 0 && al(b.dq_h, 16) && al(b.dk_h, 16) && al(dq_, 4 * sizeof(T)) &&
      al(dk_, 4 * sizeof(T))) {
    const long long n4 = (long long)S * Hk * (Dk / 4);
    reduce_gqa4<T><<<dim3((unsigned)((n4 + 255) / 256), 2), 256, 0, st>>>(
        S, Hk, H, Dk, b.dq_h, (T*)dq_, b.dk_h, (T*)dk_);
    launches += 4;
  } else {
    reduce_gqa<T><<<dim3((S + kTokWarps - 1) / kTokWarps, Hk), 32 * kTokWarps, 0, st>>>(
        S, Hk, H, Dk, b.dq_h, (T*)dq_);
    reduce_gqa<T><<<dim3((S + kTokWarps - 1) / kTokWarps, Hk), 32 * kTokWarps, 0, st>>>(
        S, Hk, H, Dk, b.dk_h, (T*)dk_);
    launches += 5;
  }
  if (dinit) {
    dinit_kernel<<<blocks(sh), 256, 0, st>>>(H, DkDv, (int)p.roots.size(), b.d_roots, b.dSi, dinit);
    ++launches;
  }
  tt_count_launches(launches);
  if (gc.rc != TT_OK) return gc.rc;
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

template <typename Fn>
int dispatch(int dtype, Fn fn) {
  switch (dtype) {
    case TT_F32: return fn(float());
    case TT_BF16: return fn(__nv_bfloat16());
    case TT_F16: return fn(__half());
    default: return TT_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace gdn
}  // namespace tt

using tt::gdn::Arena;
using tt::gdn::Plan;

extern "C" int64_t tt_gdn_segmented_gemm_workspace_size(int32_t n_segs, const int64_t* segs) {
  if (n_segs < 0 || (n_segs > 0 && !segs)) return -1;
  int64_t tiles = 0;
  for (int i = 0; i < n_segs; ++i) {
    const int64_t M = segs[13 * i], N = segs[13 * i + 1];
    if (M < 0 || N < 0 || M > 65535 * 64 || N > 65535 * 64) return -1;
    tiles += ((M + 63) / 64) * ((N + 63) / 64);
  }
  return ((int64_t)n_segs * (int64_t)sizeof(tt::gdn::SegDesc) + 255) / 256 * 256 +
         (tiles * 8 + 255) / 256 * 256 * 2;
}

extern "C" int tt_gdn_segmented_gemm(int engine, int32_t n_segs, const int64_t* segs, int32_t H,
                                     const float* A, int64_t a_hs, const float* B, int64_t b_hs,
                                     float* C, int64_t c_hs, float alpha, float beta,
                                     void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace tt::gdn;
  if (engine < 0 || engine > 7 || (engine & 3) == 2 || engine == 4 || n_segs < 0 || H <= 0 ||
      (n_segs > 0 && (!segs || !A || !B || !C)))
    return TT_ERR_INVALID_ARG;
  const int64_t need = tt_gdn_segmented_gemm_workspace_size(n_segs, segs);
  if (need < 0) return TT_ERR_INVALID_ARG;
  if (workspace_bytes < need || (n_segs > 0 && !workspace)) return TT_ERR_WORKSPACE;
  if (n_segs == 0) return TT_OK;
  Plan dummy;
  Builder bd(dummy);
  std::vector<SegDesc> v(n_segs);
  for (int i = 0; i < n_segs; ++i) {
    const int64_t* e = segs + 13 * i;
    if (e[2] < 0 || e[3] < kKFull || e[3] > kKFromCol) return TT_ERR_INVALID_ARG;
    v[i] = desc((int)e[0], (int)e[1], (int)e[2], e[4], e[5], e[6], e[7], e[8], e[9], e[10],
                e[11], e[12], (int)e[3]);
  }
  const DescSet ds = bd.add(v);
  Arena ar{(char*)workspace, workspace_bytes, 0, false};
  SegDesc* d_desc = ar.get<SegDesc>(n_segs);
  int2* d_tiles = ar.get<int2>((long long)bd.tiles.size());
  int2* d_tiles_tc = ar.get<int2>((long long)bd.tiles_tc.size());
  cudaStream_t st = (cudaStream_t)stream;
  TT_CUDA_OK(cudaMemcpyAsync(d_desc, bd.all.data(), n_segs * sizeof(SegDesc),
                             cudaMemcpyHostToDevice, st));
  if (!bd.tiles.empty())
    TT_CUDA_OK(cudaMemcpyAsync(d_tiles, bd.tiles.data(), bd.tiles.size() * sizeof(int2),
                               cudaMemcpyHostToDevice, st));
  if (!bd.tiles_tc.empty())
    TT_CUDA_OK(cudaMemcpyAsync(d_tiles_tc, bd.tiles_tc.data(), bd.tiles_tc.size() * sizeof(int2),
                               cudaMemcpyHostToDevice, st));
  // engine 0 = CUDA cores; 1 / 3 = tensor cores with TF32 / 3xTF32 products
  GemmCtx gc{d_desc, d_tiles, d_tiles_tc, &bd.all, &bd.tiles_tc, engine & 3, (engine & 4) == 0};
  if ((engine & 3) != 0 && !tt_gdn_tc_gemm_supported(bd.all.data(), 0, n_segs, A, a_hs, B, b_hs, C, c_hs))
    return TT_ERR_UNSUPPORTED;
  launch_gemm(gc, ds, H, A, a_hs, B, b_hs, C, c_hs, alpha, beta, st);
  if (gc.rc != TT_OK) return gc.rc;
  TT_CUDA_OK(cudaStreamSynchronize(st));
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

extern "C" int64_t tt_gdn_tree_workspace_size(int32_t S, int32_t H, int32_t Dk, int32_t Dv,
                                              int32_t n_nodes, const int32_t* bounds,
                                              int backward) {
  if (S < 0 || H <= 0 || Dk <= 0 || Dv <= 0 || n_nodes < 0 || (n_nodes > 0 && !bounds)) return -1;
  std::vector<int32_t> parents(n_nodes, -1);
  Plan p;
  if (tt::gdn::make_plan(p, S, H, 1, Dk, Dv, n_nodes, bounds, parents.data()) != TT_OK) return -1;
  Arena ar{nullptr, 0, 0, true};
  tt::gdn::run<float>(p, backward != 0, ar, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                      0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                      nullptr, nullptr, nullptr);
  // every level holds at least one node; descriptor count does not depend on
  // the parents beyond the level split, so size it for the worst case (a chain)
  return ar.used + (int64_t)(n_nodes + 1) * 4 * (int64_t)sizeof(tt::gdn::SegDesc) * 2 + 4096;
}

static int gdn_check(int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv, int32_t n_nodes,
                     const int32_t* bounds, const int32_t* parents, int flags) {
  if ((flags & ~(TT_GDN_QK_L2NORM | TT_GDN_EXACT_INVERSE | TT_GDN_SAVED_FORWARD)) != 0 || S < 0 || Hk <= 0 || H <= 0 || H % Hk || Dk <= 0 || Dv <= 0 || Dk > 256 || Dv > 256 ||
      n_nodes < 0 || (n_nodes > 0 && (!bounds || !parents)))
    return TT_ERR_INVALID_ARG;
  return TT_OK;
}

// q / k / v token strides: 0 (packed) or at least one packed row, so the rows
// of different tokens never overlap
static int gdn_check_strides(int32_t Hk, int32_t H, int32_t Dk, int32_t Dv, int64_t q_ts,
                             int64_t k_ts, int64_t v_ts) {
  const int64_t qk_row = (int64_t)Hk * Dk, v_row = (int64_t)H * Dv;
  if ((q_ts != 0 && q_ts < qk_row) || (k_ts != 0 && k_ts < qk_row) || (v_ts != 0 && v_ts < v_row))
    return TT_ERR_INVALID_ARG;
  return TT_OK;
}

static int gdn_check_capture(int32_t n_nodes, int32_t n_capture, const int32_t* capture_nodes) {
  if (n_capture < 0 || (n_capture > 0 && !capture_nodes)) return TT_ERR_INVALID_ARG;
  std::vector<char> seen(n_nodes, 0);
  for (int i = 0; i < n_capture; ++i) {
    const int c = capture_nodes[i];
    if (c < 0 || c >= n_nodes || seen[c]) return TT_ERR_INVALID_ARG;
    seen[c] = 1;
  }
  return TT_OK;
}

extern "C" int tt_gdn_tree_fwd_ex(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk,
                                  int32_t Dv, const void* q, const void* k, const void* v,
                                  const float* g, const float* beta, int32_t n_nodes,
                                  const int32_t* bounds, const int32_t* parents,
                                  const float* initial_state, int flags, void* out,
                                  float* last_state, int32_t n_capture,
                                  const int32_t* capture_nodes, float* captured,
                                  int64_t q_token_stride, int64_t k_token_stride,
                                  int64_t v_token_stride, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  int rc = gdn_check(S, Hk, H, Dk, Dv, n_nodes, bounds, parents, flags);
  if (rc != TT_OK) return rc;
  if ((rc = gdn_check_capture(n_nodes, n_capture, capture_nodes)) != TT_OK) return rc;
  if (n_capture > 0 && !captured) return TT_ERR_INVALID_ARG;
  if ((rc = gdn_check_strides(Hk, H, Dk, Dv, q_token_stride, k_token_stride,
                              v_token_stride)) != TT_OK)
    return rc;
  if (S == 0 || n_nodes == 0) return TT_OK;
  Plan p;
  if ((rc = tt::gdn::make_plan(p, S, H, Hk, Dk, Dv, n_nodes, bounds, parents)) != TT_OK) return rc;
  p.q_ts = q_token_stride;
  p.k_ts = k_token_stride;
  p.v_ts = v_token_stride;
  Arena ar{(char*)workspace, workspace_bytes, 0, false};
  return tt::gdn::dispatch(dtype, [&](auto tag) {
    using T = decltype(tag);
    return tt::gdn::run<T>(p, false, ar, q, k, v, g, beta, initial_state, flags, out,
                           last_state, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                           nullptr, nullptr, (cudaStream_t)stream, n_capture, capture_nodes,
                           captured, nullptr);
  });
}

extern "C" int tt_gdn_tree_fwd(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                               const void* q, const void* k, const void* v, const float* g,
                               const float* beta, int32_t n_nodes, const int32_t* bounds,
                               const int32_t* parents, const float* initial_state,
                               int flags, void* out, float* last_state, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  return tt_gdn_tree_fwd_ex(dtype, S, Hk, H, Dk, Dv, q, k, v, g, beta, n_nodes, bounds, parents,
                            initial_state, flags, out, last_state, 0, nullptr, nullptr, 0, 0, 0,
                            workspace, workspace_bytes, stream);
}

extern "C" int tt_gdn_tree_bwd_ex(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk,
                                  int32_t Dv, const void* q, const void* k, const void* v,
                                  const float* g, const float* beta, int32_t n_nodes,
                                  const int32_t* bounds, const int32_t* parents,
                                  const float* initial_state, int flags, const void* dout,
                                  const float* dlast, int32_t n_capture,
                                  const int32_t* capture_nodes, const float* dcaptured, void* dq,
                                  void* dk, void* dv, float* dg, float* dbeta, float* dinit,
                                  int64_t q_token_stride, int64_t k_token_stride,
                                  int64_t v_token_stride, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  int rc = gdn_check(S, Hk, H, Dk, Dv, n_nodes, bounds, parents, flags);
  if (rc != TT_OK) return rc;
  if ((rc = gdn_check_capture(n_nodes, n_capture, capture_nodes)) != TT_OK) return rc;
  if ((rc = gdn_check_strides(Hk, H, Dk, Dv, q_token_stride, k_token_stride,
                              v_token_stride)) != TT_OK)
    return rc;
  if (S == 0 || n_nodes == 0) return TT_OK;
  Plan p;
  if ((rc = tt::gdn::make_plan(p, S, H, Hk, Dk, Dv, n_nodes, bounds, parents)) != TT_OK) return rc;
  p.q_ts = q_token_stride;
  p.k_ts = k_token_stride;
  p.v_ts = v_token_stride;
  Arena ar{(char*)workspace, workspace_bytes, 0, false};
  return tt::gdn::dispatch(dtype, [&](auto tag) {
    using T = decltype(tag);
    return tt::gdn::run<T>(p, true, ar, q, k, v, g, beta, initial_state, flags, nullptr,
                           nullptr, dout, dlast, dq, dk, dv, dg, dbeta, dinit,
                           (cudaStream_t)stream, n_capture, capture_nodes, nullptr,
                           n_capture > 0 ? dcaptured : nullptr);
  });
}

extern "C" int tt_gdn_tree_bwd(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                               const void* q, const void* k, const void* v, const float* g,
                               const float* beta, int32_t n_nodes, const int32_t* bounds,
                               const int32_t* parents, const float* initial_state,
                               int flags, const void* dout, const float* dlast, void* dq,
                               void* dk, void* dv, float* dg, float* dbeta, float* dinit,
                               void* workspace, int64_t workspace_bytes, void* stream) {
  return tt_gdn_tree_bwd_ex(dtype, S, Hk, H, Dk, Dv, q, k, v, g, beta, n_nodes, bounds, parents,
                            initial_state, flags, dout, dlast, 0, nullptr, nullptr, dq, dk, dv,
                            dg, dbeta, dinit, 0, 0, 0, workspace, workspace_bytes, stream);
}

extern "C" int64_t tt_gdn_gemm_flops(void) {
  return tt::gdn::g_gemm_flops.load(std::memory_order_relaxed);
}

extern "C" int64_t tt_gdn_gemm_tc_flops(void) {
  return tt::gdn::g_gemm_tc_flops.load(std::memory_order_relaxed);
}

extern "C" int tt_gdn_set_gemm_mode(int mode) {
  const int prev = tt::gdn::gemm_mode();
  mode &= 7;
  tt::gdn::g_gemm_mode.store((mode & 3) == 3 ? 0 : mode);
  return prev;
}
