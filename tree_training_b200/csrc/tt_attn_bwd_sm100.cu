// Tree attention backward on the 5th-generation tensor cores (sm_100a).
//
// The gradient torch autograd takes through the reference's SDPA call
// (loss.backward() at tree_grad_hybrid.py:533-535 / tree_grad_ckpt.py:107),
// computed without atomics in two kernels that recompute P from the saved
// row log-sum-exp:
//
//   dK/dV kernel  one CTA per (kv head, 128-key tile); loops over the q heads
//                 of its GQA group and the q tiles the work list marks
//                 visible.  S^T = K Q^T and dP^T = V dO^T (A, B from shared
//                 memory); the softmax warps turn them into P^T and
//                 dS^T = P^T (dP^T - delta) and store both back into TMEM as
//                 16-bit; then dV += P^T dO and dK += dS^T Q read A from TMEM.
//   dQ kernel     one CTA per (q head, 128-row tile), the forward's loop:
//                 S = Q K^T, dP = dO V^T, dS = P (dP - delta) into TMEM,
//                 dQ += dS K.
//
// TMEM (512 columns): dK/dV kernel S^T|P^T [0,128), dP^T|dS^T [128,256),
// dV [256,384), dK [384,512); dQ kernel S|dS [0,128), dP [128,256),
// dQ [256,384).  Warp roles as in the forward: warp 0 TMA, warp 1 MMA,
// warps 2-5 elementwise (one thread per TMEM lane).
#include <type_traits>

#include "tt_sm100.cuh"

namespace tt {
namespace sm100 {
namespace {

constexpr int kT = 128;                   // rows per tile (keys or queries)
constexpr int kD = 128;                   // head dim
constexpr int kTileBytes = kT * kD * 2;
constexpr int kHalfBytes = kTileBytes / 2;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdBarriers {
  uint64_t fixed_full;      // the tiles loaded once (K,V or Q,dO)
  uint64_t a_full[2];       // streamed tile A (Q or K)
  uint64_t b_full[2];       // streamed tile B (dO or V)
  uint64_t ab_empty[2];
  uint64_t sdp_full;        // S and dP accumulators ready
  uint64_t ew_full;         // P / dS written back to TMEM (128 arrivals)
  uint64_t acc_done;        // every MMA of the CTA finished
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

constexpr size_t kSmemBytes = 1024 + 6 * kTileBytes + sizeof(BwdBarriers);

__device__ __forceinline__ void raise_abort(BwdBarriers* sh, int32_t* status) {
  set_status(status, TT_ERR_DEVICE_TIMEOUT);
  *reinterpret_cast<volatile int32_t*>(&sh->abort) = 1;
}

__device__ __forceinline__ void init_barriers(BwdBarriers* sh) {
  mbar_init(&sh->fixed_full, 1);
  for (int s = 0; s < 2; ++s) {
    mbar_init(&sh->a_full[s], 1);
    mbar_init(&sh->b_full[s], 1);
    mbar_init(&sh->ab_empty[s], 1);
  }
  mbar_init(&sh->sdp_full, 1);
  mbar_init(&sh->ew_full, 128);
  mbar_init(&sh->acc_done, 1);
  mbar_init(&sh->drain, 1);
  sh->abort = 0;
  fence_mbar_init();
}

// 128x128 (K = 128) product of two K-major 128-byte-swizzled smem tiles.
__device__ __forceinline__ void mma_tile_ss(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr,
                                            uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
    mma_ss(d_tmem, desc_sw128(a_addr + off, 16, 1024), desc_sw128(b_addr + off, 16, 1024), idesc,
           kk > 0 ? 1u : 0u);
  }
}

// D[128 x 128] (+)= A[128 x 128 from TMEM, 16-bit] * B, B an MN-major smem
// tile [K rows][128] (K = 128 rows of 128 dims).
__device__ __forceinline__ void mma_tile_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr,
                                            uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kT / 16; ++kk)
    mma_ts(d_tmem, a_tmem + kk * 8, desc_sw128(b_addr + kk * 2048, kHalfBytes, 1024), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

template <bool kBf16>
__device__ __forceinline__ void store_row32(void* base, const float (&v)[32], float mul) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack2<kBf16>(v[2 * i] * mul, v[2 * i + 1] * mul);
  uint4* dst = reinterpret_cast<uint4*>(base);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

// ===================================================================== dK/dV
template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dkdv_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                 int n_q, int n_kv, int rep, const int32_t* __restrict__ kv_lo,
                 const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ bwd_ptr,
                 const int32_t* __restrict__ bwd_list, const float* __restrict__ lse,
                 const float* __restrict__ delta, float scale_log2, float scale,
                 void* __restrict__ dk_, int64_t dk_st, int64_t dk_sh, void* __restrict__ dv_,
                 int64_t dv_st, int64_t dv_sh, int32_t* status) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sK = base;
  uint8_t* sV = sK + kTileBytes;
  uint8_t* sQ = sV + kTileBytes;           // 2 stages
  uint8_t* sDO = sQ + 2 * kTileBytes;      // 2 stages
  BwdBarriers* sh = reinterpret_cast<BwdBarriers*>(sDO + 2 * kTileBytes);
  const volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.x;
  const int kt = blockIdx.y;                 // root-side tiles (longest lists) first
  const int e0 = bwd_ptr[kt];
  const int n_list = bwd_ptr[kt + 1] - e0;
  const int n_it = rep * n_list;
  const int ld = lse_ld(n_q);

  if (threadIdx.x == 0) init_barriers(sh);
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_do);
      mbar_arrive_expect_tx(&sh->fixed_full, 2 * kTileBytes);
      tma_load_3d(sK, &tm_k, &sh->fixed_full, 0, kt * kT, hk);
      tma_load_3d(sK + kHalfBytes, &tm_k, &sh->fixed_full, 64, kt * kT, hk);
      tma_load_3d(sV, &tm_v, &sh->fixed_full, 0, kt * kT, hk);
      tma_load_3d(sV + kHalfBytes, &tm_v, &sh->fixed_full, 64, kt * kT, hk);
      int issued[2] = {0, 0};
      bool ok = true;
      for (int it = 0; it < n_it; ++it) {
        const int s = it & 1;
        if (it >= 2) ok = mbar_wait(&sh->ab_empty[s], ((it >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        const int h = hk * rep + it / n_list;
        const int qt = bwd_list[e0 + it % n_list] >> 1;
        uint8_t* q_dst = sQ + s * kTileBytes;
        uint8_t* o_dst = sDO + s * kTileBytes;
        mbar_arrive_expect_tx(&sh->a_full[s], kTileBytes);
        tma_load_3d(q_dst, &tm_q, &sh->a_full[s], 0, qt * kT, h);
        tma_load_3d(q_dst + kHalfBytes, &tm_q, &sh->a_full[s], 64, qt * kT, h);
        mbar_arrive_expect_tx(&sh->b_full[s], kTileBytes);
        tma_load_3d(o_dst, &tm_do, &sh->b_full[s], 0, qt * kT, h);
        tma_load_3d(o_dst + kHalfBytes, &tm_do, &sh->b_full[s], 64, qt * kT, h);
        issued[s] += 1;
      }
      if (!ok) {
        raise_abort(sh, status);
        mbar_wait(&sh->fixed_full, 0, nullptr);
        for (int s = 0; s < 2; ++s)
          if (issued[s] > 0) {
            mbar_wait(&sh->a_full[s], (issued[s] - 1) & 1, nullptr);
            mbar_wait(&sh->b_full[s], (issued[s] - 1) & 1, nullptr);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t id_ss = idesc_f16(kBf16, kT, kT, false);
      constexpr uint32_t id_ts = idesc_f16(kBf16, kT, kD, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      const uint32_t q_addr = smem_u32(sQ), o_addr = smem_u32(sDO);
      bool ok = mbar_wait(&sh->fixed_full, 0, abort_flag);
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it & 1;
        ok = mbar_wait(&sh->a_full[s], (it >> 1) & 1, abort_flag);
        if (ok) ok = mbar_wait(&sh->b_full[s], (it >> 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        mma_tile_ss(tmem + kColS, k_addr, q_addr + s * kTileBytes, id_ss);    // S^T = K Q^T
        mma_tile_ss(tmem + kColDP, v_addr, o_addr + s * kTileBytes, id_ss);   // dP^T = V dO^T
        tc_commit(&sh->sdp_full);
        ok = mbar_wait(&sh->ew_full, it & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        mma_tile_ts(tmem + kColDV, tmem + kColS, o_addr + s * kTileBytes, id_ts, it > 0);
        mma_tile_ts(tmem + kColDK, tmem + kColDP, q_addr + s * kTileBytes, id_ts, it > 0);
        tc_commit(&sh->ab_empty[s]);
      }
      tc_commit(&sh->acc_done);
      if (!ok) {
        raise_abort(sh, status);
        tc_commit(&sh->drain);
        mbar_wait(&sh->drain, 0, nullptr);
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;          // key within the tile = TMEM lane
    const int j = kt * kT + r;
    const int lo = j < n_kv ? kv_lo[j] : 0;
    const int hi = j < n_kv ? kv_hi[j] : 0;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int h = hk * rep + it / n_list;
      const int ent = bwd_list[e0 + it % n_list];
      const int q0 = (ent >> 1) * kT;
      const bool partial = ent & 1;
      const float4* lse4 = reinterpret_cast<const float4*>(lse + static_cast<int64_t>(h) * ld + q0);
      const float4* del4 = reinterpret_cast<const float4*>(delta + static_cast<int64_t>(h) * ld + q0);
      ok = mbar_wait(&sh->sdp_full, it & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kT / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld32(lane_addr + kColS + c * 32, sv);
        tmem_ld32(lane_addr + kColDP + c * 32, dp);
        uint32_t pw[16], dw[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 l4 = __ldg(lse4 + c * 8 + i);
          const float4 d4 = __ldg(del4 + c * 8 + i);
          const float la[4] = {l4.x, l4.y, l4.z, l4.w};
          const float da[4] = {d4.x, d4.y, d4.z, d4.w};
          float p[4], ds[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = c * 32 + i * 4 + u;
            float pv = exp2f(fmaf(sv[i * 4 + u], scale_log2, -la[u] * kLog2e));
            if (partial && !visible(lo, hi, q0 + col)) pv = 0.f;
            p[u] = pv;
            ds[u] = pv * (dp[i * 4 + u] - da[u]);
          }
          pw[2 * i] = pack2<kBf16>(p[0], p[1]);
          pw[2 * i + 1] = pack2<kBf16>(p[2], p[3]);
          dw[2 * i] = pack2<kBf16>(ds[0], ds[1]);
          dw[2 * i + 1] = pack2<kBf16>(ds[2], ds[3]);
        }
        // 16 packed columns; chunk c overwrites columns already read
        tmem_st16(lane_addr + kColS + c * 16, pw);
        tmem_st16(lane_addr + kColDP + c * 16, dw);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sh->ew_full);
    }
    if (ok && n_it > 0) {
      ok = mbar_wait(&sh->acc_done, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      // TMEM loads are warp-collective: every lane loads, only real keys store
      tc_fence_after();
      T* dv = reinterpret_cast<T*>(dv_) + static_cast<int64_t>(j) * dv_st + hk * dv_sh;
      T* dk = reinterpret_cast<T*>(dk_) + static_cast<int64_t>(j) * dk_st + hk * dk_sh;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float a[32];
        if (n_it > 0) {
          tmem_ld32(lane_addr + kColDV + c * 32, a);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = 0.f;
        }
        if (j < n_kv) store_row32<kBf16>(dv + c * 32, a, 1.f);
        if (n_it > 0) tmem_ld32(lane_addr + kColDK + c * 32, a);
        if (j < n_kv) store_row32<kBf16>(dk + c * 32, a, scale);
      }
    } else {
      raise_abort(sh, status);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ======================================================================== dQ
template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dq_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
               int n_q, int n_kv, int rep, const int32_t* __restrict__ kv_lo,
               const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ fwd_ptr,
               const int32_t* __restrict__ fwd_list, const float* __restrict__ lse,
               const float* __restrict__ delta, float scale_log2, float scale,
               void* __restrict__ dq_, int64_t dq_st, int64_t dq_sh, int32_t* status) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = base;
  uint8_t* sDO = sQ + kTileBytes;
  uint8_t* sK = sDO + kTileBytes;          // 2 stages
  uint8_t* sV = sK + 2 * kTileBytes;       // 2 stages
  BwdBarriers* sh = reinterpret_cast<BwdBarriers*>(sV + 2 * kTileBytes);
  const volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int qt = gridDim.y - 1 - blockIdx.y;
  const int hk = h / rep;
  const int e0 = fwd_ptr[qt];
  const int n_it = fwd_ptr[qt + 1] - e0;
  const int ld = lse_ld(n_q);

  if (threadIdx.x == 0) init_barriers(sh);
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&sh->fixed_full, 2 * kTileBytes);
      tma_load_3d(sQ, &tm_q, &sh->fixed_full, 0, qt * kT, h);
      tma_load_3d(sQ + kHalfBytes, &tm_q, &sh->fixed_full, 64, qt * kT, h);
      tma_load_3d(sDO, &tm_do, &sh->fixed_full, 0, qt * kT, h);
      tma_load_3d(sDO + kHalfBytes, &tm_do, &sh->fixed_full, 64, qt * kT, h);
      int issued[2] = {0, 0};
      bool ok = true;
      for (int it = 0; it < n_it; ++it) {
        const int s = it & 1;
        if (it >= 2) ok = mbar_wait(&sh->ab_empty[s], ((it >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        const int kt = fwd_list[e0 + it] >> 1;
        uint8_t* k_dst = sK + s * kTileBytes;
        uint8_t* v_dst = sV + s * kTileBytes;
        mbar_arrive_expect_tx(&sh->a_full[s], kTileBytes);
        tma_load_3d(k_dst, &tm_k, &sh->a_full[s], 0, kt * kT, hk);
        tma_load_3d(k_dst + kHalfBytes, &tm_k, &sh->a_full[s], 64, kt * kT, hk);
        mbar_arrive_expect_tx(&sh->b_full[s], kTileBytes);
        tma_load_3d(v_dst, &tm_v, &sh->b_full[s], 0, kt * kT, hk);
        tma_load_3d(v_dst + kHalfBytes, &tm_v, &sh->b_full[s], 64, kt * kT, hk);
        issued[s] += 1;
      }
      if (!ok) {
        raise_abort(sh, status);
        mbar_wait(&sh->fixed_full, 0, nullptr);
        for (int s = 0; s < 2; ++s)
          if (issued[s] > 0) {
            mbar_wait(&sh->a_full[s], (issued[s] - 1) & 1, nullptr);
            mbar_wait(&sh->b_full[s], (issued[s] - 1) & 1, nullptr);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t id_ss = idesc_f16(kBf16, kT, kT, false);
      constexpr uint32_t id_ts = idesc_f16(kBf16, kT, kD, true);
      const uint32_t q_addr = smem_u32(sQ), o_addr = smem_u32(sDO);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(&sh->fixed_full, 0, abort_flag);
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it & 1;
        ok = mbar_wait(&sh->a_full[s], (it >> 1) & 1, abort_flag);
        if (ok) ok = mbar_wait(&sh->b_full[s], (it >> 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        mma_tile_ss(tmem + kColS, q_addr, k_addr + s * kTileBytes, id_ss);    // S = Q K^T
        mma_tile_ss(tmem + kColDP, o_addr, v_addr + s * kTileBytes, id_ss);   // dP = dO V^T
        tc_commit(&sh->sdp_full);
        ok = mbar_wait(&sh->ew_full, it & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        mma_tile_ts(tmem + kColDQ, tmem + kColS, k_addr + s * kTileBytes, id_ts, it > 0);
        tc_commit(&sh->ab_empty[s]);
      }
      tc_commit(&sh->acc_done);
      if (!ok) {
        raise_abort(sh, status);
        tc_commit(&sh->drain);
        mbar_wait(&sh->drain, 0, nullptr);
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int row = qt * kT + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float l2 = lse[static_cast<int64_t>(h) * ld + row] * kLog2e;   // padded rows: +inf
    const float dr = delta[static_cast<int64_t>(h) * ld + row];
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int ent = fwd_list[e0 + it];
      const int j0 = (ent >> 1) * kT;
      const bool partial = ent & 1;
      const bool vec = j0 + kT <= n_kv;
      ok = mbar_wait(&sh->sdp_full, it & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kT / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld32(lane_addr + kColS + c * 32, sv);
        tmem_ld32(lane_addr + kColDP + c * 32, dp);
        float p[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = exp2f(fmaf(sv[i], scale_log2, -l2));
        if (partial) {
          if (vec) {
            const int4* lo4 = reinterpret_cast<const int4*>(kv_lo + j0 + c * 32);
            const int4* hi4 = reinterpret_cast<const int4*>(kv_hi + j0 + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int4 a = __ldg(lo4 + i), z = __ldg(hi4 + i);
              if (!visible(a.x, z.x, row)) p[4 * i + 0] = 0.f;
              if (!visible(a.y, z.y, row)) p[4 * i + 1] = 0.f;
              if (!visible(a.z, z.z, row)) p[4 * i + 2] = 0.f;
              if (!visible(a.w, z.w, row)) p[4 * i + 3] = 0.f;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int jj = j0 + c * 32 + i;
              if (!(jj < n_kv && visible(__ldg(kv_lo + jj), __ldg(kv_hi + jj), row))) p[i] = 0.f;
            }
          }
        }
        uint32_t dw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          dw[i] = pack2<kBf16>(p[2 * i] * (dp[2 * i] - dr), p[2 * i + 1] * (dp[2 * i + 1] - dr));
        tmem_st16(lane_addr + kColS + c * 16, dw);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sh->ew_full);
    }
    if (ok && n_it > 0) {
      ok = mbar_wait(&sh->acc_done, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      T* dq = reinterpret_cast<T*>(dq_) + static_cast<int64_t>(row) * dq_st + h * dq_sh;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float a[32];
        if (n_it > 0) {
          tmem_ld32(lane_addr + kColDQ + c * 32, a);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = 0.f;
        }
        if (row < n_q) store_row32<kBf16>(dq + c * 32, a, scale);
      }
    } else {
      raise_abort(sh, status);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// delta[h, i] = sum_d O[i,h,d] dO[i,h,d] over the padded [hq, ld] layout
// (one warp per (row, head), 4 dims per lane).
template <typename T>
__global__ void attn_bwd_delta_tc(int n_q, int hq, const T* __restrict__ out,
                                  const T* __restrict__ dout, int64_t do_st, int64_t do_sh,
                                  float* __restrict__ delta) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int ld = lse_ld(n_q);
  if (w >= ld * hq) return;
  const int i = w / hq, h = w % hq;
  float acc = 0.f;
  if (i < n_q) {
    const uint2 a = *reinterpret_cast<const uint2*>(out + (static_cast<int64_t>(i) * hq + h) * kD + lane * 4);
    const uint2 b = *reinterpret_cast<const uint2*>(dout + i * do_st + h * do_sh + lane * 4);
    const T* pa = reinterpret_cast<const T*>(&a);
    const T* pb = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int u = 0; u < 4; ++u) acc = fmaf(to_f32(pa[u]), to_f32(pb[u]), acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[static_cast<int64_t>(h) * ld + i] = acc;
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int make_map(CUtensorMap* map, bool bf16, const void* ptr, int64_t n_tok, int64_t n_head,
             int64_t st_tok, int64_t st_head) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return TT_ERR_CUDA;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (st_tok * 2) % 16 || (st_head * 2) % 16)
    return TT_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)n_tok, (cuuint64_t)n_head};
  cuuint64_t strides[2] = {(cuuint64_t)(st_tok * 2), (cuuint64_t)(st_head * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TT_OK : TT_ERR_UNSUPPORTED;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Zero a [n_tok, n_head, 128] 16-bit gradient with arbitrary token/head strides
// (used when the other side of the attention is empty).
__global__ void zero_rows(uint16_t* p, int n_tok, int n_head, int64_t st, int64_t sh) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(n_tok) * n_head * kD) return;
  const int d = idx % kD;
  const int64_t rh = idx / kD;
  p[(rh / n_head) * st + (rh % n_head) * sh + d] = 0;
}

int zero_grad(void* p, int n_tok, int n_head, int64_t st, int64_t sh, cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(n_tok) * n_head * kD;
  if (n == 0) return 0;
  zero_rows<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((uint16_t*)p, n_tok, n_head, st, sh);
  return 1;
}

}  // namespace
}  // namespace sm100
}  // namespace tt

int tt_launch_attn_bwd_sm100(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                             int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, const void* out, const void* dout,
                             int64_t do_st, int64_t do_sh, const float* lse,
                             const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                             const int32_t* fwd_list, const int32_t* bwd_ptr,
                             const int32_t* bwd_list, float scale, void* dq, int64_t dq_st,
                             int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
                             int64_t dv_st, int64_t dv_sh, float* delta, int phases,
                             int32_t* status, cudaStream_t st) {
  using namespace tt::sm100;
  if (D != kD || (dtype != TT_BF16 && dtype != TT_F16)) return TT_ERR_UNSUPPORTED;
  if (!aligned16(kv_lo) || !aligned16(kv_hi) || !aligned16(lse) || !aligned16(delta) ||
      !aligned16(out) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv) ||
      (dq_st * 2) % 16 || (dq_sh * 2) % 16 || (dk_st * 2) % 16 || (dk_sh * 2) % 16 ||
      (dv_st * 2) % 16 || (dv_sh * 2) % 16 || (do_st * 2) % 16 || (do_sh * 2) % 16)
    return TT_ERR_UNSUPPORTED;
  const bool bf16 = dtype == TT_BF16;
  if (n_q == 0 || n_kv == 0) {
    // one side empty: every gradient on the other side is zero
    int n = 0;
    if (phases & TT_BWD_DKDV)
      n += zero_grad(dk, n_kv, hkv, dk_st, dk_sh, st) + zero_grad(dv, n_kv, hkv, dv_st, dv_sh, st);
    if (phases & TT_BWD_DQ) n += zero_grad(dq, n_q, hq, dq_st, dq_sh, st);
    tt_count_launches(n);
    return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
  }
  CUtensorMap mq, mk, mv, mdo;
  int rc;
  if ((rc = make_map(&mq, bf16, q, n_q, hq, q_st, q_sh)) != TT_OK) return rc;
  if ((rc = make_map(&mk, bf16, k, n_kv, hkv, k_st, k_sh)) != TT_OK) return rc;
  if ((rc = make_map(&mv, bf16, v, n_kv, hkv, v_st, v_sh)) != TT_OK) return rc;
  if ((rc = make_map(&mdo, bf16, dout, n_q, hq, do_st, do_sh)) != TT_OK) return rc;
  const int ld = tt::lse_ld(n_q);
  const int warps = ld * hq;
  int launches = 0;
  if (warps > 0 && (phases & TT_BWD_PREP)) {
    if (bf16)
      attn_bwd_delta_tc<__nv_bfloat16><<<(warps + 7) / 8, 256, 0, st>>>(
          n_q, hq, (const __nv_bfloat16*)out, (const __nv_bfloat16*)dout, do_st, do_sh, delta);
    else
      attn_bwd_delta_tc<__half><<<(warps + 7) / 8, 256, 0, st>>>(
          n_q, hq, (const __half*)out, (const __half*)dout, do_st, do_sh, delta);
    ++launches;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  const int rep = hq / hkv;
  if (phases & TT_BWD_DKDV) {
    auto kdkdv = bf16 ? attn_bwd_dkdv_tc<true> : attn_bwd_dkdv_tc<false>;
    TT_CUDA_OK(cudaFuncSetAttribute(kdkdv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemBytes));
    dim3 g(hkv, (n_kv + kT - 1) / kT);
    kdkdv<<<g, kThreads, kSmemBytes, st>>>(mq, mk, mv, mdo, n_q, n_kv, rep, kv_lo, kv_hi,
                                           bwd_ptr, bwd_list, lse, delta, scale_log2, scale, dk,
                                           dk_st, dk_sh, dv, dv_st, dv_sh, status);
    ++launches;
  }
  if (phases & TT_BWD_DQ) {
    auto kdq = bf16 ? attn_bwd_dq_tc<true> : attn_bwd_dq_tc<false>;
    TT_CUDA_OK(cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemBytes));
    dim3 g(hq, (n_q + kT - 1) / kT);
    kdq<<<g, kThreads, kSmemBytes, st>>>(mq, mk, mv, mdo, n_q, n_kv, rep, kv_lo, kv_hi, fwd_ptr,
                                         fwd_list, lse, delta, scale_log2, scale, dq, dq_st,
                                         dq_sh, status);
    ++launches;
  }
  tt_count_launches(launches);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
