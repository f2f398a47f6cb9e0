// Tree attention forward on the 5th-generation tensor cores (sm_100a).
//
// Replaces the SDPA call the reference reaches through HF
// (TF/integrations/sdpa_attention.py:92-101) with its dense additive mask
// (dfs_tree_forward.py:548-550, tree_grad_hybrid.py:313-317): for a 128-row
// query tile, O = softmax(Q K^T * scale + M) V over the kv tiles the host work
// list marks visible, M evaluated in registers from the per-key row intervals
// [kv_lo, kv_hi).
//
// One CTA handles the same query tile for two q heads of one GQA group: they
// read the same K/V tiles and the same mask, so each K/V tile feeds two
// 128x128 score tiles (half the K/V traffic per FLOP of one head per CTA) and
// the two softmax warpgroups alternate with the tensor core (ping-pong):
//
//   warp 0    TMA producer: Q of both heads once, then K/V tiles (+ the key
//             intervals of partial tiles) into a 2-stage ring
//   warp 1    MMA issuer:   S0 = Q0 K^T, S1 = Q1 K^T, then per head
//             O_g += P_g V with P_g read from TMEM, S_g of the next tile issued
//             as soon as PV_g is
//   warps 2-5 softmax of head 0, warps 6-9 softmax of head 1: one thread per
//             query row (= TMEM lane), lazy O rescaling (max grows > 2^8),
//             P written over S in TMEM, final normalisation and store.
// TMEM columns: S0|P0 [0,128), S1|P1 [128,256), O0 [256,384), O1 [384,512).
// With an odd group size the last CTA of a group has one valid head.
#include <type_traits>

#include "tt_sm100.cuh"

namespace tt {
namespace sm100 {
namespace {

constexpr int kBM = 128;                  // query rows per tile
constexpr int kBN = 128;                  // keys per tile
constexpr int kD = 128;                   // head dim
constexpr int kStages = 2;                // K ring and V ring depth
constexpr int kAuxStages = 4;             // key-interval ring depth
constexpr int kTileBytes = kBM * kD * 2;  // one 128 x 128 16-bit tile
constexpr int kHalfBytes = kTileBytes / 2;  // one 64-column swizzle block
constexpr int kAuxBytes = 2 * kBN * 4;      // kv_lo[128] + kv_hi[128] of a tile
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;   // log2 units
#ifndef TT_FWD_EMU_PER8
#define TT_FWD_EMU_PER8 2
#endif
constexpr int kEmuPer8 = TT_FWD_EMU_PER8;   // exp2 column pairs of 8 on the FMA pipe

struct FwdBarriers {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t v_full[kStages];
  uint64_t k_empty[kStages];    // the last score MMA of the stage's tile completed
  uint64_t v_empty[kStages];    // the last PV MMA of the stage's tile completed
  uint64_t aux_full[kAuxStages];
  uint64_t s_full[2];       // per head
  uint64_t p_full[2];       // per head, 128 arrivals
  uint64_t o_done[2];       // per head
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

constexpr size_t kSmemBytes =
    1024 + kTileBytes * (2 + 2 * kStages) + kAuxStages * kAuxBytes + sizeof(FwdBarriers);

__device__ __forceinline__ void raise_abort(FwdBarriers* sh, int32_t* status) {
  set_status(status, TT_ERR_DEVICE_TIMEOUT);
  *reinterpret_cast<volatile int32_t*>(&sh->abort) = 1;
}

// 10 warps share the SM's 4 register-file partitions (16K registers each), so
// a partition holds up to 3 warps: 168 registers per thread at most.
template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
            const __grid_constant__ CUtensorMap tm_v, int n_q, int n_kv, int hq, int rep,
            int pairs_per_group, const int32_t* __restrict__ kv_lo,
            const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ fwd_ptr,
            const int32_t* __restrict__ fwd_list, float scale_log2, void* __restrict__ out_,
            float* __restrict__ lse, int32_t* status) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = base;                                // 2 heads
  uint8_t* sK = sQ + 2 * kTileBytes;                 // kStages
  uint8_t* sV = sK + kStages * kTileBytes;           // kStages
  uint8_t* aux = sV + kStages * kTileBytes;          // kAuxStages x (kv_lo, kv_hi)
  FwdBarriers* sh = reinterpret_cast<FwdBarriers*>(aux + kAuxStages * kAuxBytes);
  const volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.x / pairs_per_group;
  const int h0 = hk * rep + 2 * (blockIdx.x % pairs_per_group);
  const int n_heads = (h0 + 1 < (hk + 1) * rep) ? 2 : 1;
  const int qt = gridDim.y - 1 - blockIdx.y;  // heavier (later) tiles first
  const int e0 = fwd_ptr[qt];
  const int n_it = fwd_ptr[qt + 1] - e0;

  if (threadIdx.x == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->v_full[s], 1);
      mbar_init(&sh->k_empty[s], 1);
      mbar_init(&sh->v_empty[s], 1);
    }
    for (int a = 0; a < kAuxStages; ++a) mbar_init(&sh->aux_full[a], 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(&sh->s_full[g], 1);
      mbar_init(&sh->p_full[g], 128);
      mbar_init(&sh->o_done[g], 1);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_it > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&sh->q_full, n_heads * kTileBytes);
      for (int g = 0; g < n_heads; ++g) {
        tma_load_3d(sQ + g * kTileBytes, &tm_q, &sh->q_full, 0, qt * kBM, h0 + g);
        tma_load_3d(sQ + g * kTileBytes + kHalfBytes, &tm_q, &sh->q_full, 64, qt * kBM, h0 + g);
      }
      // loads issued so far, kept as totals and bit masks (no per-stage
      // arrays: indexed at run time they would live in local memory)
      int k_issued = 0, v_issued = 0;
      uint32_t aux_any = 0, aux_par = 0;   // bit a: stage a loaded / odd count
      bool ok = true;
      // K of tile it reuses the stage once the score MMAs of tile it-2 are
      // done, V once its PV MMAs are; those releases come in the order
      // K(it), V(it), K(it+1), ... so one thread issues them in that order.
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it % kStages;
        const int ent = fwd_list[e0 + it];
        const int kt = ent >> 1;
        if (it >= kStages) ok = mbar_wait(&sh->k_empty[s], ((it / kStages) - 1) & 1, abort_flag);
        if (!ok) break;
        uint8_t* k_dst = sK + s * kTileBytes;
        mbar_arrive_expect_tx(&sh->k_full[s], kTileBytes);
        tma_load_3d(k_dst, &tm_k, &sh->k_full[s], 0, kt * kBN, hk);
        tma_load_3d(k_dst + kHalfBytes, &tm_k, &sh->k_full[s], 64, kt * kBN, hk);
        ++k_issued;
        if (ent & 1) {
          // the key intervals of a partial tile: read by the softmax warps,
          // whose progress past tile it is implied by the release of K(it+2)
          const int a = it % kAuxStages;
          uint8_t* a_dst = aux + a * kAuxBytes;
          mbar_arrive_expect_tx(&sh->aux_full[a], kAuxBytes);
          bulk_load(a_dst, kv_lo + kt * kBN, kAuxBytes / 2, &sh->aux_full[a]);
          bulk_load(a_dst + kAuxBytes / 2, kv_hi + kt * kBN, kAuxBytes / 2, &sh->aux_full[a]);
          aux_any |= 1u << a;
          aux_par ^= 1u << a;
        }
        if (it >= kStages) ok = mbar_wait(&sh->v_empty[s], ((it / kStages) - 1) & 1, abort_flag);
        if (!ok) break;
        mbar_arrive_expect_tx(&sh->v_full[s], kTileBytes);
        tma_load_3d(sV + s * kTileBytes, &tm_v, &sh->v_full[s], 0, kt * kBN, hk);
        tma_load_3d(sV + s * kTileBytes + kHalfBytes, &tm_v, &sh->v_full[s], 64, kt * kBN, hk);
        ++v_issued;
      }
      if (!ok) {
        raise_abort(sh, status);
        // let the copies already in flight land before the CTA exits: stage s
        // received loads it = s, s + kStages, ... < issued, the last of which
        // completes phase (count - 1) & 1
        mbar_wait(&sh->q_full, 0, nullptr);
        for (int s = 0; s < kStages; ++s) {
          const int nk = k_issued > s ? (k_issued - 1 - s) / kStages + 1 : 0;
          const int nv = v_issued > s ? (v_issued - 1 - s) / kStages + 1 : 0;
          if (nk > 0) mbar_wait(&sh->k_full[s], (nk - 1) & 1, nullptr);
          if (nv > 0) mbar_wait(&sh->v_full[s], (nv - 1) & 1, nullptr);
        }
        for (int a = 0; a < kAuxStages; ++a)
          if ((aux_any >> a) & 1u) mbar_wait(&sh->aux_full[a], ((aux_par >> a) & 1u) ^ 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t id_s = idesc_f16(kBf16, kBM, kBN, false);
      constexpr uint32_t id_o = idesc_f16(kBf16, kBM, kD, true);
      // descriptors built once; an address offset o adds o >> 4 (the start
      // field holds address >> 4 and shared addresses stay below 256 KiB)
      const uint64_t d_q = desc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t d_k = desc_sw128(smem_u32(sK), 16, 1024);
      const uint64_t d_v = desc_sw128(smem_u32(sV), kHalfBytes, 1024);
      auto issue_s = [&](int g, int it) {
        const uint64_t dq = d_q + ((g * kTileBytes) >> 4);
        const uint64_t dk = d_k + (((it % kStages) * kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
          mma_ss(tmem + g * 128, dq + off, dk + off, id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[g]);
      };
      auto issue_pv = [&](int g, int it) {
        const uint64_t dv = d_v + (((it % kStages) * kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts(tmem + 256 + g * 128, tmem + g * 128 + kk * 8, dv + ((kk * 2048) >> 4), id_o,
                 (it > 0 || kk > 0) ? 1u : 0u);
        if (it == n_it - 1) tc_commit(&sh->o_done[g]);   // the final O_g
      };
      bool ok = mbar_wait(&sh->q_full, 0, abort_flag);
      if (ok) ok = mbar_wait(&sh->k_full[0], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int g = 0; g < n_heads; ++g) issue_s(g, 0);
        tc_commit(&sh->k_empty[0]);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        const bool more = it + 1 < n_it;
        const int s1 = (it + 1) % kStages;
        bool k_next = false;
        for (int g = 0; g < n_heads && ok; ++g) {
          ok = mbar_wait(&sh->p_full[g], it & 1, abort_flag);
          if (ok && g == 0) ok = mbar_wait(&sh->v_full[s], ph, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_pv(g, it);
          if (more) {
            if (!k_next) {
              ok = mbar_wait(&sh->k_full[s1], ((it + 1) / kStages) & 1, abort_flag);
              if (!ok) break;
              tc_fence_after();
              k_next = true;
            }
            issue_s(g, it + 1);
          }
        }
        if (ok) {
          tc_commit(&sh->v_empty[s]);
          if (more) tc_commit(&sh->k_empty[s1]);
        }
      }
      if (!ok) {
        raise_abort(sh, status);
        tc_commit(&sh->drain);
        mbar_wait(&sh->drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int g = (warp - 2) >> 2;          // head of this warpgroup
    const int quad = warp & 3;              // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;         // row within the tile
    const int row = qt * kBM + r;
    const int h = h0 + g;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t col_s = g * 128, col_o = 256 + g * 128;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint32_t aux_phase = 0;   // bit a: parity of the next load of interval stage a
    if (g < n_heads) {
      for (int it = 0; it < n_it; ++it) {
        const int ent = fwd_list[e0 + it];
        const bool partial = ent & 1;
        ok = mbar_wait(&sh->s_full[g], it & 1, abort_flag);
        // interval stages are loaded for partial tiles only, so their phase
        // is counted here rather than derived from it
        const int as = it % kAuxStages;
        if (ok && partial) {
          ok = mbar_wait(&sh->aux_full[as], (aux_phase >> as) & 1u, abort_flag);
          aux_phase ^= 1u << as;
        }
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        float sv[kBN];
        tmem_ld128(lane_addr + col_s, sv);
        if (partial) {
          const int4* lo4 = reinterpret_cast<const int4*>(aux + as * kAuxBytes);
          const int4* hi4 = reinterpret_cast<const int4*>(aux + as * kAuxBytes + kAuxBytes / 2);
#pragma unroll
          for (int c = 0; c < kBN / 4; ++c) {
            const int4 a = lo4[c], z = hi4[c];
            if (!visible(a.x, z.x, row)) sv[4 * c + 0] = -INFINITY;
            if (!visible(a.y, z.y, row)) sv[4 * c + 1] = -INFINITY;
            if (!visible(a.z, z.z, row)) sv[4 * c + 2] = -INFINITY;
            if (!visible(a.w, z.w, row)) sv[4 * c + 3] = -INFINITY;
          }
        }
        // row max: 3-input max over 4 independent chains
        float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int c = 4; c < kBN; c += 2) mx4[(c >> 1) & 3] = fmax3(mx4[(c >> 1) & 3], sv[c], sv[c + 1]);
        const float mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]);
        const float m_new = fmaxf(m_run, mx * scale_log2);
        float alpha = 1.f;
        bool need = false;
        if (m_run == -INFINITY) {
          m_run = m_new;  // every earlier P of this row was 0: nothing to rescale
        } else if (m_new > m_run + kRescaleThreshold) {
          alpha = exp2f(m_run - m_new);
          m_run = m_new;
          need = true;
        }
        l_run *= alpha;
        const float mb = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sc2 = make_float2(scale_log2, scale_log2), nmb2 = make_float2(-mb, -mb);
        // exponentials: kEmuPer8 of every 8 column pairs on the FMA pipe, the
        // rest on the SFU; 4 independent paired partial sums
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        // (P goes back to TMEM a quarter row at a time: 16 packed registers
        // live beside the score row instead of 32, which keeps the thread
        // within its 168 registers)
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x = ffma2(make_float2(sv[qq * 32 + 2 * i], sv[qq * 32 + 2 * i + 1]), sc2, nmb2);
            float2 pr;
            if ((i & 7) < kEmuPer8) {
              pr = exp2_poly2(x);
            } else {
              pr.x = fast_exp2(x.x);
              pr.y = fast_exp2(x.y);
            }
            acc[i & 3] = fadd2(acc[i & 3], pr);
            pk[i] = pack2<kBf16>(pr.x, pr.y);
          }
          tmem_st16(lane_addr + col_s + qq * 16, pk);
        }
        const float2 a01 = fadd2(acc[0], acc[1]), a23 = fadd2(acc[2], acc[3]);
        l_run += (a01.x + a23.x) + (a01.y + a23.y);
        tmem_st_wait();
        if (__any_sync(0xffffffffu, need)) {
          // O_g *= alpha before PV_g(it) adds to it (the MMA warp issues that
          // only after p_full).  PV_g(it-1) has completed: the commit that
          // signalled S_g(it) was issued after it, and a commit tracks every
          // earlier MMA.  Done after the P stores, when the score row is no
          // longer live (fewer registers at the peak).
#pragma unroll 1
          for (int c = 0; c < kD / 16; ++c) {
            float o[16];
            uint32_t w[16];
            tmem_ld16(lane_addr + col_o + c * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(o[i] * alpha);
            tmem_st16(lane_addr + col_o + c * 16, w);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&sh->p_full[g]);
      }
      if (ok && n_it > 0) {
        ok = mbar_wait(&sh->o_done[g], 0, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* out = reinterpret_cast<T*>(out_) + static_cast<int64_t>(row) * hq * kD + h * kD;
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          if (n_it > 0) {
            tmem_ld32(lane_addr + col_o + c * 32, o);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0.f;
          }
          if (row < n_q) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = pack2<kBf16>(o[2 * i] * inv, o[2 * i + 1] * inv);
            uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
        // rows past n_q are the padding of the [hq, lse_ld(n_q)] layout: +inf
        lse[static_cast<int64_t>(h) * lse_ld(n_q) + row] =
            (row < n_q && l_run > 0.f) ? (m_run + __log2f(l_run)) * 0.69314718055994531f
                                       : INFINITY;
      } else {
        raise_abort(sh, status);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [tokens, heads, 128] 16-bit tensor -> 3-D map {dim, token, head}, box
// {64, 128, 1}, 128-byte swizzle, zero fill outside the tensor.
int make_map(CUtensorMap* map, bool bf16, const void* ptr, int64_t n_tok, int64_t n_head,
             int64_t st_tok, int64_t st_head) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TT_ERR_CUDA;
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

}  // namespace
}  // namespace sm100
}  // namespace tt

int tt_launch_attn_fwd_sm100(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                             int32_t D, const void* q, int64_t q_st, int64_t q_sh,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, const int32_t* kv_lo,
                             const int32_t* kv_hi, const int32_t* fwd_ptr,
                             const int32_t* fwd_list, float scale, void* out, float* lse,
                             int32_t* status, cudaStream_t st) {
  using namespace tt::sm100;
  if (D != kD || (dtype != TT_BF16 && dtype != TT_F16)) return TT_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(kv_lo) & 15) || (reinterpret_cast<uintptr_t>(kv_hi) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return TT_ERR_UNSUPPORTED;
  if (n_q == 0) return TT_OK;
  const bool bf16 = dtype == TT_BF16;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, bf16, q, n_q, hq, q_st, q_sh)) != TT_OK) return rc;
  if ((rc = make_map(&mk, bf16, k, n_kv, hkv, k_st, k_sh)) != TT_OK) return rc;
  if ((rc = make_map(&mv, bf16, v, n_kv, hkv, v_st, v_sh)) != TT_OK) return rc;
  const int n_qt = (n_q + kBM - 1) / kBM;
  const int rep = hq / hkv;
  const int pairs = (rep + 1) / 2;            // CTAs per GQA group (two heads each)
  dim3 grid(hkv * pairs, n_qt);
  const float scale_log2 = scale * 1.4426950408889634f;
  auto kern = bf16 ? attn_fwd_tc<true> : attn_fwd_tc<false>;
  TT_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemBytes));
  kern<<<grid, kThreads, kSmemBytes, st>>>(mq, mk, mv, n_q, n_kv, hq, rep, pairs, kv_lo, kv_hi,
                                           fwd_ptr, fwd_list, scale_log2, out, lse, status);
  tt_count_launches(1);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
