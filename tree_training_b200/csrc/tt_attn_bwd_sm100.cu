// Tree attention backward on the 5th-generation tensor cores (sm_100a).
//
// The gradient torch autograd takes through the reference's SDPA call
// (loss.backward() at tree_grad_hybrid.py:533-535 / tree_grad_ckpt.py:107),
// computed without atomics in two kernels that recompute P from the saved
// row log-sum-exp:
//
//   dK/dV kernel  one CTA per (kv head, 128-key tile); K and V are copied once
//                 into TMEM as 16-bit A operands; streams the q heads of its
//                 GQA group x the q tiles the work list marks visible, as
//                 64-row sub-tiles of Q and dO.  S^T = K Q^T and dP^T = V dO^T
//                 (A from TMEM, B from shared memory); the elementwise warps
//                 turn them into P^T and dS^T = P^T (dP^T - delta), written as
//                 16-bit tiles to shared memory (the K / V tiles' space); then
//                 dV += P^T dO and dK += dS^T Q.
//   dQ kernel     one CTA per (q head, 128-row tile); Q and dO are copied once
//                 into TMEM as 16-bit A operands; streams the visible kv tiles
//                 whole (128 keys): S = Q K^T, dP = dO V^T (A from TMEM, B from
//                 shared memory, N = 128), dS = P (dP - delta) as a 16-bit tile
//                 in shared memory (the Q / dO tiles' space), dQ += dS K.
//
// dK/dV streams its sub-tiles through a 4-stage ring (each stage: two 64 x
// 128 16-bit sub-tiles + their 64 row terms, bulk-copied on the same
// mbarrier), dQ its kv tiles through a 2-stage ring of 128-row tiles with
// their key intervals; stages are released per (sub-)tile.  Each kernel keeps
// one S/dP TMEM buffer, released as soon as the elementwise warps have loaded
// it (not when the MMAs that consume P / dS finish), so the next S/dP MMAs run
// while the elementwise warps still compute.  P / dS tiles rotate through two
// shared-memory buffers, released by the commit of the MMAs that read them.
// Reading the fixed operand from TMEM keeps the S/dP MMAs off the
// shared-memory port, which the streamed operands, the P / dS tiles and the
// accumulating MMAs share.  TMEM (512 cols):
//   dK/dV kernel: S [0,64), dP [64,128), K [128,192), V [192,256) (16-bit
//                 pairs), dV [256,384), dK [384,512);
//   dQ kernel:    S [0,128), dP [128,256), dQ [256,384), Q [384,448),
//                 dO [448,512) (16-bit pairs).
// Warps: 0 TMA producer, 1 S/dP MMA issuer, 2..9 elementwise (two warps per
// TMEM lane quadrant; in dK/dV warp half h owns columns [32h, 32h+32) of each
// sub-tile, in dQ keys [64h, 64h+64) of each tile, and the matching part of
// each P / dS tile row), 10 the issuer of the accumulating MMAs.
#include <type_traits>

#include "tt_sm100.cuh"

namespace tt {
namespace sm100 {
namespace {

constexpr int kT = 128;                     // rows of the fixed tiles and of a list tile
constexpr int kD = 128;                     // head dim
constexpr int kSub = 64;                    // rows of a streamed sub-tile
constexpr int kMaxStages = 4;               // streamed ring depth
constexpr int kStagesDkdv = 4;
constexpr int kNbDkdv = 1;                  // S/dP TMEM buffers: dK/dV kernel (K, V, dV, dK fill the rest)
constexpr int kNbPDkdv = 2;                 // P^T / dS^T shared-memory buffers: dK/dV kernel
constexpr int kTileBytes = kT * kD * 2;     // fixed tile (128 rows)
constexpr int kTileHalf = kTileBytes / 2;   // one 64-dim swizzle block of a fixed tile
constexpr int kSubBytes = kSub * kD * 2;    // streamed sub-tile (64 rows)
constexpr int kSubHalf = kSubBytes / 2;     // one 64-dim swizzle block of a sub-tile
constexpr int kAuxHalf = kSub * 4;          // 64 four-byte entries
constexpr int kAuxBytes = 2 * kAuxHalf;     // per stage: two 64-entry arrays
constexpr int kPTile = kT * kSub * 2;       // 128 x 64 16-bit P / dS tile (A operand in smem)
constexpr int kThreads = 352;            // 11 warps (roles below)
constexpr int kEw = 256;                    // elementwise threads
constexpr int kEwWarps = kEw / 32;          // arrivals on the elementwise warps' barriers
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdBarriers {
  uint64_t fixed_full;       // the two tiles loaded once (K,V or Q,dO)
  uint64_t x_tmem_full;      // the fixed tiles copied into TMEM (256 arrivals)
  uint64_t a_full[kMaxStages];  // streamed sub-tile A (Q or K) + its aux arrays
  uint64_t b_full[kMaxStages];  // streamed sub-tile B (dO or V)
  uint64_t ab_empty[kMaxStages];
  uint64_t sdp_full[2];      // S and dP of a sub-tile ready (per TMEM buffer)
  uint64_t sdp_free[2];      // the elementwise warps loaded S and dP (256 arrivals)
  uint64_t ew_full[2];       // P / dS of a sub-tile written to shared memory (256 arrivals)
  uint64_t pds_free[2];      // dK/dV storing dS: a P / dS buffer's MMAs and dS store are done
  uint64_t acc_done;         // every MMA of the CTA finished
  uint64_t drain;            // abort path of the S/dP issuer
  uint64_t drain_acc;        // abort path of the accumulation issuer
  uint32_t tmem_base;
  int32_t abort;
};

// dK/dV: K, V (whose space holds the P^T and dS^T tiles once K and V sit in
// TMEM), the ring; dQ: Q, dO (whose space holds the dS tiles once Q and dO sit
// in TMEM), the ring.
constexpr size_t kSmemDkdv = 1024 + 2 * kTileBytes + kStagesDkdv * (2 * kSubBytes + kAuxBytes) +
                             sizeof(BwdBarriers);
static_assert(2 * kNbPDkdv * kPTile <= 2 * kTileBytes, "P^T / dS^T tiles alias the K, V tiles");
static_assert(kSmemDkdv <= 232448, "shared memory per block");
// a P / dS buffer is released with the ring stage of the sub-tile that read it
static_assert(kStagesDkdv % kNbPDkdv == 0, "buffer / stage rotation");

// One arrival per warp: every lane has fenced its own tcgen05 / shared-memory
// accesses, the warp synchronises, and lane 0 arrives for all 32.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void raise_abort(BwdBarriers* sh, int32_t* status) {
  set_status(status, TT_ERR_DEVICE_TIMEOUT);
  *reinterpret_cast<volatile int32_t*>(&sh->abort) = 1;
}

__device__ __forceinline__ void init_barriers(BwdBarriers* sh) {
  mbar_init(&sh->fixed_full, 1);
  mbar_init(&sh->x_tmem_full, kEwWarps);
  for (int s = 0; s < kMaxStages; ++s) {
    mbar_init(&sh->a_full[s], 1);
    mbar_init(&sh->b_full[s], 1);
    mbar_init(&sh->ab_empty[s], 1);
  }
  for (int b = 0; b < 2; ++b) {
    mbar_init(&sh->sdp_full[b], 1);
    mbar_init(&sh->sdp_free[b], kEwWarps);
    mbar_init(&sh->ew_full[b], kEwWarps);
    mbar_init(&sh->pds_free[b], 2);   // the MMAs' commit + the dS store's read
  }
  mbar_init(&sh->acc_done, 1);
  mbar_init(&sh->drain, 1);
  mbar_init(&sh->drain_acc, 1);
  sh->abort = 0;
  fence_mbar_init();
}

// A shared-memory descriptor moved by `off` bytes: the start field holds
// address >> 4 and shared addresses stay below 256 KiB, so the sum never
// carries out of the field.  Lets the MMA warp build each descriptor once and
// add constant offsets in the issue loop.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t off) { return d + (off >> 4); }

// D[128 x 64] = X[128 x 128, 16-bit in TMEM] * A[64 x 128]^T: X's dims d sit
// as 16-bit pairs in columns x_tmem + d/2, A is a streamed K-major sub-tile.
__device__ __forceinline__ void mma_ts_n64(uint32_t d_tmem, uint32_t x_tmem, uint64_t da,
                                           uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint32_t oa = (kk >> 2) * kSubHalf + (kk & 3) * 32;
    mma_ts(d_tmem, x_tmem + kk * 8, desc_add(da, oa), idesc, kk > 0 ? 1u : 0u);
  }
}

// Copies row r, dims [64 half, 64 half + 64), of a fixed 128-row tile (K-major,
// 128-byte swizzle: 16-byte chunk j of row r at chunk j ^ (r & 7)) into 32
// TMEM columns of the calling thread's lane, two 16-bit dims per column.
__device__ __forceinline__ void tile_row_to_tmem(const uint8_t* tile, int r, int half,
                                                 uint32_t taddr) {
  const uint8_t* row = tile + half * kTileHalf + r * 128;
  uint32_t w[32];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 c = *reinterpret_cast<const uint4*>(row + ((j ^ (r & 7)) << 4));
    w[4 * j] = c.x;
    w[4 * j + 1] = c.y;
    w[4 * j + 2] = c.z;
    w[4 * j + 3] = c.w;
  }
  tmem_st32(taddr, w);
}

// D[128 x 128] (+)= A[128 x 64] * B[64 rows x 128 dims]: A a P / dS tile in
// shared memory (K-major, 128-byte swizzle), B a streamed sub-tile read MN-major.
__device__ __forceinline__ void mma_ss_k64(uint32_t d_tmem, uint64_t da, uint64_t db,
                                           uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kSub / 16; ++kk)
    mma_ss(d_tmem, desc_add(da, kk * 32), desc_add(db, kk * 2048), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

// Writes 32 16-bit values (w: 16 pairs) as columns [32 half, 32 half + 32) of
// row r of a P / dS tile: 128-byte rows, 16-byte chunk j stored at j ^ (r & 7).
__device__ __forceinline__ void store_tile_row(uint8_t* tile, int r, int half,
                                               const uint32_t (&w)[16]) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(row + (((4 * half + c) ^ (r & 7)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
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

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                    ~static_cast<uintptr_t>(1023));
}

// Streams `n_u` (A, B) sub-tile pairs through the ring; `coord(u, &row,
// &head, &aux_a, &aux_b)` gives the sub-tile's first row / head and the two
// 256-byte arrays to bulk-copy with sub-tile A.
template <int KS, typename Coord>
__device__ __forceinline__ void produce(BwdBarriers* sh, const volatile int32_t* abort_flag,
                                        int32_t* status, int n_u, uint8_t* ringA, uint8_t* ringB,
                                        uint8_t* aux, const CUtensorMap* ta,
                                        const CUtensorMap* tb, Coord coord) {
  int issued[KS] = {};
  bool ok = true;
  for (int u = 0; u < n_u; ++u) {
    const int s = u % KS;
    if (u >= KS) ok = mbar_wait(&sh->ab_empty[s], ((u / KS) - 1) & 1, abort_flag);
    if (!ok) break;
    int row, head;
    const void *xa, *xb;
    coord(u, &row, &head, &xa, &xb);
    uint8_t* a_dst = ringA + s * kSubBytes;
    uint8_t* b_dst = ringB + s * kSubBytes;
    uint8_t* x_dst = aux + s * kAuxBytes;
    mbar_arrive_expect_tx(&sh->a_full[s], kSubBytes + kAuxBytes);
    tma_load_3d(a_dst, ta, &sh->a_full[s], 0, row, head);
    tma_load_3d(a_dst + kSubHalf, ta, &sh->a_full[s], 64, row, head);
    bulk_load(x_dst, xa, kAuxHalf, &sh->a_full[s]);
    bulk_load(x_dst + kAuxHalf, xb, kAuxHalf, &sh->a_full[s]);
    mbar_arrive_expect_tx(&sh->b_full[s], kSubBytes);
    tma_load_3d(b_dst, tb, &sh->b_full[s], 0, row, head);
    tma_load_3d(b_dst + kSubHalf, tb, &sh->b_full[s], 64, row, head);
    issued[s] += 1;
  }
  if (!ok) {
    raise_abort(sh, status);
    mbar_wait(&sh->fixed_full, 0, nullptr);
    for (int s = 0; s < KS; ++s)
      if (issued[s] > 0) {
        mbar_wait(&sh->a_full[s], (issued[s] - 1) & 1, nullptr);
        mbar_wait(&sh->b_full[s], (issued[s] - 1) & 1, nullptr);
      }
  }
}

// The MMAs of both kernels come from two issuing threads.  A thread that
// issues tcgen05.mma runs at most about one MMA ahead of the tensor pipe, so
// every barrier wait of a single issuer leaves the pipe idle; with two
// issuers each one's waits are covered by the other's MMAs.  Sub-tile u uses
// ring stage s = u % KS and buffer b = u % 2:
//   S/dP issuer (warp 1):  S_b = X * A_s^T, dP_b = Y * B_s^T  (X, Y the fixed
//       tiles), after the stage landed and after the elementwise warps loaded
//       sub-tile u-2's S/dP out of TMEM buffer b (sdp_free);
//   accumulation issuer (warp 10): the kernel's products reading the P / dS
//       tiles once the elementwise warps wrote them (ew_full); it alone
//       accumulates into dK/dV or dQ, in sub-tile order, so the result does
//       not depend on how the two instruction streams interleave.  Its commit
//       releases the ring stage (ab_empty) and with it the P / dS buffer of
//       the sub-tile: one commit per sub-tile.
// The fixed tiles X, Y are A operands in TMEM (x_addr, y_addr: TMEM column
// addresses, filled by the elementwise warps before x_tmem_full completes).
template <int NB, int KS>
__device__ __forceinline__ void sdp_issuer(BwdBarriers* sh, const volatile int32_t* abort_flag,
                                           int32_t* status, uint32_t tmem, int n_u,
                                           uint32_t x_addr, uint32_t y_addr, uint32_t ring_a,
                                           uint32_t ring_b, uint32_t id_s) {
  bool ok = mbar_wait(&sh->x_tmem_full, 0, abort_flag);
  const uint64_t da = desc_sw128(ring_a, 16, 1024), db = desc_sw128(ring_b, 16, 1024);
  for (int u = 0; u < n_u && ok; ++u) {
    const int s = u % KS, b = u % NB;
    const uint32_t ph = (u / KS) & 1;
    if (u >= NB && !(ok = mbar_wait(&sh->sdp_free[b], ((u - NB) / NB) & 1, abort_flag))) break;
    if (!(ok = mbar_wait(&sh->a_full[s], ph, abort_flag))) break;
    if (!(ok = mbar_wait(&sh->b_full[s], ph, abort_flag))) break;
    tc_fence_after();
    mma_ts_n64(tmem + 64 * b, x_addr, desc_add(da, s * kSubBytes), id_s);
    mma_ts_n64(tmem + 64 * NB + 64 * b, y_addr, desc_add(db, s * kSubBytes), id_s);
    tc_commit(&sh->sdp_full[b]);
  }
  if (!ok) {
    raise_abort(sh, status);
    tc_commit(&sh->drain);
    mbar_wait(&sh->drain, 0, nullptr);
  }
}

template <int NB, int KS, typename Acc>
__device__ __forceinline__ void acc_issuer(BwdBarriers* sh, const volatile int32_t* abort_flag,
                                           int32_t* status, int n_u, Acc acc) {
  bool ok = true;
  for (int u = 0; u < n_u && ok; ++u) {
    const int b = u % NB, s = u % KS;
    if (!(ok = mbar_wait(&sh->ew_full[b], (u / NB) & 1, abort_flag))) break;
    tc_fence_after();
    acc(s, b, u > 0);
    // the stage's last reader: sdp(u) completed before the elementwise warps
    // started on sub-tile u, and acc(u) waited for them
    tc_commit(&sh->ab_empty[s]);
  }
  if (ok) {
    tc_commit(&sh->acc_done);
  } else {
    raise_abort(sh, status);
    tc_commit(&sh->drain_acc);
    mbar_wait(&sh->drain_acc, 0, nullptr);
  }
}

// ===================================================================== dK/dV
// kStoreDS: the CTA also stores each 16-bit dS^T sub-tile it computes into the
// workspace slot of its (q head, q tile, kv tile) triple, where the dQ-from-dS
// kernel reads it back (ds_ws: the slots of q heads hk0 * rep ...; e2f: the
// fwd-list index of every bwd-list entry; n_pairs: slots per q head).  The
// CTA's kv head is hk0 + blockIdx.x.
template <bool kBf16, bool kStoreDS>
__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dkdv_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                 int n_q, int n_kv, int rep, const int32_t* __restrict__ kv_lo,
                 const int32_t* __restrict__ kv_hi, const int32_t* __restrict__ bwd_ptr,
                 const int32_t* __restrict__ bwd_list, const float* __restrict__ lse,
                 const float* __restrict__ delta, float scale_log2, float scale,
                 void* __restrict__ dk_, int64_t dk_st, int64_t dk_sh, void* __restrict__ dv_,
                 int64_t dv_st, int64_t dv_sh, const int32_t* __restrict__ kt_order,
                 int32_t* status, int hk0, uint8_t* __restrict__ ds_ws,
                 const int32_t* __restrict__ e2f, int64_t n_pairs) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* sK = base;
  uint8_t* sV = sK + kTileBytes;
  constexpr int KS = kStagesDkdv;
  uint8_t* rQ = sV + kTileBytes;                 // KS x Q sub-tile
  uint8_t* rDO = rQ + KS * kSubBytes;            // KS x dO sub-tile
  uint8_t* sPt = sK;                             // kNbPDkdv x P^T tile, once K is in TMEM
  uint8_t* sDSt = sK + kNbPDkdv * kPTile;        // kNbPDkdv x dS^T tile, once V is in TMEM
  uint8_t* aux = rDO + KS * kSubBytes;           // KS x (LSE[64], delta[64])
  BwdBarriers* sh = reinterpret_cast<BwdBarriers*>(aux + KS * kAuxBytes);
  const volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = hk0 + static_cast<int>(blockIdx.x);
  // key tile: in work order (longest list first) when the order is given,
  // else in key order, where the root-side tiles with the longest lists come first
  const int kt = kt_order ? kt_order[blockIdx.y] : static_cast<int>(blockIdx.y);
  const int e0 = bwd_ptr[kt];
  const int n_list = bwd_ptr[kt + 1] - e0;
  const int n_u = 2 * rep * n_list;          // 64-row sub-tiles
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
  constexpr uint32_t kColK = 128, kColV = 192;   // K, V as 16-bit pairs (A of S^T, dP^T)
  constexpr uint32_t kColDV = 256, kColDK = 384;
  static_assert(64 * kNbDkdv * 2 <= kColK, "dK/dV kernel TMEM map");

  if (warp == 0) {
    if (lane == 0 && n_u > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_do);
      mbar_arrive_expect_tx(&sh->fixed_full, 2 * kTileBytes);
      tma_load_3d(sK, &tm_k, &sh->fixed_full, 0, kt * kT, hk);
      tma_load_3d(sK + kTileHalf, &tm_k, &sh->fixed_full, 64, kt * kT, hk);
      tma_load_3d(sV, &tm_v, &sh->fixed_full, 0, kt * kT, hk);
      tma_load_3d(sV + kTileHalf, &tm_v, &sh->fixed_full, 64, kt * kT, hk);
      produce<KS>(sh, abort_flag, status, n_u, rQ, rDO, aux, &tm_q, &tm_do,
              [&](int u, int* row, int* head, const void** xa, const void** xb) {
                const int it = u >> 1;
                const int h = hk * rep + it / n_list;
                const int q0 = (bwd_list[e0 + it % n_list] >> 1) * kT + (u & 1) * kSub;
                *row = q0;
                *head = h;
                *xa = lse + static_cast<int64_t>(h) * ld + q0;
                *xb = delta + static_cast<int64_t>(h) * ld + q0;
              });
    }
  } else if (warp == 1) {
    if (lane == 0 && n_u > 0) {
      constexpr uint32_t id_s = idesc_f16(kBf16, kT, kSub, false);
      sdp_issuer<kNbDkdv, KS>(sh, abort_flag, status, tmem, n_u, tmem + kColK,
                                    tmem + kColV, smem_u32(rQ), smem_u32(rDO), id_s);
    }
  } else if (warp == 10) {
    if (lane == 0 && n_u > 0) {
      constexpr uint32_t id_o = idesc_f16(kBf16, kT, kD, true);
      // B of dV += P^T dO and dK += dS^T Q: the ring's dO / Q sub-tiles, MN-major
      const uint64_t d_do = desc_sw128(smem_u32(rDO), kSubHalf, 1024);
      const uint64_t d_q = desc_sw128(smem_u32(rQ), kSubHalf, 1024);
      // A of dV += P^T dO and dK += dS^T Q: the P^T / dS^T tiles, K-major
      const uint64_t d_pt = desc_sw128(smem_u32(sPt), 16, 1024);
      const uint64_t d_dst = desc_sw128(smem_u32(sDSt), 16, 1024);
      auto acc = [&](int s, int b, bool accumulate) {
        mma_ss_k64(tmem + kColDV, desc_add(d_pt, b * kPTile), desc_add(d_do, s * kSubBytes),
                   id_o, accumulate);
        mma_ss_k64(tmem + kColDK, desc_add(d_dst, b * kPTile), desc_add(d_q, s * kSubBytes),
                   id_o, accumulate);
      };
      if constexpr (!kStoreDS) {
        acc_issuer<kNbPDkdv, KS>(sh, abort_flag, status, n_u, acc);
      } else {
        // As acc_issuer, and after the MMAs of sub-tile u this thread also
        // bulk-stores its dS^T buffer (16 KB, in the swizzled layout the dQ
        // kernel's MMAs read) into the sub-tile's half of the workspace slot.
        // Buffer b is rewritten two sub-tiles later, once pds_free[b] saw
        // both the MMAs' commit and, one iteration on, the end of the
        // store's shared-memory read.  The slot index of entry it + 1 is
        // loaded one entry ahead.
        const int n_it = n_u >> 1;
        int f = 0, f_next = e2f[e0];
        bool ok = true;
        for (int u = 0; u < n_u && ok; ++u) {
          const int b = u % kNbPDkdv, s = u % KS, it = u >> 1;
          if ((u & 1) == 0) {
            f = f_next;
            if (it + 1 < n_it) f_next = e2f[e0 + (it + 1) % n_list];
          }
          if (!(ok = mbar_wait(&sh->ew_full[b], (u / kNbPDkdv) & 1, abort_flag))) break;
          tc_fence_after();
          acc(s, b, u > 0);
          tc_commit(&sh->ab_empty[s]);
          tc_commit(&sh->pds_free[b]);
          if (f >= 0 && f < n_pairs) {
            const int hl = hk * rep + it / n_list - hk0 * rep;   // q head within the pass
            uint8_t* dst = ds_ws + (static_cast<int64_t>(hl) * n_pairs + f) * (2 * kPTile) +
                           (u & 1) * kPTile;
            bulk_store(dst, sDSt + b * kPTile, kPTile);
          } else {
            set_status(status, TT_ERR_WORKSPACE);   // a list entry without a slot
          }
          bulk_commit();
          bulk_wait_read<1>();
          if (u >= 1) mbar_arrive(&sh->pds_free[(u - 1) % kNbPDkdv]);
        }
        bulk_wait<0>();   // every store landed before the CTA's shared memory goes
        if (ok) {
          tc_commit(&sh->acc_done);
        } else {
          raise_abort(sh, status);
          tc_commit(&sh->drain_acc);
          mbar_wait(&sh->drain_acc, 0, nullptr);
        }
      }
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;          // key within the tile = TMEM lane
    const int j = kt * kT + r;
    const int lo = j < n_kv ? kv_lo[j] : 0;
    const int hi = j < n_kv ? kv_hi[j] : 0;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    if (n_u > 0) {
      // K and V rows into TMEM, where S^T = K Q^T and dP^T = V dO^T read their
      // A operand; their shared-memory tiles then hold the P^T / dS^T tiles
      ok = mbar_wait(&sh->fixed_full, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tile_row_to_tmem(sK, r, half, lane_addr + kColK + 32 * half);
        tile_row_to_tmem(sV, r, half, lane_addr + kColV + 32 * half);
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(&sh->x_tmem_full, lane);
      }
      // every elementwise thread has read its K / V rows before any P^T / dS^T
      // row lands there (all 256 reach this point: the wait is bounded)
      asm volatile("bar.sync 1, %0;" ::"n"(kEw) : "memory");
    }
    for (int u = 0; u < n_u && ok; ++u) {
      const int it = u >> 1, b = u % kNbDkdv, s = u % KS, pb = u % kNbPDkdv;
      const int ent = bwd_list[e0 + it % n_list];
      const int q0 = (ent >> 1) * kT + (u & 1) * kSub + half * 32;   // first q row of this warp
      const bool partial = ent & 1;
      ok = mbar_wait(&sh->sdp_full[b], (u / kNbDkdv) & 1, abort_flag);
      if (ok) ok = mbar_wait(&sh->a_full[s], (u / KS) & 1, abort_flag);   // aux visible
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const uint32_t cs = 64 * b + 32 * half, cp = 64 * kNbDkdv + 64 * b + 32 * half;
      float sv[32], dp[32];
      tmem_ld32x2(lane_addr + cs, lane_addr + cp, sv, dp);
      tc_fence_before();
      warp_arrive(&sh->sdp_free[b], lane);     // the S/dP buffer may be overwritten
      const float4* L4 = reinterpret_cast<const float4*>(aux + s * kAuxBytes) + half * 8;
      const float4* D4 = reinterpret_cast<const float4*>(aux + s * kAuxBytes + kAuxHalf) + half * 8;
      uint32_t pw[16], dw[16];
      const float2 sc2 = make_float2(scale_log2, scale_log2);
      const float2 nlog2e = make_float2(-kLog2e, -kLog2e);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 l4 = L4[i], d4 = D4[i];
        // exponent argument s * scale - lse (log2 units), two columns per
        // instruction; one pair in four takes the FMA-pipe exp2 so the SFU is
        // not the only unit doing exponentials (masked columns are zeroed
        // after, so their out-of-range arguments do not matter)
        const float2 x01 = ffma2(make_float2(sv[4 * i], sv[4 * i + 1]), sc2,
                                 fmul2(make_float2(l4.x, l4.y), nlog2e));
        const float2 x23 = ffma2(make_float2(sv[4 * i + 2], sv[4 * i + 3]), sc2,
                                 fmul2(make_float2(l4.z, l4.w), nlog2e));
        float2 p01 = (i & 1) ? exp2_poly2(x01) : make_float2(fast_exp2(x01.x), fast_exp2(x01.y));
        float2 p23 = make_float2(fast_exp2(x23.x), fast_exp2(x23.y));
        if (partial) {
          if (!visible(lo, hi, q0 + 4 * i + 0)) p01.x = 0.f;
          if (!visible(lo, hi, q0 + 4 * i + 1)) p01.y = 0.f;
          if (!visible(lo, hi, q0 + 4 * i + 2)) p23.x = 0.f;
          if (!visible(lo, hi, q0 + 4 * i + 3)) p23.y = 0.f;
        }
        const float2 ds01 = fmul2(p01, fadd2(make_float2(dp[4 * i], dp[4 * i + 1]),
                                             make_float2(-d4.x, -d4.y)));
        const float2 ds23 = fmul2(p23, fadd2(make_float2(dp[4 * i + 2], dp[4 * i + 3]),
                                             make_float2(-d4.z, -d4.w)));
        pw[2 * i] = pack2<kBf16>(p01.x, p01.y);
        pw[2 * i + 1] = pack2<kBf16>(p23.x, p23.y);
        dw[2 * i] = pack2<kBf16>(ds01.x, ds01.y);
        dw[2 * i + 1] = pack2<kBf16>(ds23.x, ds23.y);
      }
      if (u >= kNbPDkdv) {                     // the MMAs of sub-tile u - 2 read this buffer
        // (buffer pb was last read by sub-tile u - 2, whose MMAs' commit
        // releases ring stage (u - 2) % KS; storing dS, its store read it too)
        if constexpr (kStoreDS)
          ok = mbar_wait(&sh->pds_free[pb], ((u - kNbPDkdv) / kNbPDkdv) & 1, abort_flag);
        else
          ok = mbar_wait(&sh->ab_empty[(u - kNbPDkdv) % KS], ((u - kNbPDkdv) / KS) & 1,
                         abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      store_tile_row(sPt + pb * kPTile, r, half, pw);
      store_tile_row(sDSt + pb * kPTile, r, half, dw);
      fence_proxy_async_smem();
      warp_arrive(&sh->ew_full[pb], lane);
    }
    if (ok && n_u > 0) {
      ok = mbar_wait(&sh->acc_done, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      // TMEM loads are warp-collective: every lane loads, only real keys store
      tc_fence_after();
      T* dv = reinterpret_cast<T*>(dv_) + static_cast<int64_t>(j) * dv_st + hk * dv_sh;
      T* dk = reinterpret_cast<T*>(dk_) + static_cast<int64_t>(j) * dk_st + hk * dk_sh;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        float a[32];
        if (n_u > 0) {
          tmem_ld32(lane_addr + kColDV + c * 32, a);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = 0.f;
        }
        if (j < n_kv) store_row32<kBf16>(dv + c * 32, a, 1.f);
        if (n_u > 0) tmem_ld32(lane_addr + kColDK + c * 32, a);
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
// Whole 128-key kv tiles per step (N = 128 MMAs), one S/dP TMEM buffer, a
// 2-stage ring of K / V tiles.  Tile u of the CTA's list:
//   S = Q K^T, dP = dO V^T            (warp 1; A = Q / dO from TMEM)
//   dS = P (dP - delta) -> smem tile  (warps 2-9; each thread loads the 64
//                                      keys of its row at once, which frees
//                                      the S/dP buffer, then computes them as
//                                      two 32-key passes)
//   dQ += dS K                        (warp 10; A = dS, B = K from smem)
constexpr int kStagesDq2 = 2;
constexpr int kAuxQ = kT * 4;               // 128 four-byte key intervals
constexpr size_t kSmemDq2 = 1024 + 2 * kTileBytes + kStagesDq2 * (2 * kTileBytes + 2 * kAuxQ) +
                            sizeof(BwdBarriers);
static_assert(kSmemDq2 <= 232448, "shared memory per block");
static_assert(kStagesDq2 <= kMaxStages, "ring barriers");

// D[128 x 128] = X[128 x 128, 16-bit in TMEM] * A[128 x 128]^T, A a K-major
// 128-row tile in shared memory (two 64-dim swizzle blocks).
__device__ __forceinline__ void mma_ts_n128(uint32_t d_tmem, uint32_t x_tmem, uint64_t da,
                                            uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint32_t oa = (kk >> 2) * kTileHalf + (kk & 3) * 32;
    mma_ts(d_tmem, x_tmem + kk * 8, desc_add(da, oa), idesc, kk > 0 ? 1u : 0u);
  }
}

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
  constexpr int KS = kStagesDq2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* sQ = base;
  uint8_t* sDO = sQ + kTileBytes;
  uint8_t* rK = sDO + kTileBytes;                // KS x K tile
  uint8_t* rV = rK + KS * kTileBytes;            // KS x V tile
  uint8_t* aux = rV + KS * kTileBytes;           // KS x (kv_lo[128], kv_hi[128])
  uint8_t* sDS = sQ;                             // 2 x dS tile, once Q and dO are in TMEM
  BwdBarriers* sh = reinterpret_cast<BwdBarriers*>(aux + KS * 2 * kAuxQ);
  const volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int qt = gridDim.y - 1 - blockIdx.y;
  const int hk = h / rep;
  const int e0 = fwd_ptr[qt];
  const int n_u = fwd_ptr[qt + 1] - e0;          // kv tiles
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
  constexpr uint32_t kColS = 0, kColP = 128, kColDQ = 256;
  constexpr uint32_t kColQ = 384, kColDO = 448;   // Q, dO as 16-bit pairs

  if (warp == 0) {
    if (lane == 0 && n_u > 0) {
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&sh->fixed_full, 2 * kTileBytes);
      tma_load_3d(sQ, &tm_q, &sh->fixed_full, 0, qt * kT, h);
      tma_load_3d(sQ + kTileHalf, &tm_q, &sh->fixed_full, 64, qt * kT, h);
      tma_load_3d(sDO, &tm_do, &sh->fixed_full, 0, qt * kT, h);
      tma_load_3d(sDO + kTileHalf, &tm_do, &sh->fixed_full, 64, qt * kT, h);
      int issued[KS] = {};
      bool ok = true;
      for (int u = 0; u < n_u; ++u) {
        const int s = u % KS;
        if (u >= KS && !(ok = mbar_wait(&sh->ab_empty[s], ((u / KS) - 1) & 1, abort_flag))) break;
        const int j0 = (fwd_list[e0 + u] >> 1) * kT;
        uint8_t* k_dst = rK + s * kTileBytes;
        uint8_t* v_dst = rV + s * kTileBytes;
        uint8_t* x_dst = aux + s * 2 * kAuxQ;
        mbar_arrive_expect_tx(&sh->a_full[s], kTileBytes + 2 * kAuxQ);
        tma_load_3d(k_dst, &tm_k, &sh->a_full[s], 0, j0, hk);
        tma_load_3d(k_dst + kTileHalf, &tm_k, &sh->a_full[s], 64, j0, hk);
        bulk_load(x_dst, kv_lo + j0, kAuxQ, &sh->a_full[s]);
        bulk_load(x_dst + kAuxQ, kv_hi + j0, kAuxQ, &sh->a_full[s]);
        mbar_arrive_expect_tx(&sh->b_full[s], kTileBytes);
        tma_load_3d(v_dst, &tm_v, &sh->b_full[s], 0, j0, hk);
        tma_load_3d(v_dst + kTileHalf, &tm_v, &sh->b_full[s], 64, j0, hk);
        issued[s] += 1;
      }
      if (!ok) {
        raise_abort(sh, status);
        mbar_wait(&sh->fixed_full, 0, nullptr);
        for (int s = 0; s < KS; ++s)
          if (issued[s] > 0) {
            mbar_wait(&sh->a_full[s], (issued[s] - 1) & 1, nullptr);
            mbar_wait(&sh->b_full[s], (issued[s] - 1) & 1, nullptr);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_u > 0) {
      // S / dP issuer: tile u waits for the elementwise warps to have loaded
      // tile u-1 out of the single S/dP buffer, and for its K / V stage
      constexpr uint32_t id_s = idesc_f16(kBf16, kT, kT, false);
      const uint64_t dk = desc_sw128(smem_u32(rK), 16, 1024);
      const uint64_t dv = desc_sw128(smem_u32(rV), 16, 1024);
      bool ok = mbar_wait(&sh->x_tmem_full, 0, abort_flag);
      for (int u = 0; u < n_u && ok; ++u) {
        const int s = u % KS;
        const uint32_t ph = (u / KS) & 1;
        if (u >= 1 && !(ok = mbar_wait(&sh->sdp_free[0], (u - 1) & 1, abort_flag))) break;
        if (!(ok = mbar_wait(&sh->a_full[s], ph, abort_flag))) break;
        if (!(ok = mbar_wait(&sh->b_full[s], ph, abort_flag))) break;
        tc_fence_after();
        mma_ts_n128(tmem + kColS, tmem + kColQ, desc_add(dk, s * kTileBytes), id_s);
        mma_ts_n128(tmem + kColP, tmem + kColDO, desc_add(dv, s * kTileBytes), id_s);
        tc_commit(&sh->sdp_full[0]);
      }
      if (!ok) {
        raise_abort(sh, status);
        tc_commit(&sh->drain);
        mbar_wait(&sh->drain, 0, nullptr);
      }
    }
  } else if (warp == 10) {
    if (lane == 0 && n_u > 0) {
      // dQ += dS K, in tile order (the only accumulating MMAs: deterministic);
      // the commit releases the K / V stage and the dS buffer of tile u
      constexpr uint32_t id_o = idesc_f16(kBf16, kT, kD, true);
      const uint64_t d_k = desc_sw128(smem_u32(rK), kTileHalf, 1024);   // B, MN-major
      const uint64_t d_ds = desc_sw128(smem_u32(sDS), 16, 1024);        // A, K-major
      bool ok = true;
      for (int u = 0; u < n_u && ok; ++u) {
        const int s = u % KS, b = u & 1;
        if (!(ok = mbar_wait(&sh->ew_full[b], (u >> 1) & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk) {
          const uint32_t oa = b * kTileBytes + (kk >> 2) * kTileHalf + (kk & 3) * 32;
          mma_ss(tmem + kColDQ, desc_add(d_ds, oa), desc_add(d_k, s * kTileBytes + kk * 2048),
                 id_o, (u > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&sh->ab_empty[s]);
      }
      if (ok) {
        tc_commit(&sh->acc_done);
      } else {
        raise_abort(sh, status);
        tc_commit(&sh->drain_acc);
        mbar_wait(&sh->drain_acc, 0, nullptr);
      }
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;              // keys [64 half, 64 half + 64) of a tile
    const int r = quad * 32 + lane;
    const int row = qt * kT + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float l2 = lse[static_cast<int64_t>(h) * ld + row] * kLog2e;   // padded rows: +inf
    const float dr = delta[static_cast<int64_t>(h) * ld + row];
    bool ok = true;
    if (n_u > 0) {
      // Q and dO rows into TMEM, where S = Q K^T and dP = dO V^T read their A
      // operand; their shared-memory tiles then hold the dS tiles
      ok = mbar_wait(&sh->fixed_full, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tile_row_to_tmem(sQ, r, half, lane_addr + kColQ + 32 * half);
        tile_row_to_tmem(sDO, r, half, lane_addr + kColDO + 32 * half);
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(&sh->x_tmem_full, lane);
      }
      // every elementwise thread has read its Q / dO rows before any dS row
      // lands in their space (all 256 reach this point: the wait is bounded)
      asm volatile("bar.sync 1, %0;" ::"n"(kEw) : "memory");
    }
    const float2 sc2 = make_float2(scale_log2, scale_log2), nl2 = make_float2(-l2, -l2);
    const float2 ndr = make_float2(-dr, -dr);
    for (int u = 0; u < n_u && ok; ++u) {
      const int s = u % KS, b = u & 1;
      const bool partial = fwd_list[e0 + u] & 1;
      ok = mbar_wait(&sh->sdp_full[0], u & 1, abort_flag);
      if (ok && partial) ok = mbar_wait(&sh->a_full[s], (u / KS) & 1, abort_flag);
      if (ok && u >= 2)   // the dQ MMAs of tile u - 2 read dS buffer b
        ok = mbar_wait(&sh->ab_empty[(u - 2) % KS], ((u - 2) / KS) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint8_t* ds_box = sDS + b * kTileBytes + half * kTileHalf;
      float sva[2][32], dpa[2][32];
      tmem_ld32x2(lane_addr + kColS + 64 * half, lane_addr + kColP + 64 * half, sva[0], dpa[0]);
      tmem_ld32x2(lane_addr + kColS + 64 * half + 32, lane_addr + kColP + 64 * half + 32, sva[1],
                  dpa[1]);
      tc_fence_before();
      warp_arrive(&sh->sdp_free[0], lane);       // S/dP fully loaded: next tile's MMAs may run
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const uint32_t c0 = 64 * half + 32 * pass;
        float (&sv)[32] = sva[pass];
        float (&dp)[32] = dpa[pass];
        float p[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          // two columns per instruction; one pair in four on the FMA-pipe exp2
          const float2 x = ffma2(make_float2(sv[2 * i], sv[2 * i + 1]), sc2, nl2);
          const float2 e =
              (i & 3) == 3 ? exp2_poly2(x) : make_float2(fast_exp2(x.x), fast_exp2(x.y));
          p[2 * i] = e.x;
          p[2 * i + 1] = e.y;
        }
        if (partial) {
          // key intervals of these 32 keys, zero-padded past n_kv (never visible)
          const int4* LO = reinterpret_cast<const int4*>(aux + s * 2 * kAuxQ + c0 * 4);
          const int4* HI = reinterpret_cast<const int4*>(aux + s * 2 * kAuxQ + kAuxQ + c0 * 4);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int4 a = LO[i], z = HI[i];
            if (!visible(a.x, z.x, row)) p[4 * i + 0] = 0.f;
            if (!visible(a.y, z.y, row)) p[4 * i + 1] = 0.f;
            if (!visible(a.z, z.z, row)) p[4 * i + 2] = 0.f;
            if (!visible(a.w, z.w, row)) p[4 * i + 3] = 0.f;
          }
        }
        uint32_t dw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 ds = fmul2(make_float2(p[2 * i], p[2 * i + 1]),
                                  fadd2(make_float2(dp[2 * i], dp[2 * i + 1]), ndr));
          dw[i] = pack2<kBf16>(ds.x, ds.y);
        }
        store_tile_row(ds_box, r, pass, dw);
      }
      fence_proxy_async_smem();
      warp_arrive(&sh->ew_full[b], lane);
    }
    if (ok && n_u > 0) {
      ok = mbar_wait(&sh->acc_done, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      T* dq = reinterpret_cast<T*>(dq_) + static_cast<int64_t>(row) * dq_st + h * dq_sh;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        float a[32];
        if (n_u > 0) {
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

// ================================================================ dQ from dS
// The stored-dS backward's second kernel: dQ = scale * sum over the q tile's
// kv list of dS K, where dS is read back from the workspace slots the dK/dV
// kernel stored (no recompute of S and dP).  Persistent: one CTA per SM walks
// the work items (q head of the pass, 128-row q tile), item i = q tile
// n_qt - 1 - i / n_heads (the deepest tiles, with the longest lists, first;
// the heads of one q tile next to each other, so their K tiles meet in L2),
// head i % n_heads, CTA c taking items c, c + grid, ...  Warp 0 streams the
// (dS slot, K tile) pairs of all its items through a 3-stage ring (the 32 KB
// slot by one bulk copy, K by TMA); warp 1 issues dQ += dS K (M = 128 rows,
// N = 128 dims, K = 128 keys: A = dS, MN-major, read from the two 64-row dS^T
// sub-tiles of the slot; B = K, MN-major) in list order, so the sum is
// deterministic, into one of two TMEM accumulators (item parity); warps 2-5
// write an item's dQ while the next item accumulates in the other one.
constexpr int kStagesDqs = 3;
constexpr int kThreadsDqs = 192;
constexpr int kEpiWarpsDqs = 4;
struct DqsBarriers {
  uint64_t full[kStagesDqs];
  uint64_t empty[kStagesDqs];
  uint64_t acc_full[2];      // an item's accumulation finished (MMA commit)
  uint64_t acc_empty[2];     // the epilogue read the accumulator (4 warp arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};
constexpr size_t kSmemDqs = 1024 + kStagesDqs * 2 * kTileBytes + sizeof(DqsBarriers);
static_assert(kSmemDqs <= 232448, "shared memory per block");

template <bool kBf16>
__global__ void __launch_bounds__(kThreadsDqs, 1)
attn_bwd_dq_ds_tc(const __grid_constant__ CUtensorMap tm_k, int n_q, int rep, int h0,
                  int n_heads, int n_qt, const int32_t* __restrict__ fwd_ptr,
                  const int32_t* __restrict__ fwd_list, const uint8_t* __restrict__ ds_ws,
                  int64_t n_pairs, float scale, void* __restrict__ dq_, int64_t dq_st,
                  int64_t dq_sh, int32_t* status) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  constexpr int KS = kStagesDqs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* rDS = base;                          // KS x dS slot (two 64-row dS^T sub-tiles)
  uint8_t* rK = rDS + KS * kTileBytes;          // KS x K tile
  DqsBarriers* sh = reinterpret_cast<DqsBarriers*>(rK + KS * kTileBytes);
  volatile int32_t* abort_flag = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = n_heads * n_qt;
  // an item's q tile, q head within the pass and kv list [e0, e0 + n)
  // (a list that would run past the slots is reported and treated as empty)
  auto item = [&](int i, int* qt, int* hl, int* e0, int* n) {
    *qt = n_qt - 1 - i / n_heads;
    *hl = i % n_heads;
    *e0 = fwd_ptr[*qt];
    *n = fwd_ptr[*qt + 1] - *e0;
    if (*e0 < 0 || *n < 0 || static_cast<int64_t>(*e0) + *n > n_pairs) {
      set_status(status, TT_ERR_WORKSPACE);
      *n = 0;
    }
  };
  auto give_up = [&]() {
    set_status(status, TT_ERR_DEVICE_TIMEOUT);
    *abort_flag = 1;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh->acc_full[b], 1);
      mbar_init(&sh->acc_empty[b], kEpiWarpsDqs);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_k);
      int issued[KS] = {};
      bool ok = true;
      int u = 0;                                 // ring position over all items
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        int qt, hl, e0, n;
        item(i, &qt, &hl, &e0, &n);
        const int hk = (h0 + hl) / rep;
        const uint8_t* slots = ds_ws + (static_cast<int64_t>(hl) * n_pairs + e0) * kTileBytes;
        for (int j = 0; j < n; ++j, ++u) {
          const int s = u % KS;
          if (u >= KS && !(ok = mbar_wait(&sh->empty[s], ((u / KS) - 1) & 1, abort_flag))) break;
          const int j0 = (fwd_list[e0 + j] >> 1) * kT;
          mbar_arrive_expect_tx(&sh->full[s], 2 * kTileBytes);
          bulk_load(rDS + s * kTileBytes, slots + static_cast<int64_t>(j) * kTileBytes,
                    kTileBytes, &sh->full[s]);
          tma_load_3d(rK + s * kTileBytes, &tm_k, &sh->full[s], 0, j0, hk);
          tma_load_3d(rK + s * kTileBytes + kTileHalf, &tm_k, &sh->full[s], 64, j0, hk);
          issued[s] += 1;
        }
      }
      if (!ok) {
        give_up();
        for (int s = 0; s < KS; ++s)
          if (issued[s] > 0) mbar_wait(&sh->full[s], (issued[s] - 1) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id = idesc_f16_ab(kBf16, kT, kD, true, true);
      const uint64_t d_ds = desc_sw128(smem_u32(rDS), kPTile, 1024);   // A, MN-major
      const uint64_t d_k = desc_sw128(smem_u32(rK), kTileHalf, 1024);  // B, MN-major
      bool ok = true;
      int u = 0, it = 0;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++it) {
        int qt, hl, e0, n;
        item(i, &qt, &hl, &e0, &n);
        const int b = it & 1;
        // the epilogue has read this accumulator's previous item
        if (it >= 2 && !(ok = mbar_wait(&sh->acc_empty[b], ((it >> 1) - 1) & 1, abort_flag)))
          break;
        tc_fence_after();
        for (int j = 0; j < n; ++j, ++u) {
          const int s = u % KS;
          if (!(ok = mbar_wait(&sh->full[s], (u / KS) & 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            mma_ss(tmem + 128 * b, desc_add(d_ds, s * kTileBytes + kk * 2048),
                   desc_add(d_k, s * kTileBytes + kk * 2048), id, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh->empty[s]);
        }
        if (ok) tc_commit(&sh->acc_full[b]);
      }
      if (!ok) {
        give_up();
        tc_commit(&sh->drain);
        mbar_wait(&sh->drain, 0, nullptr);
      }
    }
  } else if (warp < 2 + kEpiWarpsDqs) {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;              // q row within the tile = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    int it = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++it) {
      int qt, hl, e0, n;
      item(i, &qt, &hl, &e0, &n);
      const int b = it & 1;
      bool ok = mbar_wait(&sh->acc_full[b], (it >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        give_up();
        break;
      }
      tc_fence_after();
      const int row = qt * kT + r;
      T* dq = reinterpret_cast<T*>(dq_) + static_cast<int64_t>(row) * dq_st + (h0 + hl) * dq_sh;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float a[32];
        if (n > 0) {
          tmem_ld32(lane_addr + 128 * b + c * 32, a);
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) a[x] = 0.f;
        }
        if (row < n_q) store_row32<kBf16>(dq + c * 32, a, scale);
      }
      tc_fence_before();
      warp_arrive(&sh->acc_empty[b], lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// e2f[e] = the index in the fwd lists of bwd-list entry e (the same
// (q tile, kv tile) pair): a bwd list holds its q tiles in ascending order, so
// each fwd entry finds its bwd entry by binary search.  Entries left unset
// keep the caller's -1, which the storing dK/dV kernel reports instead of
// storing.  One block per q tile.
__global__ void map_bwd_to_fwd(int n_qt, const int32_t* __restrict__ fwd_ptr,
                               const int32_t* __restrict__ fwd_list,
                               const int32_t* __restrict__ bwd_ptr,
                               const int32_t* __restrict__ bwd_list, int n_kt,
                               int32_t* __restrict__ e2f) {
  const int qt = blockIdx.x;
  if (qt >= n_qt) return;
  for (int f = fwd_ptr[qt] + threadIdx.x; f < fwd_ptr[qt + 1]; f += blockDim.x) {
    const int kt = fwd_list[f] >> 1;
    if (kt < 0 || kt >= n_kt) continue;
    int lo = bwd_ptr[kt], hi = bwd_ptr[kt + 1];
    const int end = hi;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((bwd_list[mid] >> 1) < qt) lo = mid + 1;
      else hi = mid;
    }
    if (lo < end && (bwd_list[lo] >> 1) == qt) e2f[lo] = f;
  }
}

// order[r] = the key tile with the r-th longest work list (ties: lower tile
// first), so the dK/dV CTAs that take longest are dispatched first.  Thread i
// counts the tiles that sort before tile i; n_tiles^2 comparisons in all.
__global__ void order_tiles_by_work(int n_tiles, const int32_t* __restrict__ ptr,
                                   int32_t* __restrict__ order) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tiles) return;
  const int wi = ptr[i + 1] - ptr[i];
  int rank = 0;
  for (int j = 0; j < n_tiles; ++j) {
    const int wj = ptr[j + 1] - ptr[j];
    rank += (wj > wi || (wj == wi && j < i)) ? 1 : 0;
  }
  order[rank] = i;
}

// delta[h, i] = sum_d O[i,h,d] dO[i,h,d] over the padded [hq, ld] layout.
// Half a warp per (row, head) pair, 8 dims (16 bytes) per lane, and each warp
// issues the loads of its kDeltaPairs pairs before any arithmetic, so enough
// bytes are in flight to stream O and dO at HBM rate.  Rows i >= n_q write 0.
constexpr int kDeltaPairs = 4;

template <typename T>
__global__ void attn_bwd_delta_tc(int n_q, int hq, const T* __restrict__ out,
                                  const T* __restrict__ dout, int64_t do_st, int64_t do_sh,
                                  float* __restrict__ delta) {
  constexpr int kPass = kDeltaPairs / 2;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, l16 = lane & 15;
  const int ld = lse_ld(n_q);
  const int64_t total = static_cast<int64_t>(ld) * hq;
  uint4 a[kPass], b[kPass];
  int64_t pair[kPass];
#pragma unroll
  for (int k = 0; k < kPass; ++k) {
    pair[k] = warp * kDeltaPairs + 2 * k + (lane >> 4);
    a[k] = b[k] = make_uint4(0u, 0u, 0u, 0u);
    if (pair[k] < total) {
      const int i = static_cast<int>(pair[k] / hq), h = static_cast<int>(pair[k] % hq);
      if (i < n_q) {
        a[k] = *reinterpret_cast<const uint4*>(out + (static_cast<int64_t>(i) * hq + h) * kD +
                                               l16 * 8);
        b[k] = *reinterpret_cast<const uint4*>(dout + i * do_st + h * do_sh + l16 * 8);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kPass; ++k) {
    const T* pa = reinterpret_cast<const T*>(&a[k]);
    const T* pb = reinterpret_cast<const T*>(&b[k]);
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = fmaf(to_f32(pa[u]), to_f32(pb[u]), acc);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (l16 == 0 && pair[k] < total) {
      const int i = static_cast<int>(pair[k] / hq), h = static_cast<int>(pair[k] % hq);
      delta[static_cast<int64_t>(h) * ld + i] = acc;
    }
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [tokens, heads, 128] 16-bit tensor -> 3-D map {dim, token, head}, box
// {64, box_rows, 1}, 128-byte swizzle, zero fill outside the tensor.
int make_map(CUtensorMap* map, bool bf16, const void* ptr, int64_t n_tok, int64_t n_head,
             int64_t st_tok, int64_t st_head, int box_rows) {
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
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
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
                             int64_t dv_st, int64_t dv_sh, float* delta, int32_t* kt_order,
                             int phases, int32_t* status, cudaStream_t st) {
  using namespace tt::sm100;
  if (D != kD || (dtype != TT_BF16 && dtype != TT_F16)) return TT_ERR_UNSUPPORTED;
  if (!aligned16(kv_lo) || !aligned16(kv_hi) || !aligned16(lse) || !aligned16(delta) ||
      !aligned16(out) || !aligned16(dout) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv) ||
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
  const int ld = tt::lse_ld(n_q);
  const int64_t warps = (static_cast<int64_t>(ld) * hq + kDeltaPairs - 1) / kDeltaPairs;
  int launches = 0;
  if (warps > 0 && (phases & TT_BWD_PREP)) {
    const unsigned blocks = static_cast<unsigned>((warps + 7) / 8);
    if (bf16)
      attn_bwd_delta_tc<__nv_bfloat16><<<blocks, 256, 0, st>>>(
          n_q, hq, (const __nv_bfloat16*)out, (const __nv_bfloat16*)dout, do_st, do_sh, delta);
    else
      attn_bwd_delta_tc<__half><<<blocks, 256, 0, st>>>(
          n_q, hq, (const __half*)out, (const __half*)dout, do_st, do_sh, delta);
    ++launches;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  const int rep = hq / hkv;
  int rc;
  if (phases & TT_BWD_DKDV) {
    // fixed K/V tiles (128 rows), streamed Q/dO sub-tiles (64 rows)
    CUtensorMap mq, mk, mv, mdo;
    if ((rc = make_map(&mq, bf16, q, n_q, hq, q_st, q_sh, kSub)) != TT_OK) return rc;
    if ((rc = make_map(&mk, bf16, k, n_kv, hkv, k_st, k_sh, kT)) != TT_OK) return rc;
    if ((rc = make_map(&mv, bf16, v, n_kv, hkv, v_st, v_sh, kT)) != TT_OK) return rc;
    if ((rc = make_map(&mdo, bf16, dout, n_q, hq, do_st, do_sh, kSub)) != TT_OK) return rc;
    auto kdkdv = bf16 ? attn_bwd_dkdv_tc<true, false> : attn_bwd_dkdv_tc<false, false>;
    TT_CUDA_OK(cudaFuncSetAttribute(kdkdv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemDkdv));
    const int n_tiles = (n_kv + kT - 1) / kT;
    if (kt_order) {
      order_tiles_by_work<<<(n_tiles + 255) / 256, 256, 0, st>>>(n_tiles, bwd_ptr, kt_order);
      ++launches;
    }
    dim3 g(hkv, n_tiles);
    kdkdv<<<g, kThreads, kSmemDkdv, st>>>(mq, mk, mv, mdo, n_q, n_kv, rep, kv_lo, kv_hi,
                                           bwd_ptr, bwd_list, lse, delta, scale_log2, scale, dk,
                                           dk_st, dk_sh, dv, dv_st, dv_sh, kt_order, status,
                                           0, nullptr, nullptr, 0);
    ++launches;
  }
  if (phases & TT_BWD_DQ) {
    // fixed Q/dO tiles (128 rows), streamed K/V sub-tiles (64 rows)
    CUtensorMap mq, mk, mv, mdo;
    if ((rc = make_map(&mq, bf16, q, n_q, hq, q_st, q_sh, kT)) != TT_OK) return rc;
    if ((rc = make_map(&mk, bf16, k, n_kv, hkv, k_st, k_sh, kT)) != TT_OK) return rc;
    if ((rc = make_map(&mv, bf16, v, n_kv, hkv, v_st, v_sh, kT)) != TT_OK) return rc;
    if ((rc = make_map(&mdo, bf16, dout, n_q, hq, do_st, do_sh, kT)) != TT_OK) return rc;
    auto kdq = bf16 ? attn_bwd_dq_tc<true> : attn_bwd_dq_tc<false>;
    TT_CUDA_OK(cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemDq2));
    dim3 g(hq, (n_q + kT - 1) / kT);
    kdq<<<g, kThreads, kSmemDq2, st>>>(mq, mk, mv, mdo, n_q, n_kv, rep, kv_lo, kv_hi, fwd_ptr,
                                         fwd_list, lse, delta, scale_log2, scale, dq, dq_st,
                                         dq_sh, status);
    ++launches;
  }
  tt_count_launches(launches);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

// The stored-dS backward (tt_tree_attn_bwd_stored): PREP = delta, the
// bwd -> fwd entry map and the work order of the key tiles; then per pass of
// kv_heads_per_pass kv heads DKDV = the storing dK/dV kernel and DQ = the
// dQ-from-dS kernel of the pass's q heads.  ds_ws holds
// rep * kv_heads_per_pass * n_pairs slots of 32 KB (n_pairs >= the number of
// tile-list entries), e2f n_pairs int32.  With one pass the phases may be
// launched by separate calls, in the order PREP, DKDV, DQ.
int tt_launch_attn_bwd_sm100_stored(
    int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv, int32_t D, const void* q,
    int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh, const void* v,
    int64_t v_st, int64_t v_sh, const void* out, const void* dout, int64_t do_st, int64_t do_sh,
    const float* lse, const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
    const int32_t* fwd_list, const int32_t* bwd_ptr, const int32_t* bwd_list, float scale,
    void* dq, int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
    int64_t dv_st, int64_t dv_sh, float* delta, int32_t* kt_order, int32_t* e2f, void* ds_ws,
    int64_t n_pairs, int32_t kv_heads_per_pass, int phases, int32_t* status, cudaStream_t st) {
  using namespace tt::sm100;
  if (D != kD || (dtype != TT_BF16 && dtype != TT_F16)) return TT_ERR_UNSUPPORTED;
  if (n_q == 0 || n_kv == 0)   // one side empty: the regular path zeroes the other side
    return tt_launch_attn_bwd_sm100(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh,
                                    v, v_st, v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi,
                                    fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh,
                                    dk, dk_st, dk_sh, dv, dv_st, dv_sh, delta, kt_order,
                                    TT_BWD_ALL, status, st);
  if (kv_heads_per_pass < 1 || kv_heads_per_pass > hkv || n_pairs < 1 || !e2f || !ds_ws ||
      (reinterpret_cast<uintptr_t>(ds_ws) & 15) || !aligned16(e2f) || !kt_order ||
      (phases & ~TT_BWD_ALL) != 0 || phases == 0 ||
      (phases != TT_BWD_ALL && kv_heads_per_pass != hkv))
    return TT_ERR_INVALID_ARG;
  int rc = TT_OK;
  const bool bf16 = dtype == TT_BF16;
  const float scale_log2 = scale * 1.4426950408889634f;
  const int rep = hq / hkv;
  const int n_kt = (n_kv + kT - 1) / kT, n_qt = (n_q + kT - 1) / kT;
  int launches = 0;
  if (phases & TT_BWD_PREP) {
    // delta (and the argument checks) as in the regular backward, then the
    // entry map and the work order of the key tiles
    rc = tt_launch_attn_bwd_sm100(dtype, n_q, n_kv, hq, hkv, D, q, q_st, q_sh, k, k_st, k_sh, v,
                                  v_st, v_sh, out, dout, do_st, do_sh, lse, kv_lo, kv_hi,
                                  fwd_ptr, fwd_list, bwd_ptr, bwd_list, scale, dq, dq_st, dq_sh,
                                  dk, dk_st, dk_sh, dv, dv_st, dv_sh, delta, kt_order,
                                  TT_BWD_PREP, status, st);
    if (rc != TT_OK) return rc;
    TT_CUDA_OK(cudaMemsetAsync(e2f, 0xFF, static_cast<size_t>(n_pairs) * 4, st));
    map_bwd_to_fwd<<<n_qt, 128, 0, st>>>(n_qt, fwd_ptr, fwd_list, bwd_ptr, bwd_list, n_kt, e2f);
    order_tiles_by_work<<<(n_kt + 255) / 256, 256, 0, st>>>(n_kt, bwd_ptr, kt_order);
    launches += 2;
  }
  CUtensorMap mq, mk, mv, mdo;
  if ((rc = make_map(&mq, bf16, q, n_q, hq, q_st, q_sh, kSub)) != TT_OK) return rc;
  if ((rc = make_map(&mk, bf16, k, n_kv, hkv, k_st, k_sh, kT)) != TT_OK) return rc;
  if ((rc = make_map(&mv, bf16, v, n_kv, hkv, v_st, v_sh, kT)) != TT_OK) return rc;
  if ((rc = make_map(&mdo, bf16, dout, n_q, hq, do_st, do_sh, kSub)) != TT_OK) return rc;
  auto kdkdv = bf16 ? attn_bwd_dkdv_tc<true, true> : attn_bwd_dkdv_tc<false, true>;
  auto kdq = bf16 ? attn_bwd_dq_ds_tc<true> : attn_bwd_dq_ds_tc<false>;
  TT_CUDA_OK(cudaFuncSetAttribute(kdkdv, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemDkdv));
  TT_CUDA_OK(cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemDqs));
  int dev = 0, n_sm = 0;
  TT_CUDA_OK(cudaGetDevice(&dev));
  TT_CUDA_OK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  for (int g0 = 0; g0 < hkv; g0 += kv_heads_per_pass) {
    const int ng = hkv - g0 < kv_heads_per_pass ? hkv - g0 : kv_heads_per_pass;
    if (phases & TT_BWD_DKDV) {
      kdkdv<<<dim3(ng, n_kt), kThreads, kSmemDkdv, st>>>(
          mq, mk, mv, mdo, n_q, n_kv, rep, kv_lo, kv_hi, bwd_ptr, bwd_list, lse, delta,
          scale_log2, scale, dk, dk_st, dk_sh, dv, dv_st, dv_sh, kt_order, status, g0,
          static_cast<uint8_t*>(ds_ws), e2f, n_pairs);
      ++launches;
    }
    if (phases & TT_BWD_DQ) {
      const int n_items = ng * rep * n_qt;
      kdq<<<n_items < n_sm ? n_items : n_sm, kThreadsDqs, kSmemDqs, st>>>(
          mk, n_q, rep, g0 * rep, ng * rep, n_qt, fwd_ptr, fwd_list,
          static_cast<const uint8_t*>(ds_ws), n_pairs, scale, dq, dq_st, dq_sh, status);
      ++launches;
    }
  }
  tt_count_launches(launches);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}
