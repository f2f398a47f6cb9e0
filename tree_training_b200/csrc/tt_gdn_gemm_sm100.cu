// Segmented fp32 GEMM of the tree GDN on the 5th-generation tensor cores.
//
// The tree GDN (tt_gdn.cu) expresses each node's chunk step as small GEMMs
// over that node's tokens (L x L, L x D and D x D products, any node length),
// batched over all nodes of a level and all heads as one list of 128 x 128
// output tiles.  This kernel runs such a list with tcgen05.mma kind::tf32:
//
//   warps 0-3  producers: stream each tile's K range as 32-wide slices of A
//              (128 x 32) and B (32 x 128) into a ring of shared-memory
//              stages with 16-byte cp.async copies (zero-filled past the
//              segment's edges), laid out in the swizzled canonical forms
//              the MMA reads: K-major (128-byte swizzle) when the operand is
//              contiguous along K in global memory, MN-major (128-byte
//              swizzle on a 32-byte base, the one MN-major form for 32-bit
//              operands) when it is contiguous along M (or N).  In 3xTF32 mode each producer then splits the
//              elements it copied into a TF32 head (round to nearest) and a
//              TF32 tail, written to a second copy of the stage.
//   warp 8     MMA issuer: 4 MMAs of 128 x 128 x 8 per slice (12 in 3xTF32
//              mode: lo*hi, hi*lo, hi*hi) into one of two TMEM accumulators,
//              then releases the stage; at the end of a tile it hands the
//              accumulator to the epilogue and moves on to the next tile in
//              the other one.
//   warps 4-7  epilogue: C = alpha * acc + beta * Cin (Cin defaults to C).
//              Each warp reads its 32 accumulator rows (TMEM lanes) 32
//              columns at a time, transposes them through shared memory and
//              stores whole 128-byte row segments.
//
// The CTAs are persistent (one per SM, tiles x heads dealt round robin), so
// the slices of the next tile stream in while the current one finishes.
// Every wait is bounded (2 s); on expiry the kernel records
// TT_ERR_DEVICE_TIMEOUT in a device status word, drains its copies and MMAs,
// frees its tensor memory and returns.
#include <cstring>
#include <mutex>

#include "tt_gdn_gemm.cuh"
#include "tt_sm100.cuh"

namespace tt {
namespace gdn {
namespace {

using namespace tt::sm100;

constexpr int kTM = kTcTile, kTN = kTcTile, kTK = 32;   // tile, K slice (fp32 elements)
constexpr int kProducerWarps = 4, kEpilogueWarps = 4;
constexpr int kMmaWarp = kProducerWarps + kEpilogueWarps;   // warp 8
constexpr int kThreads = (kMmaWarp + 1) * 32;
constexpr int kProducers = kProducerWarps * 32;
constexpr int kOpBytes = kTM * kTK * 4;                 // one 128 x 32 fp32 operand slice
constexpr int kChunksPerThread = kOpBytes / 16 / kProducers;   // 16-byte chunks (8)
constexpr uint32_t kTmemCols = 256;                     // two 128-column accumulators
constexpr int kMaxStages = 6;

template <int kSplit>
struct Ring {
  static constexpr int kStageBytes = (kSplit == 3 ? 4 : 2) * kOpBytes;   // A, B (+ lo copies)
  static constexpr int kStages = kSplit == 3 ? 2 : 4;
  static constexpr int kLag = kStages - 1;   // slices in flight per producer thread
};

struct Bars {
  uint64_t full[kMaxStages];    // producers -> MMA (kProducers arrivals; TMA + TF32: one + bytes)
  uint64_t landed[kMaxStages];  // TMA + 3xTF32: the stage's copies landed (bytes)
  uint64_t empty[kMaxStages];   // MMA -> producers (commit)
  uint64_t acc_full[2];         // MMA -> epilogue (commit)
  uint64_t acc_empty[2];        // epilogue -> MMA (128 arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};

// Epilogue staging: per epilogue warp a 32 x 32 block of the accumulator,
// padded to 33 columns (conflict-free row writes and column reads).
constexpr int kStgPitch = 33;
constexpr int kStgBytes = kEpilogueWarps * 32 * kStgPitch * 4;
// C_in of the tile, prefetched by the epilogue warps (each its 32 rows x 128
// columns) before they wait for the accumulator, so the reads of C_in overlap
// the tile's main loop instead of stalling the epilogue row by row.
constexpr int kCinBytes = kEpilogueWarps * 32 * kTN * 4;
// per epilogue warp the tile's 128 column gammas of a decay-masked product
constexpr int kGcolBytes = kEpilogueWarps * kTN * 4;
// epilogue options a launch can use (host-checked alignment)
constexpr int kEpiCinAsync = 1;   // C_in rows 16-byte aligned: prefetch them by cp.async
constexpr int kEpiVecC = 2;       // C rows 16-byte aligned: 16-byte stores

template <int kSplit>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)Ring<kSplit>::kStages * Ring<kSplit>::kStageBytes + kStgBytes +
         kCinBytes + kGcolBytes + sizeof(Bars);
}

__device__ int32_t g_status;   // first error of any launch since the last take

__device__ __forceinline__ void record_error(Bars* sh, int32_t code) {
  atomicCAS(&g_status, 0, code);
  *reinterpret_cast<volatile int32_t*>(&sh->abort) = 1;
}

// 16-byte global -> shared copy of `bytes` (0, 4, 8, 12 or 16) source bytes;
// the rest of the 16 destination bytes is zero-filled.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
// 4-byte global -> shared copy (`bytes` 0 or 4; 0 zero-fills)
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The K slices [k_begin, k_begin + n * kTK) of a tile that can hold nonzero
// products (the segment's triangular structure, kKFull ... kKFromCol).
__device__ __forceinline__ void k_range(const SegDesc& sd, int i0, int j0, int& kb, int& n) {
  int ke = sd.K;
  kb = 0;
  switch (sd.kmode) {
    case kKToRow: ke = min(ke, i0 + kTM); break;
    case kKFromRow: kb = i0; break;
    case kKToCol: ke = min(ke, j0 + kTN); break;
    case kKFromCol: kb = j0; break;
    case kKLowerC: ke = j0 >= i0 + kTM ? 0 : ke; break;
    default: break;
  }
  n = ke > kb ? (ke - kb + kTK - 1) / kTK : 0;
}

// x rounded to TF32 (nearest, ties away), as an fp32 bit pattern: the
// conversion leaves the 13 low mantissa bits unspecified, so they are cleared.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r & 0xFFFFE000u;
}

// kind::tf32 instruction descriptor: fp32 accumulator, TF32 A and B, M = N = 128.
__device__ __forceinline__ uint32_t idesc_tf32(bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Byte offset, within one operand slice, of this thread's i-th 16-byte chunk
// and the (mn, k) coordinates of its first element.
//   K-major (128-byte swizzle): 128 rows (mn) of 32 k, 128-byte rows, 8-row
//     atoms of 1 KiB; 16-byte chunk c of row r sits at chunk c ^ (r & 7).
//   MN-major (128-byte swizzle on a 32-byte base, the layout the tensor core
//     takes for 32-bit MN-major operands): four 32-element mn blocks 4 KiB
//     apart, each 32 k-rows of 128 bytes in 4-row atoms of 512 bytes; 32-byte
//     granule g of row k sits at granule g ^ (k & 3).
__device__ __forceinline__ uint32_t chunk_at(bool k_contig, int q, int& mn, int& k) {
  if (k_contig) {
    const int r = q >> 3, kc = q & 7;
    mn = r;
    k = kc * 4;
    return (uint32_t)(r * 128 + ((kc ^ (r & 7)) << 4));
  }
  const int kr = q >> 5, mc = q & 31, j = mc & 7;
  mn = mc * 4;
  k = kr;
  return (uint32_t)((mc >> 3) * 4096 + kr * 128 + ((((j >> 1) ^ (kr & 3)) << 5) | ((j & 1) << 4)));
}

// Shared-memory descriptor of an MN-major 32-bit operand in the layout above:
// lead = bytes between 32-element mn blocks, stride = bytes between 4-row k
// atoms, layout type 1 (128-byte swizzle, 32-byte base).
__device__ __forceinline__ uint64_t desc_mn32(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)1 << 61;  // SWIZZLE_128B_BASE32B
  return d;
}

// Descriptor of operand slice `addr` for the MMA of K step kk (8 k each).
__device__ __forceinline__ uint64_t op_desc(uint32_t addr, bool k_contig, int kk) {
  // K-major: +32 bytes per K step inside the 128-byte rows; MN-major: +8 rows
  return k_contig ? desc_sw128(addr + kk * 32, 16, 1024)
                  : desc_mn32(addr + kk * 1024, 4096, 512);
}

// Issue this thread's copies of one operand slice: element (mn, k) of the
// operand at base + mn * mn_st + k * k_st, mn < mn_ext, k < k_ext.
__device__ __forceinline__ void copy_slice(uint32_t dst, const float* base, int mn0, int mn_ext,
                                           int k0, int k_ext, long long mn_st, long long k_st,
                                           bool k_contig, int tid) {
#pragma unroll
  for (int i = 0; i < kChunksPerThread; ++i) {
    int mn, k;
    const uint32_t off = chunk_at(k_contig, i * kProducers + tid, mn, k);
    mn += mn0;
    k += k0;
    int n_el;
    if (k_contig)
      n_el = mn < mn_ext ? min(max(k_ext - k, 0), 4) : 0;
    else
      n_el = k < k_ext ? min(max(mn_ext - mn, 0), 4) : 0;
    const float* src = n_el > 0 ? base + (long long)mn * mn_st + (long long)k * k_st : base;
    cp_async16(dst + off, src, (uint32_t)n_el * 4u);
  }
}

// 3xTF32: replace this thread's chunks of an operand slice by their rounded
// TF32 heads and write the TF32 tails 2 * kOpBytes further on.
__device__ __forceinline__ void split_slice(uint8_t* op, bool k_contig, int tid) {
#pragma unroll
  for (int i = 0; i < kChunksPerThread; ++i) {
    int mn, k;
    const uint32_t off = chunk_at(k_contig, i * kProducers + tid, mn, k);
    float4* hp = reinterpret_cast<float4*>(op + off);
    float4* lp = reinterpret_cast<float4*>(op + off + 2 * kOpBytes);
    const float4 a = *hp;
    const uint32_t h0 = to_tf32(a.x), h1 = to_tf32(a.y), h2 = to_tf32(a.z), h3 = to_tf32(a.w);
    const float4 hi = make_float4(__uint_as_float(h0), __uint_as_float(h1), __uint_as_float(h2),
                                  __uint_as_float(h3));
    const float4 lo = make_float4(__uint_as_float(to_tf32(a.x - hi.x)),
                                  __uint_as_float(to_tf32(a.y - hi.y)),
                                  __uint_as_float(to_tf32(a.z - hi.z)),
                                  __uint_as_float(to_tf32(a.w - hi.w)));
    *hp = hi;
    *lp = lo;
  }
}

// A CTA's items (tile x head, strided by the grid) with their descriptors
// fetched one item ahead: the next item's tile record is loaded as an item
// starts and its segment descriptor once the item's work has been issued, so
// neither dependent load stalls the item in flight.
struct ItemFetch {
  const SegDesc* segs;
  const int2* tiles;
  int H, n_items, stride, next;
  int2 tl_next;
  SegDesc sd_next;
  __device__ __forceinline__ ItemFetch(const SegDesc* s, const int2* t, int h, int n, int first,
                                       int st)
      : segs(s), tiles(t), H(h), n_items(n), stride(st), next(first) {
    if (next < n_items) {
      tl_next = tiles[next / H];
      sd_next = segs[tl_next.x];
    }
  }
  __device__ __forceinline__ void advance(int2& tl, SegDesc& sd) {
    tl = tl_next;
    sd = sd_next;
    next += stride;
    if (next < n_items) tl_next = tiles[next / H];
  }
  __device__ __forceinline__ void fetch_seg() {
    if (next < n_items) sd_next = segs[tl_next.x];
  }
};

// The K slices of an item: those of its segment, then (dual pair) those of
// the second product, read from the following segment and its tensor maps.
struct ItemSlices {
  int kb1, n1, kb2, n2;
  bool kc1a, kc1b, kc2a, kc2b;
  __device__ __forceinline__ ItemSlices(const SegDesc* segs, int seg, const SegDesc& sd, int i0,
                                        int j0) {
    k_range(sd, i0, j0, kb1, n1);
    kc1a = sd.a_cs == 1;
    kc1b = sd.b_rs == 1;
    kb2 = 0;
    n2 = 0;
    kc2a = kc2b = true;
    if (sd.dual) {   // only the second product's K range and layouts are needed
      const SegDesc* p2 = segs + seg + 1;
      SegDesc sd2;
      sd2.K = p2->K;
      sd2.kmode = p2->kmode;
      k_range(sd2, i0, j0, kb2, n2);
      kc2a = p2->a_cs == 1;
      kc2b = p2->b_rs == 1;
    }
  }
  __device__ __forceinline__ int count() const { return n1 + n2; }
  // slice t: which product, its K origin and operand layouts
  __device__ __forceinline__ void at(int t, int& prod, int& k0, bool& a_kc, bool& b_kc) const {
    prod = t < n1 ? 0 : 1;
    k0 = prod == 0 ? kb1 + t * kTK : kb2 + (t - n1) * kTK;
    a_kc = prod == 0 ? kc1a : kc2a;
    b_kc = prod == 0 ? kc1b : kc2b;
  }
};

// Tensor maps of one launch's segments (kernel parameter space): map 2 i is
// operand A of segment seg_first + i, map 2 i + 1 its operand B.
constexpr int kMaxSegsPerLaunch = 120;
struct MapPack {
  CUtensorMap m[2 * kMaxSegsPerLaunch];
};

// TMA copy of one operand slice into its stage: K-contiguous operands are one
// 32 x 128 box (128-byte swizzle), MN-contiguous ones four 32 x 32 boxes
// (128-byte swizzle, 32-byte atoms), one per 32-element mn block.  Elements
// outside the segment are zero-filled by the copy.
__device__ __forceinline__ void tma_slice(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                          bool k_contig, int k0, int mn0, int h) {
  if (k_contig) {
    tma_load_3d(dst, map, bar, k0, mn0, h);
  } else {
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) tma_load_3d(dst + blk * 4096, map, bar, mn0 + 32 * blk, k0, h);
  }
}

constexpr float kLog2e = 1.4426950408889634f;

template <int kSplit, bool kTma>
__device__ __forceinline__ void gemm_body(const SegDesc* __restrict__ segs,
                                          const int2* __restrict__ tiles, int n_tiles, int H,
                                          const float* __restrict__ A, long long a_hs,
                                          const float* __restrict__ B, long long b_hs, float* C,
                                          long long c_hs, float alpha, float beta,
                                          const float* Cin, const CUtensorMap* maps,
                                          int seg_first, int epi_flags, EpiMask mask) {
  using R = Ring<kSplit>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* stg_all = reinterpret_cast<float*>(ring + (size_t)R::kStages * R::kStageBytes);
  float* cin_all = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(stg_all) + kStgBytes);
  float* gcol_all = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(cin_all) + kCinBytes);
  Bars* sh = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(gcol_all) + kGcolBytes);
  const volatile int32_t* abort_flag = &sh->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = n_tiles * H;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R::kStages; ++s) {
      mbar_init(&sh->full[s], (kTma && kSplit == 1) ? 1 : kProducers);
      mbar_init(&sh->landed[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh->acc_full[b], 1);
      mbar_init(&sh->acc_empty[b], kEpilogueWarps * 32);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sh->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (kTma && warp < kProducerWarps) {
    // ------------------------------------------------------- producers (TMA)
    // thread 0 issues each slice's copies; with 3xTF32 every producer thread
    // then splits its share of the landed stage into TF32 heads and tails
    const int tid = threadIdx.x;
    uint32_t slot = 0;
    uint32_t issued = 0, parity = 0;   // per stage: loaded at least once / parity of last use
    bool ok = true;
    ItemFetch f(segs, tiles, H, n_items, blockIdx.x, gridDim.x);
    // with TF32 products only thread 0 has work here
    for (int item = blockIdx.x; item < n_items && ok && (kSplit == 3 || tid == 0);
         item += gridDim.x) {
      int2 tl;
      SegDesc sd;
      f.advance(tl, sd);
      const int h = item % H;
      const int i0 = (tl.y >> 16) * kTM, j0 = (tl.y & 0xFFFF) * kTN;
      const CUtensorMap* ma = maps + 2 * (tl.x - seg_first);
      const ItemSlices sl(segs, tl.x, sd, i0, j0);
      const int nk = sl.count();
      for (int t = 0; t < nk; ++t, ++slot) {
        const int s = slot % R::kStages;
        const uint32_t use = slot / R::kStages;
        uint8_t* st = ring + (size_t)s * R::kStageBytes;
        if (tid == 0) {
          if (slot >= (uint32_t)R::kStages &&
              !mbar_wait(&sh->empty[s], (use - 1) & 1, abort_flag)) {
            ok = false;
          } else {
            int prod, k0;
            bool a_kc, b_kc;
            sl.at(t, prod, k0, a_kc, b_kc);
            const CUtensorMap* mp_ = ma + 2 * prod;   // the pair's second segment: next maps
            uint64_t* bar = kSplit == 3 ? &sh->landed[s] : &sh->full[s];
            mbar_arrive_expect_tx(bar, 2 * kOpBytes);
            tma_slice(st, mp_, bar, a_kc, k0, i0, h);
            tma_slice(st + kOpBytes, mp_ + 1, bar, b_kc, k0, j0, h);
            issued |= 1u << s;
            parity = (parity & ~(1u << s)) | ((use & 1u) << s);
          }
        }
        if constexpr (kSplit == 3) {
          if (ok && mbar_wait(&sh->landed[s], use & 1, abort_flag)) {
            float4* p = reinterpret_cast<float4*>(st);
#pragma unroll 4
            for (int i = 0; i < 2 * kOpBytes / 16 / kProducers; ++i) {
              const int q = i * kProducers + tid;
              const float4 a = p[q];
              const float4 hi = make_float4(
                  __uint_as_float(to_tf32(a.x)), __uint_as_float(to_tf32(a.y)),
                  __uint_as_float(to_tf32(a.z)), __uint_as_float(to_tf32(a.w)));
              p[q] = hi;
              p[q + 2 * kOpBytes / 16] = make_float4(
                  __uint_as_float(to_tf32(a.x - hi.x)), __uint_as_float(to_tf32(a.y - hi.y)),
                  __uint_as_float(to_tf32(a.z - hi.z)), __uint_as_float(to_tf32(a.w - hi.w)));
            }
            fence_proxy_async_smem();
            mbar_arrive(&sh->full[s]);
          } else {
            ok = false;
          }
        }
        if (!ok) break;
      }
      f.fetch_seg();
    }
    if (!ok) {
      record_error(sh, TT_ERR_DEVICE_TIMEOUT);
      if (tid == 0) {
        // the last copies into each stage land before the CTA exits
        for (int s = 0; s < R::kStages; ++s)
          if ((issued >> s) & 1u)
            mbar_wait(kSplit == 3 ? &sh->landed[s] : &sh->full[s], (parity >> s) & 1u, nullptr);
      }
    }
  } else if (warp < kProducerWarps) {
    // -------------------------------------------------- producers (cp.async)
    const int tid = threadIdx.x;
    uint32_t slot = 0;       // slices issued so far (all items)
    uint32_t done = 0;       // slices handed to the MMA so far
    uint32_t layouts = 0;    // 2 bits per ring stage: A K-contiguous, B K-contiguous
    bool ok = true;
    // hand slice `done` to the MMA once this thread's copies of it landed
    auto finish = [&](void) {
      const int s = done % R::kStages;
      if constexpr (kSplit == 3) {
        uint8_t* st = ring + (size_t)s * R::kStageBytes;
        const uint32_t lay = layouts >> (2 * s);
        split_slice(st, lay & 1u, tid);
        split_slice(st + kOpBytes, (lay >> 1) & 1u, tid);
      }
      fence_proxy_async_smem();
      mbar_arrive(&sh->full[s]);
      ++done;
    };
    ItemFetch f(segs, tiles, H, n_items, blockIdx.x, gridDim.x);
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      int2 tl;
      SegDesc sd;
      f.advance(tl, sd);
      const int h = item % H;
      const int i0 = (tl.y >> 16) * kTM, j0 = (tl.y & 0xFFFF) * kTN;
      const float* a = A + h * a_hs + sd.a_off;
      const float* b = B + h * b_hs + sd.b_off;
      const bool a_kc = sd.a_cs == 1, b_kc = sd.b_rs == 1;
      int kb, nk;
      k_range(sd, i0, j0, kb, nk);
      for (int t = 0; t < nk; ++t, ++slot) {
        const int s = slot % R::kStages;
        if (slot >= (uint32_t)R::kStages &&
            !mbar_wait(&sh->empty[s], ((slot / R::kStages) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t st = smem_u32(ring + (size_t)s * R::kStageBytes);
        // A(r, k) at r * a_rs + k * a_cs; B(k, n) at k * b_rs + n * b_cs
        copy_slice(st, a, i0, sd.M, kb + t * kTK, sd.K, sd.a_rs, sd.a_cs, a_kc, tid);
        copy_slice(st + kOpBytes, b, j0, sd.N, kb + t * kTK, sd.K, sd.b_cs, sd.b_rs, b_kc, tid);
        cp_async_commit();
        layouts = (layouts & ~(3u << (2 * s))) | ((a_kc ? 1u : 0u) << (2 * s)) |
                  ((b_kc ? 2u : 0u) << (2 * s));
        if (slot + 1 - done > (uint32_t)R::kLag) {
          cp_async_wait<R::kLag - 1>();
          finish();
        }
      }
      f.fetch_seg();
    }
    cp_async_wait<0>();
    if (ok) {
      while (done < slot) finish();
    } else {
      record_error(sh, TT_ERR_DEVICE_TIMEOUT);
    }
  } else if (warp == kMmaWarp) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t slot = 0;
      int acc_i = 0;
      bool ok = true;
      const uint32_t ring0 = smem_u32(ring);
      ItemFetch f(segs, tiles, H, n_items, blockIdx.x, gridDim.x);
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++acc_i) {
        int2 tl;
        SegDesc sd;
        f.advance(tl, sd);
        const ItemSlices sl(segs, tl.x, sd, (tl.y >> 16) * kTM, (tl.y & 0xFFFF) * kTN);
        const int nk = sl.count();
        const int buf = acc_i & 1;
        if (acc_i >= 2 && !mbar_wait(&sh->acc_empty[buf], ((acc_i >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * kTN;
        for (int t = 0; t < nk; ++t, ++slot) {
          const int s = slot % R::kStages;
          int prod, k0;
          bool a_kc, b_kc;
          sl.at(t, prod, k0, a_kc, b_kc);
          const uint32_t idesc = idesc_tf32(!a_kc, !b_kc);
          if (!mbar_wait(&sh->full[s], (slot / R::kStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = ring0 + s * R::kStageBytes, sb = sa + kOpBytes;
#pragma unroll
          for (int kk = 0; kk < kTK / 8; ++kk) {
            const uint64_t da = op_desc(sa, a_kc, kk);
            const uint64_t db = op_desc(sb, b_kc, kk);
            const uint32_t acc0 = (t > 0 || kk > 0) ? 1u : 0u;
            if constexpr (kSplit == 3) {
              const uint64_t da_lo = op_desc(sa + 2 * kOpBytes, a_kc, kk);
              const uint64_t db_lo = op_desc(sb + 2 * kOpBytes, b_kc, kk);
              mma_tf32(d, da_lo, db, idesc, acc0);
              mma_tf32(d, da, db_lo, idesc, 1u);
              mma_tf32(d, da, db, idesc, 1u);
            } else {
              mma_tf32(d, da, db, idesc, acc0);
            }
          }
          tc_commit(&sh->empty[s]);
        }
        if (!ok) break;
        tc_commit(&sh->acc_full[buf]);
        f.fetch_seg();
      }
      if (!ok) record_error(sh, TT_ERR_DEVICE_TIMEOUT);
      // every MMA issued has completed before the accumulators are freed
      tc_commit(&sh->drain);
      mbar_wait(&sh->drain, 0, nullptr);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    int acc_i = 0;
    ItemFetch f(segs, tiles, H, n_items, blockIdx.x, gridDim.x);
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++acc_i) {
      int2 tl;
      SegDesc sd;
      f.advance(tl, sd);
      const int h = item % H;
      const int i0 = (tl.y >> 16) * kTM, j0 = (tl.y & 0xFFFF) * kTN;
      const int buf = acc_i & 1;
      const float* cin = Cin ? Cin : C;
      const long long hoff = h * c_hs + sd.c_off;
      const int rows = sd.M - (i0 + quad * 32);      // rows of this warp's block in C
      // C_in prefetch: lane l copies columns [4l, 4l + 4) of each of the warp's
      // 32 rows (one 512-byte row segment per instruction), zero-filled past
      // the segment; it lands while the tile's MMAs run.  Row r's 16-byte
      // chunk c sits at slot c ^ r of the row, so a warp reading one chunk of
      // each of its 32 rows spreads over every bank.
      float* cinb = cin_all + quad * 32 * kTN;
      const bool pre = (epi_flags & kEpiCinAsync) && beta != 0.f;
      // 16-byte stores need 16-byte aligned rows of C, and C_in (if any)
      // already in shared memory
      const bool vec = (epi_flags & kEpiVecC) && (beta == 0.f || pre);
      if (pre) {
        const int col = j0 + 4 * lane;
        const int ncol = min(max(sd.N - col, 0), 4);
        const float* base = cin + hoff + (long long)(i0 + quad * 32) * sd.c_rs + col;
        const uint32_t dst0 = smem_u32(cinb);
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
          const int n_el = r < rows ? ncol : 0;
          cp_async16(dst0 + r * kTN * 4 + ((lane ^ r) << 4),
                     n_el > 0 ? base + (long long)r * sd.c_rs : cin, (uint32_t)n_el * 4u);
        }
        cp_async_commit();
      }
      // decay mask: this lane's row gamma (vec path, log2 units) and the
      // tile's 128 column gammas, copied into this warp's shared-memory row
      // before the accumulator wait (they land while the MMAs run)
      const int row_t = i0 + quad * 32 + lane;
      const float* gam_h =
          mask.mode != kMaskNone ? mask.gam + h * mask.gam_hs + sd.tok0 : nullptr;
      float g_row = 0.f;
      float* gcb = gcol_all + quad * kTN;
      if (kTma && mask.mode != kMaskNone) {
        if (row_t < sd.M) g_row = gam_h[row_t] * kLog2e;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = j0 + 4 * lane + e;
          cp_async4(smem_u32(gcb + 4 * lane + e), m < sd.N ? gam_h + m : gam_h,
                    m < sd.N ? 4u : 0u);
        }
        cp_async_commit();
      }
      bool ok = mbar_wait(&sh->acc_full[buf], (acc_i >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        cp_async_wait<0>();                    // the copies land before the CTA exits
        record_error(sh, TT_ERR_DEVICE_TIMEOUT);
        break;
      }
      tc_fence_after();
      if (pre) {
        cp_async_wait<0>();
        __syncwarp();
      }
      if (kTma && mask.mode != kMaskNone) {
        cp_async_wait<0>();
        __syncwarp();
      }
      bool empty_k;                            // no MMA wrote this accumulator
      {
        int kb, nk;
        k_range(sd, i0, j0, kb, nk);
        if (nk == 0 && sd.dual) {
          SegDesc sd2;
          sd2.K = segs[tl.x + 1].K;
          sd2.kmode = segs[tl.x + 1].kmode;
          k_range(sd2, i0, j0, kb, nk);
        }
        empty_k = nk == 0;
      }
      // without 16-byte aligned rows of C, each 32 x 32 block goes through
      // shared memory so that the warp stores (and reads C_in) one 128-byte
      // row segment per instruction
      float* stg = stg_all + quad * 32 * kStgPitch;
#pragma unroll 1
      for (int cc = 0; cc < kTN / 32; ++cc) {
        float v[32];
        tmem_ld32(lane_addr + buf * kTN + cc * 32, v);
        // (the TMA-staged kernel only: the cp.async one takes no mask).  The
        // decay is exp(gam_i - gam_m) = 2^(log2e gam_i - log2e gam_m), on the
        // SFU (about 2 ulp); masked columns select 0.
        if (kTma && mask.mode != kMaskNone && !empty_k) {   // lane = row of the block
          const int c0 = j0 + cc * 32;
          const bool strict = mask.mode == kMaskA;
          const float sgn = strict ? -1.f : 1.f;
          const int lim = strict ? row_t : row_t + 1;   // kept columns: m < lim
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float d = fast_exp2(fmaf(-gcb[cc * 32 + i], kLog2e, g_row));
            v[i] = c0 + i < lim ? sgn * v[i] * d : 0.f;
          }
        }
        if (vec) {
          // straight from the accumulator rows: lane = row, eight 16-byte
          // stores of its 32 columns (no staging through shared memory)
          const long long orow = hoff + (long long)(i0 + quad * 32 + lane) * sd.c_rs;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int c = cc * 8 + k;                 // 16-byte chunk of the tile row
            const int ncol = min(max(sd.N - (j0 + 4 * c), 0), 4);
            float4 x = empty_k ? make_float4(0.f, 0.f, 0.f, 0.f)
                               : make_float4(alpha * v[4 * k], alpha * v[4 * k + 1],
                                             alpha * v[4 * k + 2], alpha * v[4 * k + 3]);
            if (pre) {
              const float4 cv =
                  *reinterpret_cast<const float4*>(cinb + lane * kTN + ((c ^ lane) << 2));
              x.x += beta * cv.x;
              x.y += beta * cv.y;
              x.z += beta * cv.z;
              x.w += beta * cv.w;
            }
            if (lane < rows && ncol > 0) {
              float* dst = C + orow + j0 + 4 * c;
              if (ncol == 4) {
                *reinterpret_cast<float4*>(dst) = x;
              } else {
                dst[0] = x.x;
                if (ncol > 1) dst[1] = x.y;
                if (ncol > 2) dst[2] = x.z;
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) stg[lane * kStgPitch + i] = empty_k ? 0.f : alpha * v[i];
          __syncwarp();
          const int gj = j0 + cc * 32 + lane;
          if (gj < sd.N && rows > 0) {
            const long long o0 = hoff + (long long)(i0 + quad * 32) * sd.c_rs + gj;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              float cv[16];
              if (pre) {
#pragma unroll
                for (int rr = 0; rr < 16; ++rr) {
                  const int r = half * 16 + rr;
                  cv[rr] = cinb[r * kTN + (((cc * 8 + (lane >> 2)) ^ r) << 2) + (lane & 3)];
                }
              } else if (beta != 0.f) {
                // 16 rows' C_in loads in flight before the first store
#pragma unroll
                for (int rr = 0; rr < 16; ++rr) {
                  const int r = half * 16 + rr;
                  cv[rr] = r < rows ? cin[o0 + (long long)r * sd.c_rs] : 0.f;
                }
              }
#pragma unroll
              for (int rr = 0; rr < 16; ++rr) {
                const int r = half * 16 + rr;
                if (r < rows) {
                  float x = stg[r * kStgPitch + lane];
                  if (beta != 0.f) x += beta * cv[rr];
                  C[o0 + (long long)r * sd.c_rs] = x;
                }
              }
            }
          }
          __syncwarp();
        }
      }
      __syncwarp();   // every lane is done with this tile's C_in and gamma rows
      tc_fence_before();
      mbar_arrive(&sh->acc_empty[buf]);
      f.fetch_seg();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Operands staged with 16-byte cp.async copies (any segment layout the
// tensor maps cannot describe).
template <int kSplit>
__global__ void __launch_bounds__(kThreads, 1)
seg_gemm_tc(const SegDesc* __restrict__ segs, const int2* __restrict__ tiles, int n_tiles, int H,
            const float* __restrict__ A, long long a_hs, const float* __restrict__ B,
            long long b_hs, float* C, long long c_hs, float alpha, float beta, const float* Cin,
            EpiMask mask) {
  gemm_body<kSplit, false>(segs, tiles, n_tiles, H, A, a_hs, B, b_hs, C, c_hs, alpha, beta, Cin,
                           nullptr, 0, 0, mask);
}

// Operands staged with TMA tile copies through per-segment tensor maps.
template <int kSplit>
__global__ void __launch_bounds__(kThreads, 1)
seg_gemm_tma(const __grid_constant__ MapPack mp, int seg_first,
             const SegDesc* __restrict__ segs, const int2* __restrict__ tiles, int n_tiles, int H,
             const float* __restrict__ A, long long a_hs, const float* __restrict__ B,
             long long b_hs, float* C, long long c_hs, float alpha, float beta, const float* Cin,
             int epi_flags, EpiMask mask) {
  gemm_body<kSplit, true>(segs, tiles, n_tiles, H, A, a_hs, B, b_hs, C, c_hs, alpha, beta, Cin,
                          mp.m, seg_first, epi_flags, mask);
}

constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices];
bool g_attr_set[kMaxDevices][4];
std::mutex g_mu;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map of one operand of one segment (3-D: inner, outer, head), or false
// when the driver does not accept the layout.  K-contiguous: inner = K, outer =
// M (or N), 32 x 128 boxes, 128-byte swizzle.  MN-contiguous: inner = M (or
// N), outer = K, 32 x 32 boxes, 128-byte swizzle on 32-byte atoms.
bool encode_operand(EncodeTiledFn fn, CUtensorMap* m, const float* base, bool k_contig,
                    long long mn_ext, long long k_ext, long long outer_stride, long long head_stride,
                    int H) {
  const long long inner = k_contig ? k_ext : mn_ext, outer = k_contig ? mn_ext : k_ext;
  if (inner <= 0 || outer <= 0 || H <= 0) return false;
  long long hs = head_stride;
  if (H == 1 || hs <= 0) hs = ((outer * outer_stride * 4 + 15) / 16) * 4;   // unused dim
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)H};
  const cuuint64_t strides[2] = {(cuuint64_t)outer_stride * 4, (cuuint64_t)hs * 4};
  const cuuint32_t box[3] = {32u, k_contig ? (cuuint32_t)kTM : 32u, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r =
      fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE,
         k_contig ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace
}  // namespace gdn
}  // namespace tt

using tt::gdn::SegDesc;

bool tt_gdn_tc_gemm_supported(const SegDesc* d, int first, int count, const float* A,
                              long long a_hs, const float* B, long long b_hs, const float* C,
                              long long c_hs) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  (void)C;
  (void)c_hs;
  if (!al(A) || !al(B) || (a_hs & 3) || (b_hs & 3)) return false;
  for (int i = first; i < first + count; ++i) {
    const SegDesc& s = d[i];
    const bool a_ok = (s.a_cs == 1 && (s.a_rs & 3) == 0) || (s.a_rs == 1 && (s.a_cs & 3) == 0);
    const bool b_ok = (s.b_rs == 1 && (s.b_cs & 3) == 0) || (s.b_cs == 1 && (s.b_rs & 3) == 0);
    if (!a_ok || !b_ok || s.c_cs != 1 || (s.a_off & 3) || (s.b_off & 3)) return false;
  }
  return true;
}

int tt_gdn_seg_gemm_tc(const SegDesc* d_desc, const int2* d_tiles, int n_tiles, int H,
                       const float* A, long long a_hs, const float* B, long long b_hs, float* C,
                       long long c_hs, float alpha, float beta, const float* Cin, int split,
                       cudaStream_t st, tt::gdn::EpiMask mask) {
  using namespace tt::gdn;
  if (mask.mode != kMaskNone) return TT_ERR_UNSUPPORTED;   // masks: TMA-staged kernel only
  if (n_tiles <= 0 || H <= 0) return TT_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TT_ERR_CUDA;
  const int si = split == 3 ? 1 : 0;
  const size_t smem = split == 3 ? smem_bytes<3>() : smem_bytes<1>();
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_sms[dev] == 0 &&
        cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    if (!g_attr_set[dev][si]) {
      const cudaError_t e =
          split == 3 ? cudaFuncSetAttribute(seg_gemm_tc<3>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                     : cudaFuncSetAttribute(seg_gemm_tc<1>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return TT_ERR_CUDA;
      g_attr_set[dev][si] = true;
    }
  }
  const long long items = (long long)n_tiles * H;
  const int grid = (int)std::min<long long>(items, g_sms[dev]);
  if (split == 3)
    seg_gemm_tc<3><<<grid, kThreads, smem, st>>>(d_desc, d_tiles, n_tiles, H, A, a_hs, B, b_hs,
                                                  C, c_hs, alpha, beta, Cin, mask);
  else
    seg_gemm_tc<1><<<grid, kThreads, smem, st>>>(d_desc, d_tiles, n_tiles, H, A, a_hs, B, b_hs,
                                                  C, c_hs, alpha, beta, Cin, mask);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

int tt_gdn_seg_gemm_tma(const SegDesc* h_segs, int seg_first, int seg_count,
                        const SegDesc* d_desc, const int2* d_tiles, int n_tiles, int H,
                        const float* A, long long a_hs, const float* B, long long b_hs, float* C,
                        long long c_hs, float alpha, float beta, const float* Cin, int split,
                        cudaStream_t st, tt::gdn::EpiMask mask, tt::gdn::DualOperands dual) {
  using namespace tt::gdn;
  if (n_tiles <= 0 || H <= 0) return TT_OK;
  if (seg_count > kMaxSegsPerLaunch) return TT_ERR_INVALID_ARG;
  // a dual pair never straddles two launches
  if (seg_count > 0 && h_segs[seg_count - 1].dual) return TT_ERR_INVALID_ARG;
  const EncodeTiledFn fn = encoder();
  if (!fn) return TT_ERR_UNSUPPORTED;
  MapPack mp;
  std::memset(&mp, 0, sizeof(mp));
  for (int i = 0; i < seg_count; ++i) {
    const SegDesc& d = h_segs[i];
    if (d.M <= 0 || d.N <= 0 || d.K <= 0) continue;   // no tiles, or no slices to load
    const bool second = i > 0 && h_segs[i - 1].dual;  // the second product of a pair
    if (second && (!dual.A2 || !dual.B2)) return TT_ERR_INVALID_ARG;
    const float* Ab = second ? dual.A2 : A;
    const float* Bb = second ? dual.B2 : B;
    const long long ahs = second ? dual.a2_hs : a_hs, bhs = second ? dual.b2_hs : b_hs;
    const bool a_kc = d.a_cs == 1, b_kc = d.b_rs == 1;
    if (!encode_operand(fn, &mp.m[2 * i], Ab + d.a_off, a_kc, d.M, d.K, a_kc ? d.a_rs : d.a_cs,
                        ahs, H) ||
        !encode_operand(fn, &mp.m[2 * i + 1], Bb + d.b_off, b_kc, d.N, d.K,
                        b_kc ? d.b_cs : d.b_rs, bhs, H))
      return TT_ERR_UNSUPPORTED;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TT_ERR_CUDA;
  const int si = 2 + (split == 3 ? 1 : 0);
  const size_t smem = split == 3 ? smem_bytes<3>() : smem_bytes<1>();
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_sms[dev] == 0 &&
        cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return TT_ERR_CUDA;
    if (!g_attr_set[dev][si]) {
      const cudaError_t e =
          split == 3 ? cudaFuncSetAttribute(seg_gemm_tma<3>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                     : cudaFuncSetAttribute(seg_gemm_tma<1>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return TT_ERR_CUDA;
      g_attr_set[dev][si] = true;
    }
  }
  // the epilogue's 16-byte C_in prefetch and C stores need every row of C_in
  // and C 16-byte aligned
  const float* cin = Cin ? Cin : C;
  bool rows16 = (c_hs & 3) == 0;
  for (int i = 0; i < seg_count && rows16; ++i)
    rows16 = (h_segs[i].c_off & 3) == 0 && (h_segs[i].c_rs & 3) == 0;
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int epi_flags = (rows16 && beta != 0.f && al16(cin) ? kEpiCinAsync : 0) |
                        (rows16 && al16(C) ? kEpiVecC : 0);
  const long long items = (long long)n_tiles * H;
  const int grid = (int)std::min<long long>(items, g_sms[dev]);
  if (split == 3)
    seg_gemm_tma<3><<<grid, kThreads, smem, st>>>(mp, seg_first, d_desc, d_tiles, n_tiles, H, A,
                                                   a_hs, B, b_hs, C, c_hs, alpha, beta, Cin,
                                                   epi_flags, mask);
  else
    seg_gemm_tma<1><<<grid, kThreads, smem, st>>>(mp, seg_first, d_desc, d_tiles, n_tiles, H, A,
                                                   a_hs, B, b_hs, C, c_hs, alpha, beta, Cin,
                                                   epi_flags, mask);
  return cudaGetLastError() == cudaSuccess ? TT_OK : TT_ERR_CUDA;
}

extern "C" int tt_gdn_take_device_status(int32_t* out) {
  if (!out) return TT_ERR_INVALID_ARG;
  int32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, tt::gdn::g_status, sizeof(v)) != cudaSuccess) return TT_ERR_CUDA;
  if (v != 0) {
    const int32_t zero = 0;
    if (cudaMemcpyToSymbol(tt::gdn::g_status, &zero, sizeof(zero)) != cudaSuccess)
      return TT_ERR_CUDA;
  }
  *out = v;
  return TT_OK;
}
