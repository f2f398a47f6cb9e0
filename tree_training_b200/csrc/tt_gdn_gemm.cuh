// Segmented GEMM descriptors shared by the tree GDN's host orchestration
// (tt_gdn.cu) and its tensor-core GEMM (tt_gdn_gemm_sm100.cu).
#pragma once

#include "tt_common.cuh"

namespace tt {
namespace gdn {

// One segment of a segmented GEMM  C = alpha * A B + beta * C  (per head):
// operand element (r, c) of A lives at a_off + r * a_rs + c * a_cs (plus the
// launch's head stride), likewise B and C.  Every operand has a unit stride
// in one of its two dimensions.
struct SegDesc {
  int M, N, K;
  int kmode;   // which part of the K range can hold nonzero products (kKFull, ...)
  int tok0;    // first token of the segment's node (the decay-mask epilogue)
  int dual;    // 1: the next segment is a second product added into this one's
               // output tile (its own A, B, K range; C fields unused), 0: none
  long long a_off, a_rs, a_cs;
  long long b_off, b_rs, b_cs;
  long long c_off, c_rs, c_cs;
};

// K ranges of a segment whose A or B is triangular (the tensor-core GEMM
// skips the K slices that only meet zeros; the CUDA-core GEMM multiplies them):
//   kKFull   every k;
//   kKToRow  A lower triangular (A[r][k] = 0 for k > r): k < row + 1;
//   kKFromRow A upper triangular (the transpose of a lower one): k >= row;
//   kKToCol  B upper triangular (B[k][n] = 0 for k > n): k < col + 1;
//   kKFromCol B lower triangular: k >= col;
//   kKLowerC every k, but only C's lower triangle is wanted (the decay-masked
//            K K^T / Q K^T): a tile entirely above the diagonal gets no K
//            slice, and the tensor-core GEMM's epilogue writes it as zeros.
enum { kKFull = 0, kKToRow = 1, kKFromRow = 2, kKToCol = 3, kKFromCol = 4, kKLowerC = 5 };

// Decay mask applied by the tensor-core GEMM's epilogue to an L x L product
// of one node (row i, column m, gam the per-token cumulative log decay of
// the node's tokens, head stride gam_hs):
//   kMaskA    C = -P * exp(gam_i - gam_m) for m < i, 0 elsewhere (A of the chunk)
//   kMaskAqk  C =  P * exp(gam_i - gam_m) for m <= i, 0 elsewhere (the q-k weights)
enum { kMaskNone = 0, kMaskA = 1, kMaskAqk = 2 };
struct EpiMask {
  int mode = kMaskNone;
  const float* gam = nullptr;
  long long gam_hs = 0;
};

// Second operand pair of a launch whose segments come in dual pairs (see
// SegDesc::dual): the second segment of each pair reads A2 / B2.
struct DualOperands {
  const float* A2 = nullptr;
  long long a2_hs = 0;
  const float* B2 = nullptr;
  long long b2_hs = 0;
};

// Output tile edge of the tensor-core GEMM (tiles of the tile list are
// kTcTile x kTcTile; the CUDA-core GEMM uses 64 x 64).
constexpr int kTcTile = 128;

}  // namespace gdn
}  // namespace tt

// Tensor-core segmented GEMM over a list of 128 x 128 output tiles
// (tile = {segment index, tm << 16 | tn}) and H heads, fp32 in and out:
// split = 1 multiplies the operands as TF32 (10-bit mantissas), split = 3
// as the sum of three TF32 products (hi*hi + hi*lo + lo*hi, hi/lo the
// rounded TF32 head and tail of each fp32 value: close to fp32 products).
// Requirements (checked by tt_gdn_tc_gemm_supported): A and B with 16-byte
// aligned bases and every offset and non-unit stride a multiple of 4 floats
// (the operands are staged with 16-byte copies); C row-major (c_cs == 1).  Bounded waits report TT_ERR_DEVICE_TIMEOUT through
// tt_gdn_take_device_status.
// C = alpha A B + beta Cin, Cin (nullptr: C itself) with C's layout.
int tt_gdn_seg_gemm_tc(const tt::gdn::SegDesc* d_desc, const int2* d_tiles, int n_tiles, int H,
                       const float* A, long long a_hs, const float* B, long long b_hs, float* C,
                       long long c_hs, float alpha, float beta, const float* Cin, int split,
                       cudaStream_t st, tt::gdn::EpiMask mask = {});
// The same GEMM with the operand slices staged by TMA tile copies through
// tensor maps encoded here for each segment (the faster staging): segments
// seg_first .. seg_first + seg_count - 1 (at most 120; h_segs their host
// copies) and the tiles of exactly those segments.  TT_ERR_UNSUPPORTED when
// a segment's layout has no tensor map (the caller then uses
// tt_gdn_seg_gemm_tc).
int tt_gdn_seg_gemm_tma(const tt::gdn::SegDesc* h_segs, int seg_first, int seg_count,
                        const tt::gdn::SegDesc* d_desc, const int2* d_tiles, int n_tiles, int H,
                        const float* A, long long a_hs, const float* B, long long b_hs, float* C,
                        long long c_hs, float alpha, float beta, const float* Cin, int split,
                        cudaStream_t st, tt::gdn::EpiMask mask = {},
                        tt::gdn::DualOperands dual = {});
constexpr int kTmaMaxSegs = 120;
bool tt_gdn_tc_gemm_supported(const tt::gdn::SegDesc* h_desc, int first, int count,
                              const float* A, long long a_hs, const float* B, long long b_hs,
                              const float* C, long long c_hs);
