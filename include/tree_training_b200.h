/*
 * tree_training_b200 — C ABI of the B200 (sm_100a) tree-training hot path.
 *
 * Plain pointers and sizes only: no torch types cross this boundary.  Device
 * pointers are caller-owned (the library never allocates or frees caller
 * memory); `stream` is a cudaStream_t passed as void*.  Every function
 * returns a TT_* status; kernels never trap or assert: a bounded device wait
 * that gives up writes a nonzero code into `*status` (a device int32 the
 * caller may poll), and the host-side launcher returns TT_ERR_CUDA when a
 * launch fails.
 *
 * Index conventions (one packed sequence, batch 1, as in the reference):
 *   query rows    i in [0, n_q)   — the tokens of one partition in DFS order
 *   key columns   j in [0, n_kv)  — gateway tokens first, then the partition
 *   key j is visible to query rows [kv_lo[j], kv_hi[j]).
 * Tensors are [tokens, heads, head_dim] with the last dim contiguous; token
 * and head strides are given in elements.
 *
 * Reference citations are file:line inside Jinghui-Wang/tree-training
 * (TF/ = transformers 5.5 site-packages, which the reference calls into).
 */
#ifndef TREE_TRAINING_B200_H
#define TREE_TRAINING_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tt_status {
  TT_OK = 0,
  TT_ERR_INVALID_ARG = 1,    /* bad size, pointer, or a forest that is not in pre-order */
  TT_ERR_UNSUPPORTED = 2,    /* dtype / head_dim / stride combination not implemented */
  TT_ERR_CUDA = 3,           /* a CUDA runtime call or launch failed */
  TT_ERR_DEVICE_TIMEOUT = 4, /* a bounded device wait gave up (written to *status) */
  TT_ERR_NOT_INTERVAL = 5,   /* a mask column is not one contiguous run of rows */
  TT_ERR_WORKSPACE = 6,      /* workspace smaller than the *_workspace_size answer */
  TT_ERR_CAPACITY = 7        /* an output list is shorter than needed */
};

enum tt_dtype { TT_F32 = 0, TT_BF16 = 1, TT_F16 = 2, TT_U8 = 3 };

/* Human-readable text of a status code (static storage). */
const char* tt_status_string(int status);

/* ABI version; bumped on any signature change. */
int tt_abi_version(void);

/* Kernel path for the attention entry points: 0 = automatic (tcgen05 for
 * bf16/f16 head_dim 128, exact CUDA-core kernels otherwise), 1 = always the
 * exact CUDA-core kernels (used to cross-check the tensor-core path).  The
 * environment variable TT_KERNEL_PATH=1 sets the initial value.  Returns the
 * previous setting.  Tile shapes (tt_attn_tile_shape) follow this setting. */
int tt_set_kernel_path(int path);

/* Number of CUDA kernels this library has launched since it was loaded
 * (all entry points, all devices).  Lets a benchmark report how many of its
 * own kernels ran inside a timed region. */
int64_t tt_kernel_launches(void);

/* Floating-point operations (2 M N K per segment and head) of the tree GDN's
 * segmented GEMMs launched since the library was loaded: the algorithmic
 * GEMM work, excluding the padding of partial 64 x 64 tiles. */
int64_t tt_gdn_gemm_flops(void);

/* The part of tt_gdn_gemm_flops that ran on the tensor cores (tcgen05.mma
 * kind::tf32). */
int64_t tt_gdn_gemm_tc_flops(void);

/* Selects the tree GDN's GEMM engine; returns the previous mode.
 * 0 (default, or environment TT_GDN_GEMM unset): tensor cores, with 3xTF32
 *   products (hi*hi + hi*lo + lo*hi of the rounded TF32 head and tail of each
 *   fp32 operand) when the GDN's inputs are fp32 and TF32 products when they
 *   are bf16/fp16;
 * 1: tensor cores with 3xTF32 products for every input type;
 * 2: the CUDA-core fp32 FMA GEMM;
 * adding 4 to mode 0 or 1 stages the tensor cores' operands with cp.async
 * copies instead of TMA tile copies (for comparisons).
 * Launches whose operands are not 16-byte aligned use the CUDA-core GEMM. */
int tt_gdn_set_gemm_mode(int mode);

/* One segmented GEMM of the tree GDN's engine, for testing the engines
 * against each other: C = alpha * A B + beta * C per segment and head.
 * segs: n_segs rows of 13 int64 (M, N, K, kmode, a_off, a_rs, a_cs, b_off,
 * b_rs, b_cs, c_off, c_rs, c_cs), element (r, c) of A at A + h * a_hs +
 * a_off + r * a_rs + c * a_cs, likewise B and C; kmode 0 multiplies the whole
 * K range, 1-4 skip the K slices a triangular operand leaves zero (1: A lower,
 * 2: A upper, 3: B upper, 4: B lower triangular).  engine 0 = CUDA-core fp32
 * FMA, 1 = tensor cores with TF32 products, 3 = tensor cores with 3xTF32
 * products, operands staged by TMA; 5 / 7 = the same with cp.async staging
 * (TT_ERR_UNSUPPORTED unless A's and B's bases are 16-byte aligned,
 * their offsets and non-unit strides multiples of 4, and c_cs == 1).  Device
 * pointers; synchronises the stream before returning.  Workspace:
 * tt_gdn_segmented_gemm_workspace_size(n_segs, segs) bytes.  No counterpart
 * in the reference (a test hook of the engine behind tt_gdn_tree_fwd/_bwd). */
int64_t tt_gdn_segmented_gemm_workspace_size(int32_t n_segs, const int64_t* segs);
int tt_gdn_segmented_gemm(int engine, int32_t n_segs, const int64_t* segs, int32_t H,
                          const float* A, int64_t a_hs, const float* B, int64_t b_hs, float* C,
                          int64_t c_hs, float alpha, float beta, void* workspace,
                          int64_t workspace_bytes, void* stream);

/* Copies into *out, then clears, the first error recorded by a tree-GDN
 * tensor-core kernel on the current device since the last call
 * (TT_ERR_DEVICE_TIMEOUT when a bounded wait expired; 0 = none).
 * Synchronises with the device. */
int tt_gdn_take_device_status(int32_t* out);

/* Diagnostic: launches one kernel that waits, with the bounded wait every
 * tensor-core kernel uses, on an mbarrier phase nothing completes; after the
 * 2 s limit it records TT_ERR_DEVICE_TIMEOUT in *status (device memory) and
 * exits.  Faults nothing; the context stays usable.  For testing the failure
 * path only. */
int tt_diag_bounded_wait(int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Host packer.  Replaces the position/boundary/parent/leaf part of
 * build_dfs_tree_info (dfs_tree_forward.py:91-139) and, instead of the dense
 * [N,N] mask it builds (dfs_tree_forward.py:141-172), writes the per-key
 * visible-row intervals.  The forest comes in pre-order: node i has
 * node_len[i] tokens and parent node_parent[i] (< i, or -1 for a root).
 * pos_ids[t] = pos_offset + (tokens in t's ancestor nodes) + offset in node
 * (dfs_tree_forward.py:125-126; pos_offset is tree_grad_hybrid.py:308-310).
 * Outputs: pos_ids[N], chunk_bounds[2*n_nodes] (start,end pairs),
 * subtree_end[n_nodes] (token one past the node's subtree), leaf_ids (nodes
 * without children, DFS order; *n_leaves set), token_node[N], kv_lo[N],
 * kv_hi[N] (row intervals of the partition's own keys).  Any output pointer
 * may be NULL.  Host memory.  Returns TT_ERR_INVALID_ARG if the order is
 * not a pre-order.
 */
int tt_pack_forest(int32_t n_nodes, const int32_t* node_len, const int32_t* node_parent,
                   int32_t pos_offset, int32_t* pos_ids, int32_t* chunk_bounds,
                   int32_t* subtree_end, int32_t* leaf_ids, int32_t* n_leaves,
                   int32_t* token_node, int32_t* kv_lo, int32_t* kv_hi);

/* Gateway key intervals from the reference's additive bias vector
 * (tree_grad_hybrid.py:206-209, consumed at :313-315): bias 0 -> visible to
 * every row [0, n_q), -inf -> no row.  Host memory.  Any other value ->
 * TT_ERR_NOT_INTERVAL. */
int tt_gateway_intervals_from_bias(int32_t past_len, const float* bias, int32_t n_q,
                                   int32_t* kv_lo, int32_t* kv_hi);

/* ------------------------------------------------------------------------
 * Tile work lists (host).  For q-tiles of tile_q rows and kv-tiles of
 * tile_kv columns: fwd_ptr[n_qt+1]/fwd_list = per q-tile the visible
 * kv-tiles (ascending), bwd_ptr[n_kt+1]/bwd_list = per kv-tile the visible
 * q-tiles (ascending).  Entry = tile_index*2 + partial, where partial=0 means
 * every (row, key) of the pair is visible (the kernel skips the mask test).
 * Lists need capacity n_qt*n_kt entries (list_cap); *visible_pairs = number
 * of visible (row, key) pairs.  Any of the four list pointers may be NULL.
 */
int tt_build_tiles(int32_t n_q, int32_t n_kv, const int32_t* kv_lo, const int32_t* kv_hi,
                   int32_t tile_q, int32_t tile_kv, int32_t* fwd_ptr, int32_t* fwd_list,
                   int32_t* bwd_ptr, int32_t* bwd_list, int64_t list_cap,
                   int64_t* visible_pairs);

/* Tile shape that tt_tree_attn_fwd / _bwd expect for a dtype and head dim
 * (lists must be built with it).  kind: 0 = forward, 1 = backward. */
int tt_attn_tile_shape(int dtype, int32_t head_dim, int kind, int32_t* tile_q,
                       int32_t* tile_kv);

/* ------------------------------------------------------------------------
 * Dense mask -> key intervals (device).  Lets the reference's own drivers
 * pass their dense mask unchanged (dfs_tree_forward.py:548-550,
 * tree_grad_hybrid.py:312-317): visible = (value == 0) for float masks, or
 * nonzero for TT_U8 (bool) masks; masked = -inf / a value below -1e30.
 * A column whose visible rows are not one run, or any other value, sets
 * *status = TT_ERR_NOT_INTERVAL.  mask[i*stride_q + j*stride_kv].
 */
int tt_mask_to_intervals(int mask_dtype, int32_t n_q, int32_t n_kv, const void* mask,
                         int64_t stride_q, int64_t stride_kv, int32_t* kv_lo, int32_t* kv_hi,
                         int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Tree attention forward.  Replaces the attention call that the reference
 * reaches through HF (TF/integrations/sdpa_attention.py:92-101 with the mask
 * of dfs_tree_forward.py:548-550 / tree_grad_hybrid.py:313-317): for every
 * q head h, O = softmax(Q K^T * scale + M) V with M from the key intervals,
 * GQA by h / (hq / hkv).  out [n_q, hq, head_dim] contiguous, in `dtype`;
 * lse [hq, ld] fp32 natural-log row log-sum-exp with ld = n_q rounded up to a
 * multiple of 128 (+inf for a row that sees no key and for the ld - n_q
 * padding rows).  dtype TT_BF16 / TT_F16 run the tcgen05 path for head_dim 128 (and
 * the exact SIMT path otherwise); TT_F32 runs the SIMT path (fp32 FMA).  On the
 * tcgen05 path kv_lo/kv_hi must be 16-byte aligned and readable up to
 * round_up(n_kv, 128) entries with zeros past n_kv.
 */
int tt_tree_attn_fwd(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                     int32_t head_dim, const void* q, int64_t q_st, int64_t q_sh,
                     const void* k, int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
                     int64_t v_sh, const int32_t* kv_lo, const int32_t* kv_hi,
                     const int32_t* fwd_ptr, const int32_t* fwd_list, float scale, void* out,
                     float* lse, int32_t* status, void* stream);

/* Workspace bytes for tt_tree_attn_bwd: the fp32 row terms (delta), then one
 * int32 per 128-key tile, in which the tcgen05 path orders the dK/dV tiles by
 * work, longest first (less tail on the GPU).  A workspace holding only the
 * row terms (hq * round_up(n_q, 128) floats, rounded up to 256 bytes) is also
 * accepted; the tiles then run in key order.  Results are the same either way. */
int64_t tt_tree_attn_bwd_workspace_size(int dtype, int32_t n_q, int32_t n_kv, int32_t hq,
                                        int32_t hkv, int32_t head_dim);

/* Tree attention backward: the autograd of the call above (what torch
 * autograd computes through SDPA in the reference's loss.backward(),
 * tree_grad_hybrid.py:533-535, tree_grad_ckpt.py:103-107).  out/dout are
 * [n_q, hq, head_dim] (token/head strides given for dout); dq, dk, dv are
 * written with the given strides (dk/dv include the gateway keys, so the
 * gateway leaf tensors get gradients as with SDPA).  Deterministic for
 * dk/dv.  fwd lists drive the dQ pass, bwd lists the dK/dV pass.  On the
 * tcgen05 path kv_lo/kv_hi must be readable up to round_up(n_kv, 128) entries
 * with zeros past n_kv (whole 128-key tiles are bulk-copied), and lse, the
 * workspace and all outputs must be 16-byte aligned. */
int tt_tree_attn_bwd(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                     int32_t head_dim, const void* q, int64_t q_st, int64_t q_sh,
                     const void* k, int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
                     int64_t v_sh, const void* out, const void* dout, int64_t do_st,
                     int64_t do_sh, const float* lse, const int32_t* kv_lo,
                     const int32_t* kv_hi, const int32_t* fwd_ptr, const int32_t* fwd_list,
                     const int32_t* bwd_ptr, const int32_t* bwd_list, float scale, void* dq,
                     int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh,
                     void* dv, int64_t dv_st, int64_t dv_sh, void* workspace,
                     int64_t workspace_bytes, int phases, int32_t* status, void* stream);

/* `phases` of tt_tree_attn_bwd (bitmask; TT_BWD_ALL runs the whole backward).
 * PREP computes the fp32 row terms delta = rowsum(dO * O) into the workspace;
 * DKDV and DQ read them and are independent of each other, so a caller may
 * run them on two streams after PREP. */
enum tt_bwd_phase { TT_BWD_PREP = 1, TT_BWD_DKDV = 2, TT_BWD_DQ = 4, TT_BWD_ALL = 7 };

/* Workspace bytes for tt_tree_attn_bwd_stored: tt_tree_attn_bwd's workspace,
 * one int32 per tile-list entry, and one 32 KB dS slot per (q head of a pass,
 * tile-list entry), where a pass covers kv_heads_per_pass kv heads and their
 * hq/hkv q heads each.  n_tile_pairs: at least the number of (q tile, kv tile)
 * entries of the fwd lists (fwd_ptr[n_q tiles]).  Off the tcgen05 path (fp32,
 * head_dim != 128) this is tt_tree_attn_bwd_workspace_size; -1 for an invalid
 * n_tile_pairs / kv_heads_per_pass. */
int64_t tt_tree_attn_bwd_stored_workspace_size(int dtype, int32_t n_q, int32_t n_kv, int32_t hq,
                                               int32_t hkv, int32_t head_dim,
                                               int64_t n_tile_pairs, int32_t kv_heads_per_pass);

/* The same gradients as tt_tree_attn_bwd (all phases), scheduled without
 * recomputing S and dP for dQ: the dK/dV kernel stores every 16-bit dS tile it
 * forms into the workspace, and a second kernel sums dQ = scale * dS K over
 * each q tile's kv list from those tiles.  Both sums run in a fixed order, so
 * results are deterministic (dK/dV bit-identical to tt_tree_attn_bwd's).  The
 * kv heads are processed kv_heads_per_pass at a time, which bounds the dS
 * slots the workspace needs (tt_tree_attn_bwd_stored_workspace_size).  Off the
 * tcgen05 path it runs tt_tree_attn_bwd.  phases: TT_BWD_ALL, or, when
 * kv_heads_per_pass == hkv (one pass), PREP, DKDV and DQ as separate calls in
 * that order with the same workspace (DQ reads the dS tiles DKDV stored, so
 * unlike tt_tree_attn_bwd's the two are not independent).  Replaces the same
 * autograd of the reference's SDPA call as tt_tree_attn_bwd
 * (tree_grad_hybrid.py:533-535). */
int tt_tree_attn_bwd_stored(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                            int32_t head_dim, const void* q, int64_t q_st, int64_t q_sh,
                            const void* k, int64_t k_st, int64_t k_sh, const void* v,
                            int64_t v_st, int64_t v_sh, const void* out, const void* dout,
                            int64_t do_st, int64_t do_sh, const float* lse,
                            const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                            const int32_t* fwd_list, const int32_t* bwd_ptr,
                            const int32_t* bwd_list, float scale, void* dq, int64_t dq_st,
                            int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
                            int64_t dv_st, int64_t dv_sh, int64_t n_tile_pairs,
                            int32_t kv_heads_per_pass, void* workspace, int64_t workspace_bytes,
                            int phases, int32_t* status, void* stream);

/* Allocation-free variant of tt_tree_attn_bwd (same arguments without the
 * workspace and phases; no counterpart in the reference).  For callers that
 * cannot pass a scratch buffer and must not have the library call cudaMalloc
 * (a binding that mirrors the reference's inputs-and-outputs call, or a
 * runtime whose device memory belongs to its own pooling allocator).  Its
 * workspace (row terms and dK/dV tile order, as tt_tree_attn_bwd_workspace_size
 * sizes it) lives in a fixed 8 MiB + 64 KiB array inside the library's device
 * image, held by every GPU that loads the library until exit, so it runs the
 * same kernels in the same tile order and gives bit-identical results.
 * Problems with hq * round_up(n_q, 128) > tt_tree_attn_bwd_noalloc_max_row_terms()
 * or n_kv > 2,097,152 keys are rejected with TT_ERR_WORKSPACE before anything
 * runs.  The first call on a device looks the array up and caches its address
 * for the process (make it before any stream capture; the device of the
 * pointers must be current; not supported after a cudaDeviceReset); every
 * call shares the array, so calls whose kernels overlap on the GPU race.
 * Calls no allocating routine. */
int tt_tree_attn_bwd_noalloc(int dtype, int32_t n_q, int32_t n_kv, int32_t hq, int32_t hkv,
                             int32_t head_dim, const void* q, int64_t q_st, int64_t q_sh,
                             const void* k, int64_t k_st, int64_t k_sh, const void* v,
                             int64_t v_st, int64_t v_sh, const void* out, const void* dout,
                             int64_t do_st, int64_t do_sh, const float* lse,
                             const int32_t* kv_lo, const int32_t* kv_hi, const int32_t* fwd_ptr,
                             const int32_t* fwd_list, const int32_t* bwd_ptr,
                             const int32_t* bwd_list, float scale, void* dq, int64_t dq_st,
                             int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh, void* dv,
                             int64_t dv_st, int64_t dv_sh, int32_t* status, void* stream);

/* Largest hq * round_up(n_q, 128) that tt_tree_attn_bwd_noalloc accepts. */
int64_t tt_tree_attn_bwd_noalloc_max_row_terms(void);

/* ------------------------------------------------------------------------
 * Tree gated delta rule (GDN).  Replaces torch_chunk_gated_delta_rule_tree_varlen
 * (tree_dfs_ssm.py:38-156; same algorithm at dfs_tree_forward.py:253-353 and
 * tree_grad_hybrid_ssm.py:48-135): one chunk per tree node, each node starting
 * from the state after its PARENT node (tree_dfs_ssm.py:131-132), intra-node
 * correction T = I + A + A^2 (the reference's row loop, :119-126), fp32
 * internally.  Batch 1.  q, k: [S, Hk, Dk] with H % Hk == 0 (v-head h uses
 * k-head h / (H/Hk)); v: [S, H, Dv]; all contiguous in `dtype`; g, beta: fp32
 * [S, H].  bounds/parents: HOST int32 arrays (node i = tokens
 * [bounds[2i], bounds[2i+1]), parent < i or -1, pre-order).  initial_state:
 * fp32 [H, Dk, Dv] or NULL (zeros).  out: [S, H, Dv] in `dtype`; last_state:
 * fp32 [H, Dk, Dv] = state after the LAST DFS node (tree_dfs_ssm.py:155), or
 * NULL.  flags: TT_GDN_QK_L2NORM = x * rsqrt(sum x^2 + 1e-6) on q and k first
 * (the reference's use_qk_l2norm_in_kernel, :67-69); TT_GDN_EXACT_INVERSE =
 * replace the reference's truncated correction by the delta rule's exact
 * T = (I - A)^-1 per node (the token-by-token recurrence's result, which the
 * reference approximates); TT_GDN_SAVED_FORWARD (backward only) = the
 * workspace still holds what tt_gdn_tree_fwd computed: the backward then skips
 * recomputing the forward.  For that, call tt_gdn_tree_fwd with a workspace
 * sized by tt_gdn_tree_workspace_size(..., backward=1), leave it untouched, and
 * call tt_gdn_tree_bwd with the same workspace, inputs and other flags.  Any
 * other bit is TT_ERR_INVALID_ARG.
 * Dk, Dv <= 256.  Workspace: tt_gdn_tree_workspace_size(..., backward=0/1),
 * the same for either flag.
 */
#define TT_GDN_QK_L2NORM 1
#define TT_GDN_EXACT_INVERSE 2
#define TT_GDN_SAVED_FORWARD 4

int64_t tt_gdn_tree_workspace_size(int32_t S, int32_t H, int32_t Dk, int32_t Dv,
                                   int32_t n_nodes, const int32_t* bounds, int backward);

int tt_gdn_tree_fwd(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                    const void* q, const void* k, const void* v, const float* g,
                    const float* beta, int32_t n_nodes, const int32_t* bounds,
                    const int32_t* parents, const float* initial_state, int flags,
                    void* out, float* last_state, void* workspace, int64_t workspace_bytes,
                    void* stream);

/* Gradients of tt_gdn_tree_fwd (what torch autograd computes through the
 * reference's Python loop): dout [S, H, Dv] (`dtype`), dlast fp32 [H, Dk, Dv]
 * or NULL -> dq, dk (`dtype`, k-head layout, summed over each GQA group), dv
 * (`dtype`), dg, dbeta (fp32 [S, H]), dinit fp32 [H, Dk, Dv] (or NULL).  The
 * forward is recomputed inside (nothing is kept between the two calls). */
int tt_gdn_tree_bwd(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                    const void* q, const void* k, const void* v, const float* g,
                    const float* beta, int32_t n_nodes, const int32_t* bounds,
                    const int32_t* parents, const float* initial_state, int flags,
                    const void* dout, const float* dlast, void* dq, void* dk, void* dv,
                    float* dg, float* dbeta, float* dinit, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* Forward and backward of the tree GDN that also hand out the states after a
 * chosen set of nodes, the recurrent half of the reference's SSM gateway
 * (_ssm_varlen_capture, tree_grad_hybrid_ssm.py:48-135: captured[i] = the
 * state after node capture_nodes[i]).  capture_nodes: HOST int32 [n_capture],
 * distinct node indices; captured: fp32 [n_capture, H, Dk, Dv].  The
 * backward takes their gradients, dcaptured fp32 [n_capture, H, Dk, Dv] (or
 * NULL), and adds each to the gradient of the node's output state.  With
 * n_capture = 0 these are tt_gdn_tree_fwd / tt_gdn_tree_bwd.
 * q_token_stride, k_token_stride, v_token_stride: elements from one token's
 * q / k / v row to the next (each row still [heads, dim] contiguous), 0 for
 * packed rows; a nonzero stride below the packed row (Hk * Dk, Hk * Dk,
 * H * Dv) is TT_ERR_INVALID_ARG.  This reads q, k and v in place as the
 * columns of one token-major [S, 2 Hk Dk + H Dv] buffer, the split the
 * reference's layer makes of the conv output (dfs_tree_forward.py:403-410).
 * dq, dk, dv stay packed. */
int tt_gdn_tree_fwd_ex(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                       const void* q, const void* k, const void* v, const float* g,
                       const float* beta, int32_t n_nodes, const int32_t* bounds,
                       const int32_t* parents, const float* initial_state, int flags,
                       void* out, float* last_state, int32_t n_capture,
                       const int32_t* capture_nodes, float* captured, int64_t q_token_stride,
                       int64_t k_token_stride, int64_t v_token_stride, void* workspace,
                       int64_t workspace_bytes, void* stream);

int tt_gdn_tree_bwd_ex(int dtype, int32_t S, int32_t Hk, int32_t H, int32_t Dk, int32_t Dv,
                       const void* q, const void* k, const void* v, const float* g,
                       const float* beta, int32_t n_nodes, const int32_t* bounds,
                       const int32_t* parents, const float* initial_state, int flags,
                       const void* dout, const float* dlast, int32_t n_capture,
                       const int32_t* capture_nodes, const float* dcaptured, void* dq, void* dk,
                       void* dv, float* dg, float* dbeta, float* dinit, int64_t q_token_stride,
                       int64_t k_token_stride, int64_t v_token_stride, void* workspace,
                       int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Leaf-token cross-entropy fused with its gradient (the per-leaf
 * F.cross_entropy of make_tree_loss_fn, tree_grad_hybrid.py:546-558, and its
 * autograd, for a chunk of LM-head logits).  logits: [n_rows, ld] in `dtype`
 * (first `vocab` columns used); with write_grad != 0 overwritten with
 * weights[r] * (softmax(row) - onehot(labels[r])), else left alone; labels:
 * device int64 [n_rows] (ignore_index, negative or >= vocab: zero loss and
 * gradient); weights: device fp32 [n_rows]; loss: device fp32 [n_rows] =
 * weights[r] * (logsumexp(row) - row[label]).
 */
int tt_ce_fwd_grad(int dtype, int32_t n_rows, int32_t vocab, void* logits, int64_t ld,
                   const int64_t* labels, const float* weights, int64_t ignore_index,
                   float* loss, int write_grad, void* stream);

/* ------------------------------------------------------------------------
 * Fused attention prologue: per-head RMSNorm of q or k (weight [D] fp32, eps)
 * then the rotary embedding with the tokens' cos / sin rows (the tree's
 * depth-based positions), replacing q_norm / k_norm + apply_rotary_pos_emb of
 * transformers' Qwen3 attention (models/qwen3/modeling_qwen3.py:263-268).
 * x, y, dy, dx: [n_tok, H, D] contiguous in `dtype`; cos, sin: [n_tok, D] in
 * `dtype`; D in {64, 128, 256}.  The backward recomputes the norm from x and
 * writes per-block weight-gradient partials dw_part [blocks, D] fp32 (sum the
 * rows for dw); blocks from tt_qk_norm_rope_bwd_blocks(n_tok * H).
 */
int tt_qk_norm_rope_fwd(int dtype, int64_t n_tok, int32_t H, int32_t D, const void* x,
                        const float* weight, const void* cos_, const void* sin_, float eps,
                        void* y, void* stream);
int tt_qk_norm_rope_bwd_blocks(int64_t rows);
int tt_qk_norm_rope_bwd(int dtype, int64_t n_tok, int32_t H, int32_t D, const void* x,
                        const float* weight, const void* cos_, const void* sin_, float eps,
                        const void* dy, void* dx, float* dw_part, int32_t blocks, void* stream);

/* ------------------------------------------------------------------------
 * Fused gated RMSNorm of the GDN output: y = x * rsqrt(mean(x^2) + eps) * w *
 * silu(z) over rows of D values, replacing the layer's gated norm on the tree
 * GDN output (dfs_tree_forward.py:420-433; transformers models/qwen3_5_moe/
 * modeling_qwen3_5_moe.py Qwen3_5MoeRMSNormGated).  x, z, y, dy, dx, dz:
 * [rows, D] contiguous in `dtype`; weight [D] fp32; D in {32, 64, 128, 256}.
 * The backward recomputes the norm and writes per-block weight-gradient partials
 * dw_part [blocks, D] fp32 (sum the rows for dw); blocks from
 * tt_gated_rmsnorm_bwd_blocks(rows).
 */
int tt_gated_rmsnorm_fwd(int dtype, int64_t rows, int32_t D, const void* x, const void* z,
                         const float* weight, float eps, void* y, void* stream);
int tt_gated_rmsnorm_bwd_blocks(int64_t rows);
int tt_gated_rmsnorm_bwd(int dtype, int64_t rows, int32_t D, const void* x, const void* z,
                         const float* weight, float eps, const void* dy, void* dx, void* dz,
                         float* dw_part, int32_t blocks, void* stream);

/* ------------------------------------------------------------------------
 * Tree-correct depthwise causal conv + SiLU.  Replaces _tree_correct_conv_varlen
 * (tree_dfs_ssm.py:285-348; dfs_tree_forward.py:191-246): each token's window
 * is the K-1 tokens before it on its root-to-node path (the reference's saved
 * parent context), zero padded at roots.  x, out: [C, S] (channels x tokens,
 * token-contiguous, `dtype`); weight fp32 [C, K]; bias fp32 [C] or NULL.
 * pred: device int32 [S, K-1], pred[t, m-1] = the token m steps before t on
 * its path or -1 (tt_conv_predecessors builds it on the host).  K <= 8.
 */
int tt_conv_predecessors(int32_t n_nodes, const int32_t* bounds, const int32_t* parents,
                         int32_t K, int32_t* pred);

int tt_tree_conv_fwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                     const float* weight, const float* bias, const int32_t* pred, void* out,
                     void* stream);

/* dout [C, S] -> dx [C, S] (`dtype`), dweight fp32 [C, K], dbias fp32 [C] (or
 * NULL).  Deterministic: the SiLU-gradient term is computed once per (channel,
 * token) into `workspace` (at least tt_tree_conv_bwd_workspace_size bytes,
 * else TT_ERR_WORKSPACE), dx gathers it over each token's successors (succ
 * CSR from tt_conv_successors), dweight/dbias sum per-block partials in a
 * fixed order (no atomics). */
int tt_conv_successors(int32_t S, int32_t K, const int32_t* pred, int32_t* succ_ptr,
                       int32_t* succ_tok, int32_t* succ_lag, int64_t cap);

int64_t tt_tree_conv_bwd_workspace_size(int32_t C, int32_t S, int32_t K);

int tt_tree_conv_bwd(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                     const float* weight, const float* bias, const int32_t* pred,
                     const int32_t* succ_ptr, const int32_t* succ_tok, const int32_t* succ_lag,
                     const void* dout, void* dx, float* dweight, float* dbias,
                     void* workspace, int64_t workspace_bytes, void* stream);

/* The conv with its output (forward) or output gradient (backward) in
 * token-major memory, [S, C] with channel rows contiguous: the layout the
 * reference's layer reads after transposing the conv output and splitting it
 * into q / k / v (dfs_tree_forward.py:403-410), so those views need no
 * transposing copy.  x and dx stay [C, S].  With out_token_major /
 * dout_token_major = 0 these are tt_tree_conv_fwd / tt_tree_conv_bwd.  The
 * token-major forms need S % 4 == 0, C % 8 == 0 and 16-byte aligned x, out,
 * dout, dx and workspace (else TT_ERR_UNSUPPORTED). */
int tt_tree_conv_fwd_ex(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                        const float* weight, const float* bias, const int32_t* pred, void* out,
                        int32_t out_token_major, void* stream);

int tt_tree_conv_bwd_ex(int dtype, int32_t C, int32_t S, int32_t K, const void* x,
                        const float* weight, const float* bias, const int32_t* pred,
                        const int32_t* succ_ptr, const int32_t* succ_tok,
                        const int32_t* succ_lag, const void* dout, int32_t dout_token_major,
                        void* dx, float* dweight, float* dbias, void* workspace,
                        int64_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TREE_TRAINING_B200_H */
