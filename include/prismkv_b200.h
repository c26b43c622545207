/*
 * prismkv_b200.h -- C ABI of the B200 (sm_100a) PrismKV retrieval library.
 *
 * Conventions (the same as the reference's native bindings,
 * src/prismkv/native8b.py:46-80 and kernels/cuda_sm90/native.py:16-35):
 *   - every device buffer is passed as a uint64_t address owned by the caller;
 *   - every call is asynchronous on the caller's CUDA stream (last argument)
 *     and performs no host synchronisation and no allocation;
 *   - the return value is 0 on success, a negative PK_ERR_* for an argument
 *     error detected on the host, or a positive cudaError_t from the launch;
 *   - conditions only the device can detect (a full bucket region, a full
 *     boundary buffer, a history too long for the union's on-chip bitmap) are
 *     OR-ed into a caller-provided int32 status word (PK_STATUS_*), which the
 *     caller reads after synchronising.  Nothing is silently truncated.
 *
 * Index layout (one "unit" = one (batch row, KV head) of one layer):
 *   offsets[U, F+1] int32  start of each bucket's region in ids; region f has
 *                          capacity offsets[f+1] - offsets[f]
 *   lens[U, F]      int32  bucket sizes (the reference's FeatureIndex.counts)
 *   ids[U, ids_stride] int32 token ids, ascending within each bucket
 *   center[U, d], mean/var[U, F, d] fp32 (moments are optional)
 * This is the CSR interchange of native8b.py:66-69 with per-bucket slack so
 * that append_index can extend buckets in place.
 *
 * Workspace buffers must be zero-filled before their first use; the kernels
 * leave their counters zeroed again when they finish.  Counter positions
 * depend on the call's shape, so a workspace reused for a different shape
 * must be zero-filled again.  Calls that share a workspace must not overlap
 * on the GPU.
 */
#ifndef PRISMKV_B200_H
#define PRISMKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host-side return codes. */
#define PK_OK 0
#define PK_ERR_ARG (-1)          /* an argument is out of range               */
#define PK_ERR_UNSUPPORTED (-2)  /* shape/dtype not compiled into this build  */
#define PK_ERR_WORKSPACE (-3)    /* workspace smaller than *_workspace_bytes  */

/* Device status bits (OR-ed into the caller's int32 status word). */
#define PK_STATUS_BUCKET_FULL 1       /* append: a bucket region is full        */
#define PK_STATUS_BOUNDARY_FULL 2     /* build: boundary buffer too small       */
#define PK_STATUS_MEMBERS_FULL 4      /* build: member buffer too small         */
#define PK_STATUS_BUCKET_TOO_BIG 8    /* build: a bucket exceeds the sort limit */
#define PK_STATUS_OUT_FULL 16         /* union: output row too short            */
#define PK_STATUS_HISTORY_TOO_LONG 32 /* union: history above max_history       */
#define PK_STATUS_NEEDS_EXACT 64      /* build: bounds undecided, rerun exactly  */
#define PK_STATUS_EXCHANGE_TIMEOUT 128 /* p2p all-gather: a peer never published */

/* Element types. */
#define PK_F32 0
#define PK_BF16 1

/* Router terms for pk_route_moments (core.py:117-126). */
#define PK_TERM_COUNT 1
#define PK_TERM_MEAN 2
#define PK_TERM_VARIANCE 4

/* Library build facts: target sm version * 100 + ABI revision; head dims.
 * Every kernel is compiled for head_dim d = 128 (the reference's 8B
 * configuration); any other d returns PK_ERR_UNSUPPORTED.  The reference's
 * d = 256 configuration (its SM90 27B kernels) is not served. */
int pk_version(void);
int pk_supported_head_dim(int d);

/* ------------------------------------------------------------------------
 * q_activation routing (a1 + a2).
 * Replaces the score stage of the native operators -- pack + torch.bmm +
 * fused_norm_top (src/prismkv/native8b.py:82-87, kernels/ppu_8b/pack.cu:3-4,
 * kernels/ppu_8b/route_parallel.cu:13-35; kernels/cuda_sm90/native.py:158-167)
 * -- for the reference's q_activation router, src/prismkv/core.py:131-139.
 *
 * q[U, G, d] (PK_F32 or PK_BF16).  The heads of the listed units (units[n],
 * int32, or 0 for all U) are encoded with one SAE: w_enc[F, d], b_enc[F] fp32.
 * counts[U, F] int32 marks live buckets.  Outputs per listed unit u:
 *   order[u, 0..n_order[u])  candidate buckets, descending score, ties by id
 *   score[u, F]   (optional, 0 to skip) the reference's full score vector
 *   topk[u, G, k] (optional) each head's picks in rank order
 * With w_bf16[F, d] and w_norm[F] from pk_sae_prepare (both non-zero, topk
 * not requested) the activations are first approximated on the tensor cores
 * and only features whose error-bounded value can reach the top-k are
 * recomputed exactly -- the same results, far fewer fp32 operations.
 * ------------------------------------------------------------------------ */
/* Per-SAE preparation for the fast routing path: bf16 copy of W_enc and an
 * upper bound of each row's L2 norm. */
int pk_sae_prepare(uint64_t w_enc, int F, int d, uint64_t w_bf16, uint64_t w_norm, uint64_t stream);
size_t pk_route_qact_workspace_bytes(int U, int G, int F, int k);
int pk_route_qact(uint64_t q, int q_dtype, uint64_t units, int n_units,
                  uint64_t w_enc, uint64_t b_enc, uint64_t w_bf16, uint64_t w_norm,
                  float query_scale, uint64_t counts,
                  int U, int G, int d, int F, int k,
                  uint64_t workspace, uint64_t workspace_bytes,
                  uint64_t order, uint64_t n_order, int order_stride,
                  uint64_t score, uint64_t topk, uint64_t stream);

/* Feature-sharded q_activation routing: the same order as pk_route_qact
 * (core.py:131-139) with the encode split over P ranks by feature range.
 * pk_route_qact_shard encodes features [f_lo, f_hi) of every head (the
 * bound-filtered path: w_bf16 and w_norm required) and writes each head's
 * exact positive top-k among them, in rank order, to picks[U*G, k] as int32
 * (value bits, feature id) pairs; unused slots hold (0, INT32_MAX).
 * pk_route_qact_merge takes picks[P, U*G, k] of P disjoint ranges covering
 * all F features (after an all-gather), ranks each head's entries
 * exactly (value desc, feature asc) and finishes the route as
 * pk_route_qact: order[u, 0..n_order[u]), counts[U, F] marking live
 * buckets, score[U, F] optional.  No counterpart in the reference, whose
 * route runs on one device (src/prismkv/core.py:131-139). */
size_t pk_route_qact_shard_workspace_bytes(int U, int G, int F_local, int k);
int pk_route_qact_shard(uint64_t q, int q_dtype, uint64_t w_enc, uint64_t b_enc, uint64_t w_bf16, uint64_t w_norm,
                        float query_scale, int U, int G, int d, int F, int k, int f_lo, int f_hi,
                        uint64_t workspace, uint64_t workspace_bytes, uint64_t picks, uint64_t stream);
size_t pk_route_qact_merge_workspace_bytes(int U, int G, int k);
int pk_route_qact_merge(uint64_t picks, int P, uint64_t counts, int U, int G, int F, int k,
                        uint64_t workspace, uint64_t workspace_bytes, uint64_t order, uint64_t n_order,
                        int order_stride, uint64_t score, uint64_t stream);

/* ------------------------------------------------------------------------
 * moments routing (a9).
 * Replaces pack + torch.bmm + fused_norm_top / HopperTop16
 * (native8b.py:82-87; cuda_sm90/native.py:158-167; hopper_top16.cu:64-184)
 * for src/prismkv/core.py:117-130.  mean/var[U, F, d] fp32, counts[U, F].
 * score[U, F] fp32 is written (required).  order[u, 0..n_order[u]) holds
 * the first k live buckets by descending score, ties by id.
 * ------------------------------------------------------------------------ */
size_t pk_route_moments_workspace_bytes(int U, int G, int F);
int pk_route_moments(uint64_t q, int q_dtype, uint64_t mean, uint64_t var, uint64_t counts, int terms,
                     int U, int G, int d, int F, int k,
                     uint64_t workspace, uint64_t workspace_bytes,
                     uint64_t score, uint64_t order, uint64_t n_order, int order_stride, uint64_t stream);

/* ------------------------------------------------------------------------
 * Budgeted bucket union (a3; a10 when limit >= history).
 * Replaces launch_union_warp (kernels/ppu_8b/union.cu:39-49,
 * kernels/cuda_sm90/native_sources/union.cu:52-62), extended from the
 * unbudgeted OR of bitmaps to the greedy skip-overflow rule of
 * src/prismkv/core.py:152-164.  For each unit u, buckets order[u, 0..n_order[u])
 * are taken in turn; a bucket whose new (not yet chosen) tokens would push
 * the chosen count past limit[u] (int64) is skipped.  Outputs:
 * out_ids[u, 0..count[u]) ascending unique token ids, features[u, ..n_features[u])
 * accepted buckets in acceptance order, raw[u] (int64) summed sizes of the
 * accepted buckets.  history[u] (int32) bounds the token ids; the on-chip
 * bitmap is sized for max_history.
 * ------------------------------------------------------------------------ */
int pk_union(uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride,
             uint64_t order, uint64_t n_order, int order_stride,
             uint64_t history, uint64_t limit, int U, int F, int max_history,
             uint64_t out_ids, int64_t out_stride, uint64_t out_count,
             uint64_t features, uint64_t n_features, uint64_t raw,
             uint64_t status, uint64_t stream);


/* ------------------------------------------------------------------------
 * Sparse attention over selected rows plus the dense tail (a4 + a11).
 * Replaces attention_tuned (kernels/ppu_8b/av_tuned.cu:62-67), batch_av
 * (kernels/cuda_sm90/native_sources/av.cu:92-103) and HopperAV
 * (kernels/cuda_sm90/hopper_av.py:6-103); semantics of core.py:170-183.
 * Unit u = (b, h) with h = u % kv_heads reads K/V rows at
 *   base(u) = (u / kv_heads) * kv_batch_stride + (u % kv_heads) * kv_head_stride
 *   row(p)  = base(u) + p * kv_row_stride       (elements)
 * which covers both [U, total, d] and slot-major [slot, cap, H_kv, d].
 * Rows attended: ids[u, 0..count[u]) then history[u]..length[u]-1.
 * ids holds U rows of ids_stride int32 each; the kernel may read any
 * element of a row (entries past count[u] are read ahead and ignored).
 * length[u] == 0 marks an inactive unit (output zeros).  q, k, v and out
 * share `dtype`.  splits <= 0 picks a split count for the machine: about
 * two CTAs per SM over all units, whole clusters of 8 above 8 splits, at
 * most 64.
 * With partial != 0 the kernel writes per-(u, head) partials
 * (m, l, o[d]) fp32 to partial[U*G, d+2] instead of out (for pk_lse_merge).
 * ------------------------------------------------------------------------ */
size_t pk_sparse_av_workspace_bytes(int U, int G, int d, int splits);
int pk_sparse_av(uint64_t q, uint64_t k, uint64_t v, int dtype,
                 int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                 uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history, uint64_t length,
                 int U, int G, int d, int splits,
                 uint64_t workspace, uint64_t workspace_bytes,
                 uint64_t out, uint64_t partial, uint64_t stream);

/* pk_sparse_av fused with the decode KV append: unit u's new rows
 * k_new/v_new[u, d] (contiguous, dtype, 16-byte aligned; u = slot * kv_heads
 * + head) take the place of row length[u] - 1 -- the newest tail row, when
 * length[u] > history[u] -- in the attention, and are written into K and V
 * at that row.  One launch instead of batch_append followed by the attention
 * (kernels/cuda_sm90/model.py:109-137); the same fusion as
 * flash_attn_with_kvcache's k/v arguments.  No counterpart entry point in
 * the reference. */
int pk_sparse_av_append(uint64_t q, uint64_t k, uint64_t v, int dtype,
                        int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                        uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history, uint64_t length,
                        int U, int G, int d, int splits,
                        uint64_t workspace, uint64_t workspace_bytes,
                        uint64_t out, uint64_t partial, uint64_t k_new, uint64_t v_new, uint64_t stream);

/* All-gather of a small device buffer between the P <= 8 ranks of one node
 * over NVLink peer memory (no counterpart in the reference, which runs on
 * one device; the exchange step of the sequence-sharded decode).  Each rank
 * allocates an exchange region of pk_p2p_region_bytes(P, bytes) with
 * pk_p2p_alloc (zeroed device memory), exports it with pk_p2p_handle (a
 * 64-byte CUDA IPC handle), and opens every peer's with pk_p2p_open.
 * pk_p2p_allgather then copies src[bytes] (16-byte multiple) of every rank
 * into out[P, bytes] on every rank: peer_bases is a host array of the P
 * regions' addresses as mapped here (its rank-th entry local_base).  Every
 * rank must issue the same sequence of calls on its region.  A peer that
 * does not publish within max_spins polls (~64 ns each) sets
 * PK_STATUS_EXCHANGE_TIMEOUT in *status and the call completes. */
size_t pk_p2p_region_bytes(int P, int64_t bytes);
int pk_p2p_alloc(uint64_t bytes, uint64_t ptr_out);
int pk_p2p_free(uint64_t ptr);
int pk_p2p_handle(uint64_t ptr, uint64_t handle_out);
int pk_p2p_open(uint64_t handle, uint64_t ptr_out);
int pk_p2p_close(uint64_t ptr);
int pk_p2p_allgather(uint64_t src, int64_t bytes, int rank, int P, uint64_t peer_bases, uint64_t local_base,
                     uint64_t out, uint64_t status, int64_t max_spins, uint64_t stream);

/* Log-sum-exp merge of P partial states partial[P, UG, d+2] (m, l, o[d]) into
 * out[UG, d] (dtype).  The cross-GPU step of the sequence-sharded decode;
 * generalises the in-GPU split merge of av_tuned.cu:54-61. */
int pk_lse_merge(uint64_t partial, int P, int UG, int d, uint64_t out, int dtype, uint64_t stream);

/* Sequence-sharded build with the exact global BatchTopK (core.py:13-26 over
 * the whole sequence, which the reference computes on one device): rank r of
 * P holds tokens [token_base, token_base + N) of every unit and runs the
 * phases below, the host reducing between them:
 *   phase 0: tensor-core sample of this shard into the sampled histogram
 *            (workspace at layout[0], int32 [U, 8192]); sample_info[0..1] =
 *            (sampled token blocks, feature-tile stride) of this shard.
 *            Host: SUM all-reduce of the histogram.
 *   phase 1: floor from the summed histogram with global_count (N_total *
 *            key_mean) and sample_frac (entries sampled / all entries, over
 *            all shards); bound histograms above it (layout[1], [2]).
 *            Host: SUM all-reduce of both.
 *   phase 2: global cut, members by their bounds, exact values for the
 *            undecided; boundary keys with flat indices in the whole sequence
 *            (flat_base = token_base * F) at layout[5] [U, boundary_capacity],
 *            counts at layout[4], members so far at layout[3].
 *            Host: need[u] = global_count - SUM of members; all-gather of the
 *            keys into all_keys [P, U, key_cap] with counts [P, U].
 *   phase 3: every shard selects the same need[u] smallest keys and keeps
 *            its own, then writes CSR offsets/lens/ids (ids = token_base + t).
 * Any status bit stops the build (the host checks all ranks).  A shard can
 * hold more than its own N * key_mean members under the global threshold:
 * member_capacity (at most min(global_count, N * F)) sizes the member list,
 * and ids_stride must hold the shard's members plus their slack.  Same
 * arguments as pk_build_index otherwise; the fast (tensor-core) path only. */
size_t pk_build_shard_workspace_bytes(int U, int64_t N, int F, int64_t member_capacity, int64_t boundary_capacity);
int pk_build_shard_layout(int U, int64_t N, int F, int64_t member_capacity, int64_t boundary_capacity,
                          uint64_t out_offsets);
int pk_build_shard_phase(int phase, uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, uint64_t center,
                         float key_scale, uint64_t w_enc, uint64_t b_enc, uint64_t w_half, uint64_t w_norm, int U,
                         int64_t N, int d, int F, int key_mean, int64_t member_capacity, int64_t boundary_capacity,
                         uint64_t workspace, uint64_t workspace_bytes, long long global_count, double sample_frac,
                         int64_t flat_base,
                         uint64_t lens, uint64_t offsets, uint64_t ids, int64_t ids_stride, int64_t token_base,
                         float slack_frac, int slack_min, uint64_t all_keys, uint64_t key_counts, int P,
                         int64_t key_cap, uint64_t need, uint64_t sample_info, uint64_t status, uint64_t stream);

/* The key center of a sequence split across shards (the column mean of
 * core.py:99 in torch's cascade order): each shard, holding whole cascade
 * chunks of pk_key_center_chunk_rows(N_total) rows, writes its chunks' sums
 * out[U, N / chunk_rows, d]; the mean is the in-order fp32 sum of every
 * shard's chunk sums divided by N_total (N_total a multiple of the chunk). */
int64_t pk_key_center_chunk_rows(int64_t N_total);
int pk_key_center_chunks(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride, int U, int64_t N, int d,
                         int64_t N_total, uint64_t out, uint64_t stream);

/* Packs each unit's selected rows ids[u, :count[u]] and then its dense tail
 * rows [history[u], length[u]) of K and V (layout as pk_sparse_av) into
 * out_k/out_v [U, packed_rows, d] (unit-major, contiguous); slots past a
 * unit's rows are not written, and a unit with more rows than packed_rows is
 * truncated with PK_STATUS_OUT_FULL in *status (optional).  The layout-
 * control diagnostic of the reference (kernels/cuda_sm90/native_sources/
 * gather.cu:22-31, gather_kv), with its unit-major output.  Rows, strides and
 * base addresses must be 16-byte aligned. */
int pk_gather_kv(uint64_t k, uint64_t v, int dtype, int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride,
                 int64_t kv_row_stride, uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history,
                 uint64_t length, int U, int d, int64_t packed_rows, uint64_t out_k, uint64_t out_v,
                 uint64_t status, uint64_t stream);

/* Decode KV append: slot s's new rows k_new/v_new[s, kv_heads, d]
 * (contiguous, dtype) are written at row positions[s] of the caches, row(p)
 * of head h of slot s at s * kv_batch_stride + h * kv_head_stride +
 * p * kv_row_stride (elements): the slot-major [slot, capacity, H_kv, d]
 * cache of the reference, or [U, capacity, d] with kv_heads = 1.  A position
 * outside [0, capacity) leaves the slot untouched (inactive slot).  Replaces
 * batch_append (kernels/cuda_sm90/native_sources/av.cu:70-90, bound at
 * kernels/cuda_sm90/native.py:23, called by model.py:109-115).  Rows,
 * strides and base addresses must be 16-byte aligned. */
int pk_kv_append(uint64_t k_new, uint64_t v_new, uint64_t k_cache, uint64_t v_cache, int dtype,
                 int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                 uint64_t positions, int slots, int capacity, int d, uint64_t stream);

/* Sparse attention for callers that cannot allocate device memory.
 * This entry point has no counterpart in the reference.  It exists for
 * embedders that cannot hand the library a workspace: a host that reserved
 * all device memory for its own pool up front (where an extra cudaMalloc
 * would fail or fragment it), or a foreign-language caller that binds only
 * this C ABI and has no device allocator of its own.
 * Same arguments and results as pk_sparse_av without the workspace and the
 * partial output; the split scratch lives in a library-owned device array of
 * PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES (4 MiB) that every GPU loading the
 * library holds until exit.  A shape whose scratch
 * (pk_sparse_av_workspace_bytes) exceeds that returns
 * PK_ERR_SCRATCH_LIMIT; pass fewer splits (splits == 1 needs none).
 * Outside a stream capture each call looks the array's device address up
 * with the device current (a device reset moves it); a call inside a capture
 * uses the address found by the device's last uncaptured call, so make the
 * first call on each device before any stream capture.  All calls share the one
 * array, so calls that overlap on the GPU (other streams, other threads)
 * race: serialise them.  Nothing is allocated or freed. */
#define PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES (4u << 20)
#define PK_ERR_SCRATCH_LIMIT (-4)
int pk_sparse_av_noalloc(uint64_t q, uint64_t k, uint64_t v, int dtype,
                         int kv_heads, int64_t kv_batch_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                         uint64_t ids, int64_t ids_stride, uint64_t count, uint64_t history, uint64_t length,
                         int U, int G, int d, int splits, uint64_t out, uint64_t stream);

/* ------------------------------------------------------------------------
 * Index build (a5 + a6) and append (a7).
 * Replaces IndexBuilder.group + Kernels.positive_top + moments + build_bits
 * (kernels/cuda_sm90/native.py:37-82,99-115; native_sources/hist.cu:3-22,
 * moments.cu:5-24; kernels/ppu_8b/pack.cu:5-6) with the exact semantics of
 * src/prismkv/core.py:92-103 (global positive BatchTopK with the flat-index
 * tie order of core.py:13-26) and core.py:186-201.
 * Keys of unit u, row t: keys + u*unit_stride + t*row_stride (elements).
 * ------------------------------------------------------------------------ */

/* center[u, d] = mean of the unit's N key rows (core.py:98). */
int pk_key_center(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride,
                  int U, int64_t N, int d, uint64_t center, uint64_t stream);

/* w_enc rounded to fp16 [F, d] for the bound-filtered build and append (no
 * counterpart in the reference: an internal operand copy, made once per SAE). */
int pk_sae_prepare_half(uint64_t w_enc, int F, int d, uint64_t w_half, uint64_t stream);

/* Builds buckets for U units sharing one SAE (w_enc[F, d], b_enc[F]).
 * With w_half from pk_sae_prepare_half and w_norm from pk_sae_prepare (both
 * non-zero), activations are first approximated on the tensor cores (fp16
 * operands) with a per-entry error bound; only entries the bounds cannot
 * place above or below the budget threshold are recomputed exactly (same
 * memberships).  If the bounds cannot bracket the threshold (degenerate or
 * out-of-range inputs) PK_STATUS_NEEDS_EXACT is raised and the caller reruns
 * without w_half / w_norm (append_index then changes nothing).
 * Token ids are written as token_base + t.  Bucket regions get
 * ceil(len*slack_frac) + slack_min spare slots for later appends;
 * ids_stride must be >= pk_build_ids_capacity(...).  */
int64_t pk_build_ids_capacity(int64_t N, int F, int key_mean, float slack_frac, int slack_min);
size_t pk_build_workspace_bytes(int U, int64_t N, int F, int key_mean, int64_t boundary_capacity);
int pk_build_index(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride,
                   uint64_t center, float key_scale, uint64_t w_enc, uint64_t b_enc,
                   uint64_t w_half, uint64_t w_norm,
                   int U, int64_t N, int d, int F, int key_mean, int64_t token_base,
                   float slack_frac, int slack_min,
                   uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride,
                   int64_t boundary_capacity, uint64_t workspace, uint64_t workspace_bytes,
                   uint64_t status, uint64_t stream);

/* Population mean / variance of the ORIGINAL keys per bucket (core.py:76-89). */
int pk_summarize(uint64_t keys, int dtype, int64_t unit_stride, int64_t row_stride,
                 uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride,
                 int U, int d, int F, uint64_t mean, uint64_t var, uint64_t stream);

/* Folds one block's bucket moments into a running state in place:
 * mean/var[U, F, d] fp32 of the state, whose bucket sizes are counts_a[U, F]
 * (int32), absorb mean_b/var_b of a block with sizes counts_b, by the
 * parallel formula of append_index (src/prismkv/core.py:194-199, the same
 * operation order).  The reference has no separate entry point for it; the
 * sequence-sharded index folds its shards' moments in token order with it. */
int pk_merge_moments(uint64_t counts_a, uint64_t mean, uint64_t var, uint64_t counts_b, uint64_t mean_b,
                     uint64_t var_b, int U, int F, int d, uint64_t stream);

/* Appends a block of n_new keys per unit (rows at new_keys + u*unit_stride +
 * t*row_stride) to an index built with history `history`: BatchTopK over the
 * block only with the stored centers, bucket lists extended in place (token
 * ids history + t), lens updated, and -- when mean/var are non-zero --
 * moments merged with the parallel formula of core.py:194-199.  All or
 * nothing: if any bucket region would overflow, the index is left unchanged
 * and PK_STATUS_BUCKET_FULL is raised. */
size_t pk_append_workspace_bytes(int U, int64_t n_new, int d, int F, int key_mean, int64_t boundary_capacity);
int pk_append_index(uint64_t new_keys, int dtype, int64_t unit_stride, int64_t row_stride, int64_t n_new,
                    uint64_t center, float key_scale, uint64_t w_enc, uint64_t b_enc,
                    uint64_t w_half, uint64_t w_norm,
                    int U, int d, int F, int key_mean, int64_t history,
                    uint64_t offsets, uint64_t lens, uint64_t ids, int64_t ids_stride,
                    uint64_t mean, uint64_t var,
                    int64_t boundary_capacity, uint64_t workspace, uint64_t workspace_bytes,
                    uint64_t status, uint64_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PRISMKV_B200_H */
