/*
 * attention_lab_b200 -- C ABI of the B200 (sm_100a) sparse-decode hot path of attention-lab.
 *
 * Every entry point takes plain device pointers, sizes, element strides, dtype codes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream). Nothing allocates, nothing synchronises the host,
 * launches are asynchronous on the given stream, and every call returns a status code (never throws).
 * `al_last_error()` returns the message of the last failing call on the calling thread.
 *
 * Shapes use the reference's conventions (attention-lab docs/IMPLEMENTATION.md):
 *   B batch, G KV groups, h query heads per group, d head dim (= 128), r index width (<= 32), C cache capacity,
 *   caches K/V [B,G,C,d] and index table zT [B,G,r,C], both contiguous; a flat row id is (b*G+g)*C + position.
 * Element strides are in elements of the tensor's own dtype; the innermost (d) stride must be 1 where not listed.
 */
#ifndef ATTENTION_LAB_B200_H
#define ATTENTION_LAB_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define AL_OK 0
#define AL_EINVAL 1       /* invalid shape, dtype, layout or range: the reference raises ValueError */
#define AL_ESTATE 2       /* state / order violation: the reference raises RuntimeError */
#define AL_ECUDA 3        /* the CUDA runtime reported an error at launch */
#define AL_EUNSUPPORTED 4 /* valid for the reference but outside what these kernels implement (ValueError) */

/* dtype codes */
#define AL_F32 0
#define AL_BF16 1

/* Message of the last failing call on this thread ("" when none). */
const char* al_last_error(void);

/* ABI version of this library. */
int al_version(void);

/* Synchronises the current device, then returns (and clears) the error bits kernels raised since the last call:
 * 1 = a row id outside [0, B*G*C) was skipped (the row is not read). */
int al_device_status(unsigned* error_bits);

/* a8: one layer's sparse decode step, fused into one launch (replaces attention-lab
 * src/attention_lab/decode.py:145-163 `sparse_decode_step_kernel`).
 *   q_main [B,G,h,1,d] (kv dtype), q_pre [B,G,h,1,d] (idx dtype): strides for B, G, h.
 *   k_pre_new [B,G,1,d] (idx dtype) or NULL: when given, z = Wk . k_pre_new is written to zT[..., write_col] first
 *   (decode.py:156-157); write_col must lie outside [lo, hi).
 *   wq_t [G,h*d,r] (1/sqrt(r) folded in), wk [G,r,d]: idx dtype, contiguous.
 *   fixed_rows [B,G,fixed_count] int64 flat rows of F; off_lo [B,G,1] int64 flat row of candidate 0.
 *   selected_count = fixed_count + k; 0 <= k <= hi - lo.
 *   out [B,G,h,d] (kv dtype, contiguous). rows_out [B,G,selected_count] int64 flat rows or NULL: F first, then the
 *   chosen candidates in ascending position order; with canonical_order every group's list is ascending
 *   (decode.py:160-161). scores_out [B,G,hi-lo] fp32 or NULL.
 *   Top-k ties are broken towards the smaller position. cluster: CTAs per (b,g) (0 = automatic, else 1..16). */
int al_sparse_decode_step(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                          const void* q_pre, int64_t qp_sb, int64_t qp_sg, int64_t qp_sh,
                          const void* k_cache, const void* v_cache, int kv_dtype,
                          void* zT, const void* wq_t, const void* wk, int idx_dtype,
                          const void* k_pre_new, int64_t kn_sb, int64_t kn_sg,
                          const int64_t* fixed_rows, const int64_t* off_lo,
                          int B, int G, int h, int d, int r, int C,
                          int lo, int hi, int k, int selected_count, int fixed_count, int write_col,
                          float scale, int canonical_order,
                          void* out, int64_t* rows_out, float* scores_out, int cluster, void* stream);

/* a5: score the candidate columns with a given u and select (replaces decode.py:86-93 `select_rows_kernel`).
 *   u [B,G,1,r] (idx dtype, strides for B, G). Output rows_out [B,G,selected_count] int64 (required). */
int al_select_rows(const void* u, int64_t u_sb, int64_t u_sg, const void* zT, int idx_dtype,
                   const int64_t* fixed_rows, const int64_t* off_lo,
                   int B, int G, int r, int C, int lo, int hi, int k, int selected_count, int fixed_count,
                   int canonical_order, int64_t* rows_out, float* scores_out, int cluster, void* stream);

/* a7: attention over listed flat rows, read in place (replaces decode.py:131-142 `gathered_decode_step_kernel`).
 *   rows [B,G,selected_count] int64 flat rows (any order; duplicates are read twice, as index_select does). */
int al_gathered_attend(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                       const void* k_cache, const void* v_cache, int kv_dtype, const int64_t* rows,
                       int B, int G, int h, int d, int C, int selected_count, float scale,
                       void* out, int cluster, void* stream);

/* a11: dense decode read over positions [0, valid_length) (replaces decode.py:174-176 `dense_decode_step` for a
 *   single query at the end of the legal range, full.py:17-45 `sdpa_fold`). */
int al_dense_decode(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                    const void* k_cache, const void* v_cache, int kv_dtype,
                    int B, int G, int h, int d, int C, int valid_length, float scale,
                    void* out, int cluster, void* stream);

/* a1: cache append (replaces qwen_wrap.py:90-106 `LabCache.append`): K/V rows [B,G,T,d] (4 strides each, dtype
 *   new_dtype, cast to kv_dtype) go to positions [start, start+T). The index columns [start, start+T) of zT are
 *   written from z_new [B,G,r,T] (4 strides, idx dtype) when given, else computed as Wk . k_pre (k_pre [B,G,T,d],
 *   4 strides, idx dtype; the prefill index build, qwen_wrap.py:320-324) when k_pre and wk are given. */
int al_append_kvz(void* k_cache, void* v_cache, int kv_dtype,
                  const void* k_new, const int64_t* k_strides, const void* v_new, const int64_t* v_strides,
                  int new_dtype, void* zT, int idx_dtype, const void* z_new, const int64_t* z_strides,
                  const void* k_pre, const int64_t* kp_strides, const void* wk,
                  int B, int G, int C, int d, int r, int start, int T, void* stream);

/* a2: index keys (replaces indexer.py:15-17 `project_keys`): z_out [B,G,r,C_out] columns [start, start+T) =
 *   wk[g] . k_pre[b,g,t] with k_pre [B,G,T,d] (4 strides). */
int al_project_keys(const void* k_pre, const int64_t* kp_strides, const void* wk, int idx_dtype,
                    int B, int G, int T, int d, int r, void* z_out, int C_out, int start, void* stream);

/* a3: index query (replaces indexer.py:20-24 `project_queries`): u [B,G,T,r] (contiguous) from q_pre [B,G,h,T,d]
 *   (5 strides) and wq_t [G,h*d,r]; written in idx dtype, or fp32 when out_f32. */
int al_project_queries(const void* q_pre, const int64_t* qp_strides, const void* wq_t, int idx_dtype,
                       int B, int G, int h, int T, int d, int r, void* u_out, int out_f32, void* stream);

/* a4: candidate scores (replaces indexer.py:27-29 `candidate_scores`): out [B,G,T,hi-lo] (contiguous) =
 *   u [B,G,T,r] (4 strides) . zT[..., lo:hi]; written in idx dtype, or fp32 when out_f32. */
int al_candidate_scores(const void* u, const int64_t* u_strides, const void* zT, int idx_dtype,
                        int B, int G, int T, int r, int C, int lo, int hi, void* out, int out_f32, void* stream);

/* ---- context split across GPUs (config C4; the multi-GPU protocol of the path, no single reference function):
 * positions [0, L) are split into P contiguous shards, one per rank. Per layer: al_context_local_topk on every rank,
 * an all-gather of the keys, al_context_threshold, al_gathered_attend_partial, an all-gather of the partials and
 * al_lse_merge. The chosen set equals the single-device top-k of decode.py:92 exactly. */

/* e1: local top-k of one shard (the select half of decode.py:145-163 on the shard's candidates [lo, hi)): writes the
 *   z column (k_pre_new, when this shard owns write_col), rows_out [B,G,fixed_count+k] (F, then the chosen
 *   candidates in ascending position order, as flat ids of the shard's cache) and keys_out [B,G,key_stride]: the
 *   64-bit key of every chosen candidate in the same order ((score order key << 32) | (2^32-1 - position), position
 *   = key_pos + column), zero past k. fixed_count + k must be >= 1. */
int al_context_local_topk(const void* q_pre, int64_t qp_sb, int64_t qp_sg, int64_t qp_sh,
                          void* zT, const void* wq_t, const void* wk, int idx_dtype,
                          const void* k_pre_new, int64_t kn_sb, int64_t kn_sg,
                          const int64_t* fixed_rows, const int64_t* off_lo,
                          int B, int G, int h, int r, int C, int lo, int hi, int k, int fixed_count, int write_col,
                          int64_t key_pos, int key_stride, int64_t* rows_out, uint64_t* keys_out, int cluster,
                          void* stream);

/* e2: global threshold: keys [world,B,G,key_stride] (every rank's keys_out) give the k-th largest key of each
 *   segment; rows_attend [B,G,fixed_count+k_local] = rows_in (this rank's rows_out) with -1 in place of every
 *   candidate below it. */
int al_context_threshold(const uint64_t* keys, int world, int rank, int B, int G, int key_stride, int k,
                         int fixed_count, int k_local, const int64_t* rows_in, int64_t* rows_attend, void* stream);

/* e3: partial attention over rows [B,G,n_rows] (flat ids, -1 = not read) of the shard's cache (decode.py:131-142
 *   without the final normalisation): part [B,G,h,130] = (m in the log2 domain, l, unnormalised acc[128]). */
int al_gathered_attend_partial(const void* q_main, int64_t q_sb, int64_t q_sg, int64_t q_sh,
                               const void* k_cache, const void* v_cache, int kv_dtype, const int64_t* rows,
                               int B, int G, int h, int d, int C, int n_rows, float scale,
                               float* part, int cluster, void* stream);

/* e4: log-sum-exp merge of world partials [world,B,G,h,130] into out [B,G,h,d] (dtype out_dtype): the combine of
 *   the reference's partitioned attend, metal_attend.py:147-169. */
int al_lse_merge(const float* parts, int world, int B, int G, int h, int d, void* out, int out_dtype, void* stream);

/* ---- peer exchange for the context split (replaces the two all-gathers of the protocol above; no reference
 * counterpart: the reference runs on one device). Every rank allocates one region with al_xchg_create, sends the
 * 64-byte handle to the others (any host channel) and opens theirs with al_xchg_open. A region holds, at offsets the
 * caller chooses, per channel (keys, partials): a gather area with one slot per rank, a flag word per rank (written by
 * that rank over NVLink), an epoch counter and a done counter. */

/* x1: cudaMalloc a zero-filled region of `bytes` on the current device; handle_out receives its 64-byte CUDA IPC
 *   handle. */
int al_xchg_create(size_t bytes, void** region, void* handle_out);
/* x2: map a peer's region (its 64-byte handle) into this process; peer access is enabled on first use. */
int al_xchg_open(const void* handle, void** peer_region);
/* x3: unmap a peer's region (al_xchg_open) / free this rank's region (al_xchg_create). */
int al_xchg_close(void* peer_region);
int al_xchg_destroy(void* region);
/* x4: push `bytes` (a multiple of 16) from src into slot `rank` of every rank's gather area of a channel
 *   (dst: device array of the world ranks' gather-area addresses; the slot is at dst[q] + rank * bytes), then, once
 *   every copy is visible
 *   system-wide, advance this rank's epoch counter of the channel and store it into every peer's flag for this rank
 *   (peer_flags: device array of world addresses of the ranks' flag arrays; done: a zeroed word of this rank's). */
int al_xchg_push(const void* src, size_t bytes, void* const* dst, int world, int rank, unsigned* done,
                 unsigned* counter, unsigned* const* peer_flags, void* stream);
/* x5: al_context_threshold over this rank's gather area of keys [world,B,G,key_stride] once every peer's flag of the
 *   channel has reached this rank's epoch (bounded wait of `spin` polls per peer; giving up sets error bit 2). */
int al_context_threshold_peer(const uint64_t* gather, const unsigned* flags, const unsigned* counter, int spin,
                              int world, int rank, int B, int G, int key_stride, int k, int fixed_count, int k_local,
                              const int64_t* rows_in, int64_t* rows_attend, void* stream);
/* x6: al_lse_merge over this rank's gather area of partials [world,B,G,h,130], after the same bounded wait. */
int al_lse_merge_peer(const float* gather, const unsigned* flags, const unsigned* counter, int spin, int world,
                      int rank, int B, int G, int h, int d, void* out, int out_dtype, void* stream);

/* n1: al_context_threshold for callers that cannot allocate device memory: a serving runtime that has already handed
 *   all of the GPU's memory to its own pool, or code that must not call cudaMalloc where it runs (for instance while
 *   the stream is being captured into a CUDA graph). No counterpart in the reference, and nothing is allocated: rank
 *   q's keys [B,G,key_stride] are read from rank_keys[q] (device array of world addresses: this GPU's memory or a
 *   peer's mapped region) into a scratch array that is part of the library image (4 MiB on every GPU that loads the
 *   library, held until the process exits), and the threshold runs over that copy. world*B*G*key_stride may not
 *   exceed 524 288 keys (AL_EUNSUPPORTED otherwise). The first call on a device looks up the scratch's device address;
 *   make it before any stream capture. Every call shares the scratch, so calls that overlap on the GPU (different
 *   streams, or different host threads) race and must be serialised by the caller. */
int al_context_threshold_noalloc(const uint64_t* const* rank_keys, int world, int rank, int B, int G, int key_stride,
                                 int k, int fixed_count, int k_local, const int64_t* rows_in, int64_t* rows_attend,
                                 void* stream);

/* Batched prefill scorer (config C5). No single reference counterpart: the reference selects nothing during prefill
 * (qwen_wrap.py:287-289); this applies its decode-time selection (candidates of selection.py:71-79 at legal length
 * p + 1, top-k of decode.py:86-93, ties to the smaller position) to every query position p of a prefill chunk.
 *
 * u [H, T, r] bf16 (element strides u_sh, u_st; r = 32), zT [H, r, C] bf16 (strides z_sh, z_ld; C, z_sh, z_ld multiples
 * of 8, 16-byte aligned). Query row t sits at position q_pos0 + t (q_pos0 + T <= min(C, 65536)). For every (head,
 * row): idx_out[(h*T + t)*kcap + j] = the chosen candidate positions in ascending order (min(k, M) of them, M the
 * row's candidate count), -1 in the remaining slots up to kcap (k <= kcap). scores_out, when not NULL, is [H, T, C]
 * fp32 and receives the scores of every candidate column (other entries untouched). Scores are bf16 products with
 * fp32 accumulation on the tensor cores. */
int al_prefill_score_topk(const void* u, long long u_sh, long long u_st, const void* zT, long long z_sh, long long z_ld,
                          int H, int T, int C, int r, int q_pos0, int k, int kcap, int* idx_out, float* scores_out,
                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTENTION_LAB_B200_H */
