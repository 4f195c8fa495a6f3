/*
 * ssa_b200.h -- C ABI of libssa_sm100a.so, the B200 (sm_100a) implementation
 * of the SSA forward hot path: CodebookRouter (stages 1-2) and
 * sparse_exact_attention (stage 3) of chenxingqiang/SSA.
 *
 * Conventions
 *  - Every pointer in an args struct is a DEVICE pointer on the current CUDA
 *    device; sizes are element counts; strides are in ELEMENTS and the last
 *    (feature) dimension of every tensor must be contiguous.
 *  - The library never allocates device memory.  Scratch space is passed in
 *    as `workspace` (size from ssa_route_workspace_size()); the one entry
 *    point without a workspace, ssa_build_index_noalloc, uses a fixed 16 MiB
 *    array built into the library instead.
 *  - Every kernel is launched on the given stream; calls are asynchronous.
 *    Argument errors are reported synchronously through the return code.
 *    Data-dependent errors found on the device (an index outside [0, n))
 *    are OR-ed into the optional `status` word, which the caller reads after
 *    synchronising (SSA_DEVICE_* bits).
 *  - Inputs are never written.  Outputs are fully overwritten.
 *
 * Reference interfaces replaced (file:line in chenxingqiang/SSA):
 *  - ssa_route             CodebookRouter.forward            ssa/router.py:73-149
 *                          (+ _select_candidates / _build_candidate_mask,
 *                             ssa/router.py:151-259)
 *  - ssa_route_rope        apply_rotary_pos_emb + CodebookRouter.forward
 *                          (training/train_qwen.py:134-135, ssa/router.py:73-149)
 *  - ssa_code_assign       CodebookRouter.get_code_assignment ssa/router.py:261-275
 *  - ssa_sparse_attn       sparse_exact_attention            ssa/attention.py:12-115
 *  - ssa_sparse_attn_backward  its gradient (the reference differentiates
 *                          its gather + einsum with autograd)
 *  - ssa_select_from_scores, ssa_build_index, ssa_select_candidates
 *                          test hooks exposing the stage-1 selection
 *                          (ssa/router.py:129-141), the code->key index and the
 *                          candidate re-score/top-k (ssa/router.py:151-214)
 *                          on caller-provided inputs, for bit-exact parity
 *                          tests.  No reference counterpart of their own.
 */
#ifndef SSA_B200_H_
#define SSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SSA_OK = 0,
  SSA_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad stride      */
  SSA_ERR_UNSUPPORTED = 2,   /* a size outside the supported envelope        */
  SSA_ERR_WORKSPACE = 3,     /* workspace missing or too small               */
  SSA_ERR_ALIGNMENT = 4,     /* pointer/stride not 16-byte aligned           */
  SSA_ERR_CUDA = 5,          /* a CUDA launch failed                         */
  SSA_ERR_DEVICE = 6         /* device error word non-zero (ssa_read_status) */
} ssa_status;

/* Bits OR-ed into a device status word. */
#define SSA_DEVICE_INDEX_OOB 0x1   /* sparse_attn: an index < 0 or >= n was skipped  */
#define SSA_DEVICE_BAD_CODE 0x2    /* a caller-given code outside [0, n_codes) was
                                      read as code 0; the index and the indices are
                                      undefined                                     */
#define SSA_DEVICE_BAD_INDEX 0x4   /* a caller-given code->key index failed its check
                                      (a bucket or a key out of range); the indices
                                      are written as zeros                          */
#define SSA_DEVICE_INDEX_FULL 0x8  /* decode index: a bucket had no free slot; the
                                      entry was dropped (rebuild before appending
                                      more keys than min_free allows)               */
#define SSA_DEVICE_TIMEOUT 0x100   /* route: a pipeline wait gave up (~1 s); the
                                      affected codes are undefined                  */

typedef enum { SSA_F32 = 0, SSA_BF16 = 1, SSA_F16 = 2 } ssa_dtype;
typedef enum { SSA_I32 = 0, SSA_I64 = 1 } ssa_index_dtype;

/* ------------------------------------------------------------------------ */
/* Router (stages 1-2)                                                       */
/* ------------------------------------------------------------------------ */
typedef struct {
  /* sizes */
  int32_t batch;        /* independent sequences                              */
  int32_t n;            /* keys per sequence (seq_len)                        */
  int32_t n_q;          /* query rows per sequence (== n unless sharded)      */
  int32_t q_offset;     /* sequence position of query row 0 (query shard)     */
  int32_t h_q, h_kv;    /* h_q % h_kv == 0                                    */
  int32_t d;            /* head_dim                                           */
  int32_t d_s;          /* route_dim                                          */
  int32_t n_codes;      /* num_codebook                                       */
  int32_t a;            /* codes_per_query                                    */
  int32_t b;            /* codes_per_key                                      */
  int32_t top_k;        /* k                                                  */
  int32_t causal;       /* 1: keys j <= q_offset + i only                     */
  float temperature;    /* > 0; scores are divided by it (order-neutral)      */
  ssa_dtype dtype;      /* dtype of q and k                                   */
  ssa_dtype w_dtype;    /* dtype of w_qr, w_kr and codebook                   */
  int32_t codebook_heads; /* 1 (shared [N_c,d_s]) or h_kv ([h_kv,N_c,d_s])    */
  /* inputs */
  const void* q;  int64_t q_stride_b, q_stride_n, q_stride_h; /* [B,n_q,h_q,d] */
  const void* k;  int64_t k_stride_b, k_stride_n, k_stride_h; /* [B,n,h_kv,d]  */
  const void* w_qr;      /* [d_s, d] contiguous (nn.Linear weight)            */
  const void* w_kr;      /* [d_s, d] contiguous                               */
  const void* codebook;  /* [codebook_heads, n_codes, d_s] contiguous         */
  /* outputs */
  void* indices;                 /* [B, n_q, h_kv, top_k] contiguous          */
  ssa_index_dtype index_dtype;
  int32_t* q_codes;              /* optional [B, n_q, h_kv, a] contiguous     */
  int32_t* k_codes;              /* optional [B, n, h_kv, b] contiguous,
                                    16-byte aligned                           */
  int32_t* cand_counts;          /* optional [B, n_q, h_kv]: unique candidates */
  int32_t* status;               /* optional device word, SSA_DEVICE_* bits   */
} SsaRouteArgs;

/* Bytes of workspace ssa_route / ssa_code_assign need for these args. */
size_t ssa_route_workspace_size(const SsaRouteArgs* args);

/* CodebookRouter.forward(q, k, causal_mask, hard=True) -> indices
 * (ssa/router.py:73-149).  Canonical semantics: candidates are the keys that
 * share one of the query's top-a codes with their own top-b codes (and j <= i
 * when causal); they are ranked by the group-mean logit mean_g(q_g.k_j)/sqrt(d)
 * with the lower key index first among equal scores; fewer than min(k, n)
 * candidates are followed by the lowest-index non-candidate keys; k > n
 * is zero-padded (ssa/router.py:203-211). */
ssa_status ssa_route(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/* CodebookRouter.get_code_assignment(k) -> [B, n, h_kv, b] codes
 * (ssa/router.py:261-275).  Uses the k / w_kr / codebook fields of args and
 * writes args->k_codes (required). */
ssa_status ssa_code_assign(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes,
                           void* stream);

/* CodebookRouter.forward (ssa/router.py:73-149) with the key codes given:
 * reads args->k_codes [B, n, h_kv, b] -- as ssa_code_assign writes them, the
 * b codes of one key distinct -- instead of computing them from k, then
 * computes the query codes and runs stage 2 exactly as ssa_route.  For query
 * shards of one long sequence: each GPU assigns codes to its own key shard
 * (ssa_code_assign), the shards' codes and keys are gathered, and every GPU
 * routes its own queries (q_offset, n_q) against all n keys.  A code outside
 * [0, n_codes) sets SSA_DEVICE_BAD_CODE.  The reference computes the key codes
 * inline (ssa/router.py:114-130); the split is this library's. */
ssa_status ssa_route_with_key_codes(const SsaRouteArgs* args, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ssa_route_with_key_codes with the code->key index given as well:
 * bucket_ptr [B, h_kv, n_codes+1] and bucket_keys [B, h_kv, n*b] as
 * ssa_build_index writes them from args->k_codes.  For a GPU that routes
 * several query blocks of one sequence against the same keys: the index is
 * built once.  The index is checked on the device first (bucket bounds
 * non-decreasing within [0, n*b], keys in [0, n)); if the check fails,
 * SSA_DEVICE_BAD_INDEX is set and every index row is written as zeros.  No
 * reference counterpart of its own
 * (ssa/router.py:151-259 computes the candidate mask inline). */
ssa_status ssa_route_with_index(const SsaRouteArgs* args, const int32_t* bucket_ptr,
                                const int32_t* bucket_keys, void* workspace, size_t workspace_bytes,
                                void* stream);

/* Query rows given as up to SSA_MAX_SEGMENTS runs of consecutive sequence
 * positions: rows[s] rows starting at position positions[s], in order
 * (positions ascending, runs not overlapping, sum of rows = n_q).  A GPU
 * holding several blocks of one long sequence routes and attends all of them
 * in one call each.  (The reference processes one whole sequence; its
 * per-query computation, ssa/router.py:151-214 and ssa/attention.py:12-115,
 * does not depend on which other queries share the call.) */
#define SSA_MAX_SEGMENTS 8
typedef struct {
  int32_t count;
  int32_t rows[SSA_MAX_SEGMENTS];
  int32_t positions[SSA_MAX_SEGMENTS];
} SsaQuerySegments;

/* ssa_route_with_index for query rows in segments (args->q_offset is
 * ignored): row i of segment s is routed as the query at position
 * positions[s] + i, exactly as ssa_route would route it. */
ssa_status ssa_route_with_index_segments(const SsaRouteArgs* args, const SsaQuerySegments* segments,
                                         const int32_t* bucket_ptr, const int32_t* bucket_keys, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ssa_route_with_index_segments in two calls, so that a GPU of a
 * query-sharded sequence computes its query codes while the keys, their
 * codes and the index are still on their way.
 *
 * ssa_query_codes: the query half of stage 1 (ssa/router.py:102-112 and the
 * query top-a of :130): the a codes of every query group into args->q_codes
 * (required).  Reads q, w_qr and codebook.  The key fields (k, w_kr, n, b)
 * are checked as for ssa_route but not read: a caller without its keys yet
 * may describe its own query rows there (n = n_q).
 *
 * ssa_select_candidates_segments: stage 2 for query rows in segments over
 * given codes and a given index -- reads q, k, args->q_codes (a code outside
 * [0, n_codes) sets SSA_DEVICE_BAD_CODE), args->k_codes and the index
 * (checked on the device as in ssa_route_with_index); w_qr / w_kr / codebook
 * are checked but not read.  The two calls together give exactly the indices
 * of ssa_route_with_index_segments. */
ssa_status ssa_query_codes(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes, void* stream);
ssa_status ssa_select_candidates_segments(const SsaRouteArgs* args, const SsaQuerySegments* segments,
                                          const int32_t* bucket_ptr, const int32_t* bucket_keys,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* Rotary position embedding applied on load by ssa_route_rope: the
 * rotate-half form of the Qwen2 path of the reference
 * (training/train_qwen.py:134-135, transformers' apply_rotary_pos_emb):
 *   x_rot = x * cos + rotate_half(x) * sin,  rotate_half(x) = [-x2, x1],
 * evaluated elementwise in the dtype of q and k (each product and the sum
 * rounded to it, as the PyTorch expression does).  Row i of q (of k) uses
 * table row q_offset + i (row i). */
typedef struct {
  const void* cos;          /* [*, positions, d], dtype of q and k, last dim contiguous */
  const void* sin;          /* same layout as cos                          */
  int64_t table_stride_b;   /* elements between sequences; 0 shares one table */
  int64_t table_stride_n;   /* elements between positions                   */
  void* q_out;  int64_t q_out_stride_b, q_out_stride_n, q_out_stride_h; /* rotated q [B,n_q,h_q,d] */
  void* k_out;  int64_t k_out_stride_b, k_out_stride_n, k_out_stride_h; /* rotated k [B,n,h_kv,d]  */
} SsaRopeArgs;

/* RoPE + CodebookRouter.forward in one call: q and k in `args` are the
 * projections before RoPE; the routing projection rotates each row as it
 * loads it, writes the rotated rows to q_out / k_out, and stages 1-2 run on
 * the rotated tensors, so the result equals ssa_route on the rotated q and k
 * (bit for bit, with q_out / k_out equal to the PyTorch RoPE expression).
 * Pass q_out / k_out to ssa_sparse_attn afterwards.  Replaces the separate
 * apply_rotary_pos_emb of training/train_qwen.py:134-135 ahead of
 * CodebookRouter.forward (ssa/router.py:73-149).  16-bit q/k with
 * d in {64, 128} and d_s in {8, 16, 32, 64}; other shapes return
 * SSA_ERR_UNSUPPORTED.  Workspace: ssa_route_workspace_size(args). */
ssa_status ssa_route_rope(const SsaRouteArgs* args, const SsaRopeArgs* rope, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Incremental decode: the code->key index of a growing key cache            */
/* ------------------------------------------------------------------------ */
/* The reference has no decode path; its design notes keep the code->key
 * index incrementally so that a decode step need not rescan the cache
 * (ssa_design.md, incremental decode).  Bucket c of sequence bat, KV head h
 * (bh = bat * h_kv + h) owns the slots [start[c], start[c+1]) of row bh of
 * bucket_keys (and of bucket_codes) and holds its keys, ascending, in
 * [start[c], end[c]).  A build gives every bucket max(slack, its size) free
 * slots; an append writes a key's b entries at the ends of its b buckets.
 * *min_free is the fewest free slots of any bucket: the b codes of a key are
 * distinct, so appending t keys takes at most t slots of any bucket, and the
 * caller rebuilds before appending more keys than *min_free. */
typedef struct {
  int32_t* bucket_start;   /* [B, h_kv, n_codes + 1]                              */
  int32_t* bucket_end;     /* [B, h_kv, n_codes + 1] (the last column is unused)  */
  int32_t* bucket_keys;    /* [B, h_kv, entry_capacity]                           */
  int32_t* bucket_codes;   /* [B, h_kv, entry_capacity, 4], 16-byte aligned: each
                              entry's key codes (b == 4 only; NULL otherwise)     */
  int64_t entry_capacity;  /* slots per (sequence, KV head), see below            */
  int32_t slack;           /* >= 1                                                 */
  int32_t* min_free;       /* device word                                          */
  int64_t k_codes_stride_b; /* elements between the sequences of args->k_codes (a
                              cache of capacity C: C * h_kv * b); 0: n * h_kv * b */
} SsaDecodeIndex;

/* Slots per (sequence, KV head) that always suffice for up to max_keys keys:
 * 2 * max_keys * b + n_codes * slack. */
int64_t ssa_decode_index_capacity(int32_t max_keys, int32_t b, int32_t n_codes, int32_t slack);

/* (Re)builds the index of the args->n cached keys from their codes
 * args->k_codes [B, n, h_kv, b] and resets *min_free.  Workspace:
 * ssa_route_workspace_size(args).  Replaces the per-step index build of a
 * decode loop (the reference rebuilds its candidate mask from all keys,
 * ssa/router.py:216-259). */
ssa_status ssa_decode_index_build(const SsaRouteArgs* args, const SsaDecodeIndex* index, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Appends keys first .. first + count - 1 of args->k_codes (each after every
 * key already in the index) to the index: one small launch, independent of
 * the number of cached keys. */
ssa_status ssa_decode_index_append(const SsaRouteArgs* args, const SsaDecodeIndex* index, int32_t first,
                                   int32_t count, void* stream);

/* CodebookRouter.forward (ssa/router.py:73-149) for args->n_q query rows at
 * positions q_offset .. against the args->n keys of the index: the queries'
 * codes, then the candidate union, re-score and top-k of ssa_route, with the
 * index given (args->k_codes are the keys' codes).  Output as ssa_route. */
ssa_status ssa_decode_route(const SsaRouteArgs* args, const SsaDecodeIndex* index, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Sparse exact attention (stage 3)                                          */
/* ------------------------------------------------------------------------ */
typedef struct {
  int32_t batch, n_q, n;      /* query rows, keys per sequence                */
  int32_t q_offset;           /* sequence position of query row 0             */
  int32_t h_q, h_kv, d, top_k;
  int32_t causal;             /* 1: mask keys j > q_offset + i                */
  float scale;                /* logits = (q . k) / scale  (ssa/attention.py:37-38,107) */
  ssa_dtype dtype;            /* q, k, v and out                              */
  const void* q; int64_t q_stride_b, q_stride_n, q_stride_h;        /* [B,n_q,h_q,d]   */
  const void* k; int64_t k_stride_b, k_stride_n, k_stride_h;        /* [B,n,h_kv,d]    */
  const void* v; int64_t v_stride_b, v_stride_n, v_stride_h;        /* [B,n,h_kv,d]    */
  const void* indices; ssa_index_dtype index_dtype;
  int64_t idx_stride_b, idx_stride_n, idx_stride_h;                 /* [B,n_q,h_kv,k]  */
  void* out; int64_t out_stride_b, out_stride_n, out_stride_h;      /* [B,n_q,h_q,d]   */
  int32_t* status;            /* optional device word, SSA_DEVICE_* bits      */
} SsaAttnArgs;

/* sparse_exact_attention(q, k, v, indices, scale) (ssa/attention.py:12-115)
 * with the per-KV-head gather k[idx, h].  Online softmax in fp32.  A query
 * row none of whose indices is valid (with causal = 1, every index above
 * q_offset + i) gets a zero output row; the reference never masks in this
 * stage, and a softmax over no key would be 0/0. */
ssa_status ssa_sparse_attn(const SsaAttnArgs* args, void* stream);

/* ssa_sparse_attn for query rows in segments (args->q_offset is ignored):
 * with causal = 1, row i of segment s masks keys above positions[s] + i. */
ssa_status ssa_sparse_attn_segments(const SsaAttnArgs* args, const SsaQuerySegments* segments, void* stream);

/* Gradients of ssa_sparse_attn (the backward of sparse_exact_attention,
 * ssa/attention.py:12-115, which the reference differentiates with autograd).
 * args are the forward's, with args->out = the forward output (read only).
 * d_out has the strides of out; d_q is written with the strides of q (dtype
 * of q); d_k and d_v are fp32 [B, n, h_kv, d] contiguous and are zeroed
 * here, then accumulated with atomic adds (their rounding depends on the
 * order of the adds).  Indices receive no gradient. */
ssa_status ssa_sparse_attn_backward(const SsaAttnArgs* args, const void* d_out, void* d_q, float* d_k,
                                    float* d_v, void* stream);

/* ------------------------------------------------------------------------ */
/* Test hooks (bit-exact parity on caller-provided inputs)                   */
/* ------------------------------------------------------------------------ */

/* Top-`kk` of each row of fp32 `scores [rows, n_cols]`: indices sorted by
 * score descending, lower column first among equal scores; -0.0 == +0.0.
 * Runs the same selection code the fused scoring kernel uses
 * (ssa/router.py:130,141).  kk <= 32. */
ssa_status ssa_select_from_scores(const float* scores, int64_t rows, int32_t n_cols,
                                  int32_t kk, int32_t* out_idx, void* stream);

/* Code->key inverted index of k_codes [B, n, h_kv, b] (int32, contiguous):
 * bucket_ptr [B, h_kv, n_codes+1] and bucket_keys [B, h_kv, n*b] (keys
 * ascending within a bucket).  Workspace from ssa_route_workspace_size(). */
ssa_status ssa_build_index(const SsaRouteArgs* args, const int32_t* k_codes,
                           int32_t* bucket_ptr, int32_t* bucket_keys,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ssa_build_index without a workspace, for callers that cannot allocate
 * device memory -- code running where cudaMalloc is unavailable or forbidden
 * (inside a stream capture, under a runtime that owns all device memory, or
 * in a real-time loop that must not allocate).  No reference counterpart: the
 * reference never builds this index.
 *
 * Scratch (per-tile code counts and scan partials) comes from a 16 MiB array
 * inside the library, held on every GPU that loads it until the process
 * exits; calls needing more return SSA_ERR_UNSUPPORTED.  The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress), so make
 * it before any stream capture.  Every call on a device uses the same array:
 * calls that overlap on the GPU (different streams, no ordering) race and
 * corrupt each other's result.  Nothing in the array needs clearing: each call
 * writes every scratch word it reads.  The looked-up address is cached per
 * device for the life of the process: after cudaDeviceReset, or anything else
 * that destroys and recreates the device's primary context, the cached
 * address is stale and this entry point must not be called again.  Outputs
 * and limits otherwise as ssa_build_index. */
ssa_status ssa_build_index_noalloc(const SsaRouteArgs* args, const int32_t* k_codes,
                                   int32_t* bucket_ptr, int32_t* bucket_keys, void* stream);

/* Stage 2 from given codes: candidate union, causal filter, group-mean
 * re-score, top-k, filler and padding -- ssa_route without stage 1.
 * Reads args->q, args->k, args->q_codes, args->k_codes; writes
 * args->indices (and cand_counts if set). */
ssa_status ssa_select_candidates(const SsaRouteArgs* args, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Measurement hook (no reference counterpart): reads `bytes` of the device
 * buffer `buf` (16-byte aligned) `reps` times with 16-byte L2-only loads
 * across the whole GPU.  With a buffer that fits in L2, bytes * reps over the
 * launch's duration is the L2 read bandwidth the benchmark reports the
 * gather-bound kernels against.  *sink (device) is touched only to keep the
 * loads alive. */
ssa_status ssa_l2_read_probe(const void* buf, size_t bytes, int32_t reps, unsigned long long* sink, void* stream);

/* Human-readable text of a status code. */
const char* ssa_status_str(ssa_status s);

/* Text describing the last argument error of this thread (or ""). */
const char* ssa_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* SSA_B200_H_ */
