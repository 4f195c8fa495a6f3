// Kernel parameter blocks and launchers shared between the kernel files and
// the C-ABI layer (abi.cu).  Internal to libssa_sm100a.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ssa_b200.h"

namespace ssa {

// Query rows as up to kMaxSeg runs of consecutive sequence positions: row i
// of segment s (rows row[s] .. row[s+1]-1) sits at position pos[s] + i - row[s].
// Positions ascend with the row index.  One segment at q_offset is the plain
// contiguous block.
constexpr int kMaxSeg = 8;
struct QuerySegs {
  int count;
  int row[kMaxSeg + 1];
  int pos[kMaxSeg];
};
__device__ __forceinline__ int seg_pos(const QuerySegs& s, int i) {
  int k = 0;
#pragma unroll
  for (int t = 1; t < kMaxSeg; ++t) k += (t < s.count && i >= s.row[t]) ? 1 : 0;
  return s.pos[k] + (i - s.row[k]);
}
inline QuerySegs contiguous_segs(int q_offset, int n_q) {
  QuerySegs s{};
  s.count = 1;
  s.row[0] = 0;
  s.row[1] = n_q;
  s.pos[0] = q_offset;
  return s;
}

// K0: routing projection.  rows = batch*h_kv*n_rows, row order (bat, h, i).
struct RouteProjectParams {
  const void* x;           // q [B,n_rows,h_q,d] (group>1) or k [B,n_rows,h_kv,d]
  int64_t stride_b, stride_n, stride_h;
  const void* w;           // [d_s, d]
  float* out;              // [rows, d_s] L2-normalised route vectors
  int64_t rows, n_rows;
  int h_kv, group, d, d_s;
  // Optional rotate-half RoPE on load (tensor-core path only): row i of x is
  // rotated with table row pos_offset + i of rope_cos / rope_sin (dtype of x)
  // and written to x_out before it is projected.
  const void* rope_cos = nullptr;
  const void* rope_sin = nullptr;
  int64_t rope_sb = 0, rope_sn = 0, pos_offset = 0;
  void* x_out = nullptr;
  int64_t out_sb = 0, out_sn = 0, out_sh = 0;
  int32_t* status = nullptr;   // optional device word (SSA_DEVICE_TIMEOUT from the tcgen05 kernel)
};
bool route_project_rope_supported(int d, int d_s, ssa_dtype xt);
// The TMA-fed tcgen05 projection (route_tc.cu): 16-bit x without RoPE, d a
// multiple of 64, d_s in {16, 32, 64}, the group's heads contiguous in a row.
bool route_project_tc_supported(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt);
cudaError_t launch_route_project_tc(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt, cudaStream_t st);

// K1: codebook scoring + top-kk selection.  Route rows in (bat, h, i) order.
struct CodeSelectParams {
  const float* route;      // [batch_heads * n_rows, d_s]
  const float* codebook;   // normalised [codebook_heads, n_codes, d_s]
  int32_t* codes;          // out [B, n_rows, h_kv, kk]
  int64_t batch_heads, n_rows;
  int h_kv, codebook_heads, n_codes, d_s, kk;
  float temperature;
};

// K1 on tcgen05: rows in (bat, h, i) order, tiles of 128 rows within a head.
struct CodeScoreTcParams {
  const float* route;            // [batch_heads * n_rows, d_s] normalised
  const unsigned char* image;    // codebook chunk images [codebook_heads][n_codes/256][...]
  int32_t* codes;                // out [B, n_rows, h_kv, kk]
  int32_t* error;                // optional device status word
  int64_t batch_heads, n_rows, tiles_per_head;
  int h_kv, codebook_heads, n_codes, kk;
  float temperature;
};

// K2: code -> key inverted index.
struct IndexParams {
  const int32_t* k_codes;  // [B, n, h_kv, b]
  int32_t* bucket_ptr;     // [B*h_kv, n_codes+1]
  int32_t* bucket_keys;    // [B*h_kv, n*b]
  uint32_t* counts;        // [B*h_kv, n_codes, tiles] workspace
  uint32_t* partials;      // [B*h_kv, chunks] workspace
  int32_t* status;         // optional device word (SSA_DEVICE_BAD_CODE)
  int64_t k_codes_sb;      // elements between sequences of k_codes (n*h_kv*b when contiguous)
  int batch, n, h_kv, b, n_codes, tile_keys, tiles;
  int64_t chunks;          // scan chunks per (bat, h)
  int store_entry;         // 0: bucket_keys holds key rows j; 1: entry numbers j * b + slot
};

constexpr int kIndexSortEntries = 4096;  // entries sorted per tile
constexpr int kScanChunk = 4096;

inline int index_tile_keys(int b) { return kIndexSortEntries / b; }

// Checks a caller-given code->key index (bucket bounds non-decreasing within
// [0, n*b], keys in [0, n)); any violation sets *bad and SSA_DEVICE_BAD_INDEX.
// bucket_codes[e] = the 4 codes of key bucket_keys[e] (b == 4), so that a walk
// over the index reads an entry's key and its codes side by side; an entry
// outside [0, n) gets codes -1.
cudaError_t launch_index_codes(const int32_t* bucket_keys, const int32_t* k_codes, int4* bucket_codes,
                               int64_t batch_heads, int n, int h_kv, cudaStream_t st);
cudaError_t launch_validate_index(const int32_t* bucket_ptr, const int32_t* bucket_keys, int64_t batch_heads,
                                  int n_codes, int n, int b, int32_t* bad, int32_t* status, cudaStream_t st);

// The code->key index of a growing key cache (decode_index.cu): bucket c of
// (bat, h) = bh owns slots [start[c], start[c+1]) and holds its keys,
// ascending, in [start[c], end[c]) of keys + bh * entry_capacity.
struct DecodeIndexParams {
  int32_t* start;              // [B*h_kv, n_codes+1]
  int32_t* end;                // [B*h_kv, n_codes+1]
  int32_t* keys;               // [B*h_kv, entry_capacity]
  int4* codes;                 // optional (b == 4): each entry's key codes, [B*h_kv, entry_capacity]
  int32_t* min_free;           // optional device word: fewest free slots of any bucket (atomicMin)
  const int32_t* k_codes;      // [B, n, h_kv, b] codes of the cached keys ...
  int64_t k_codes_sb;          // ... sequences k_codes_sb elements apart
  int32_t* status;             // optional device word (SSA_DEVICE_BAD_CODE, SSA_DEVICE_INDEX_FULL)
  int64_t entry_capacity;
  int batch, n, h_kv, b, n_codes, slack;
};
// Lays the packed index (packed_ptr [B*h_kv, n_codes+1], packed_keys
// [B*h_kv, n*b]) out with max(slack, size) free slots after every bucket.
cudaError_t launch_decode_index_layout(const DecodeIndexParams& p, const int32_t* packed_ptr,
                                       const int32_t* packed_keys, cudaStream_t st);
// Appends keys first .. first+count-1 (each above every key already indexed).
cudaError_t launch_decode_index_append(const DecodeIndexParams& p, int first, int count, cudaStream_t st);

// Measurement hook (probe.cu): L2-only 16-byte reads of `bytes` of buf, `reps` times.
cudaError_t launch_l2_read_probe(const void* buf, size_t bytes, int reps, unsigned long long* sink, cudaStream_t st);

// K3: candidate union + causal filter + re-score + top-k + filler.
struct RescoreParams {
  const void* q; int64_t q_sb, q_sn, q_sh;
  const void* k; int64_t k_sb, k_sn, k_sh;
  const int32_t* q_codes;      // [B, n_q, h_kv, a]
  const int32_t* k_codes;      // [B, n, h_kv, b], sequences k_codes_sb elements apart
  int64_t k_codes_sb;
  const int32_t* bucket_ptr;   // [B*h_kv, n_codes+1]
  const int32_t* bucket_keys;  // [B*h_kv, n*b]
  void* out; int index_i64;    // [B, n_q, h_kv, top_k]
  int32_t* cand_counts;        // optional [B, n_q, h_kv]
  int32_t* status;             // optional device word (SSA_DEVICE_BAD_CODE)
  const int32_t* index_bad;    // optional: non-zero when a caller-given index failed validation
  const int4* bucket_codes;    // optional (b == 4): the codes of each index entry's key, [B*h_kv, n*4]
  // The index layout.  Packed (bucket_end NULL): bucket c of (bat, h) holds the
  // entries [ptr[c], ptr[c+1]) of bucket_keys + bh * entry_stride, with
  // ptr = bucket_ptr + bh * ptr_stride, ptr_stride = n_codes + 1 and
  // entry_stride = n * b.  With free room after each bucket (the decode index):
  // bucket c holds [ptr[c], bucket_end[bh * ptr_stride + c]) and entry_stride is
  // the entry capacity of one (bat, h); bucket_codes uses the same entry offsets.
  const int32_t* bucket_end;
  int64_t ptr_stride, entry_stride;
  int batch, n, n_q, q_offset, h_kv, group, d, a, b, n_codes, top_k, causal;
  QuerySegs seg;               // positions of the query rows (ascending)
  int cap;                     // shared-memory candidate capacity (power of two)
  int tier1_rows;              // warp path: query rows per (bat, h) the first tier takes (the
                               // lowest positions; 0 means all n_q)
  int32_t* ovf_count;          // workspace: units left to the general path ...
  int32_t* ovf_next;           // ... the next of them a general-path CTA claims ...
  int32_t* ovf_list;           // ... and their indices [B * n_q * h_kv]
  int32_t* ovf2_count;         // workspace: units passed from the first warp tier ...
  int32_t* ovf2_next;          // ... the next of them a second-tier warp claims ...
  int32_t* ovf2_list;          // ... and their indices [B * n_q * h_kv]
  int32_t* ovf3_count;         // workspace: units passed from the second warp tier to the third,
  int32_t* ovf3_next;          // the claim counter and
  int32_t* ovf3_list;          // their indices [B * n_q * h_kv]
  // Bucket-major path (rescore_bucket.cu), used when qbar is set.  Unit
  // u = (bat * h_kv + h) * n_q + i (row order) indexes the per-unit arrays.
  void* qbar;                  // [units, 2, d] group-mean query, 16-bit hi row then lo row
  int32_t* q_ptr;              // [B*h_kv, n_codes+1] code->query index of q_codes: entry
  int32_t* q_rows;             // [B*h_kv, n_q*a] numbers row * a + slot, ascending within a code
  uint32_t* q_counts;          // index-build scratch for that index
  uint32_t* q_partials;
  int32_t* part;               // [units, a+1]: offset of each of the unit's buckets in its
                               // segment; part[a] = the segment's length
  int64_t* seg_off;            // [units] start of the unit's segment in cand, -1 if none
  uint64_t* cand;              // candidate ranking keys of all segments (0 = dropped entry)
  int64_t cand_capacity;       // entries of cand
  unsigned long long* cursor;  // segment claim counter (zeroed by the launcher)
};

// Entries of (bat, h) = bh in the index, and the range [lo, hi) of bucket c.
__device__ __forceinline__ const int32_t* bucket_base(const RescoreParams& p, int bh) {
  return p.bucket_keys + static_cast<int64_t>(bh) * p.entry_stride;
}
__device__ __forceinline__ void bucket_range(const RescoreParams& p, int bh, int c, int& lo, int& hi) {
  const int32_t* ptr = p.bucket_ptr + static_cast<int64_t>(bh) * p.ptr_stride;
  lo = ptr[c];
  hi = p.bucket_end ? p.bucket_end[static_cast<int64_t>(bh) * p.ptr_stride + c] : ptr[c + 1];
}

// A caller-given code->key index that failed validation: the unit's indices
// are written as zeros (and its candidate count as 0) instead of being
// computed from the index.  Threads tid = 0 .. nthreads-1 of the unit call
// this with the same result.
__device__ __forceinline__ bool rescore_skip_bad_index(const RescoreParams& p, int bat, int i, int h, int tid,
                                                      int nthreads) {
  if (!p.index_bad || *p.index_bad == 0) return false;
  const int64_t row = (static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h;
  for (int e = tid; e < p.top_k; e += nthreads) {
    if (p.index_i64) static_cast<int64_t*>(p.out)[row * p.top_k + e] = 0;
    else static_cast<int32_t*>(p.out)[row * p.top_k + e] = 0;
  }
  if (p.cand_counts && tid == 0) p.cand_counts[row] = 0;
  return true;
}

// K4: sparse exact attention.
struct AttnParams {
  const void* q; int64_t q_sb, q_sn, q_sh;
  const void* k; int64_t k_sb, k_sn, k_sh;
  const void* v; int64_t v_sb, v_sn, v_sh;
  const void* idx; int64_t i_sb, i_sn, i_sh; int index_i64;
  void* out; int64_t o_sb, o_sn, o_sh;
  int32_t* status;
  int batch, n_q, n, q_offset, h_kv, group, d, top_k, causal;
  QuerySegs seg;               // positions of the query rows
  float inv_scale;
};

// Backward of K4: the forward's arguments (with `out` = the forward output,
// read) plus the output gradient (strides of `out`), dQ (strides of q) and
// fp32 dK / dV accumulators [B, n, h_kv, d] (row stride acc_sn), zeroed by
// the caller.
struct AttnBwdParams {
  AttnParams fwd;
  const void* d_out;
  void* d_q;
  float* d_k;
  float* d_v;
  int64_t acc_sn;
};

cudaError_t launch_route_project(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt,
                                 cudaStream_t st);
cudaError_t launch_codebook_normalize(const void* cb, ssa_dtype wt, float* out, int64_t rows,
                                      int d_s, cudaStream_t st);
cudaError_t launch_code_select(const CodeSelectParams& p, cudaStream_t st);
bool code_score_tc_supported(int d_s, int n_codes);
size_t codebook_image_bytes(int heads, int n_codes, int d_s);
cudaError_t launch_codebook_image(const float* cbn, void* img, int heads, int n_codes, int d_s,
                                  cudaStream_t st);
cudaError_t launch_code_score_tc(const CodeScoreTcParams& p, int d_s, cudaStream_t st);
cudaError_t launch_select_from_scores(const float* scores, int64_t rows, int n_cols, int kk,
                                      int32_t* out, cudaStream_t st);
cudaError_t launch_build_index(const IndexParams& p, cudaStream_t st);
cudaError_t launch_rescore(const RescoreParams& p, ssa_dtype dt, cudaStream_t st);
bool rescore_mma_supported(const RescoreParams& p, ssa_dtype dt);
cudaError_t launch_rescore_mma(const RescoreParams& p, ssa_dtype dt, cudaStream_t st);
// The bucket-major path: shapes it takes (16-bit, d 64 or 128, b 4, a <= 32,
// min(top_k, n) <= 512, packed index), and its stages up to the point where
// the units it could not hold are on the second walking tier's list
// (ovf2_list / ovf2_count, zeroed by the caller).
bool rescore_bucket_supported(int d, int a, int b, int k_eff, bool packed_index, ssa_dtype dt);
template <typename T, int D>
cudaError_t launch_rescore_bucket(const RescoreParams& p, cudaStream_t st);
size_t rescore_smem_bytes(int cap, int top_k);
cudaError_t launch_sparse_attn(const AttnParams& p, ssa_dtype dt, cudaStream_t st);
bool sparse_attn_mma_supported(const AttnParams& p, ssa_dtype dt);
cudaError_t launch_sparse_attn_mma(const AttnParams& p, ssa_dtype dt, cudaStream_t st);
cudaError_t launch_sparse_attn_bwd(const AttnBwdParams& p, ssa_dtype dt, cudaStream_t st);

}  // namespace ssa
