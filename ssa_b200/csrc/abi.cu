// C-ABI entry points of libssa_sm100a.so (declared in include/ssa_b200.h).
//
// This layer validates arguments, lays out the caller's workspace and
// launches the stage kernels on the caller's stream.  It never allocates.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace {

thread_local std::string g_last_error;

ssa_status fail(ssa_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
ssa_status fail(ssa_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

ssa_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SSA_OK;
  return fail(SSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t elem_size(ssa_dtype t) { return t == SSA_F32 ? 4 : 2; }
bool valid_dtype(ssa_dtype t) { return t == SSA_F32 || t == SSA_BF16 || t == SSA_F16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool stride16(int64_t s, ssa_dtype t) { return (s * static_cast<int64_t>(elem_size(t))) % 16 == 0; }

constexpr size_t kAlign = 256;
size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

constexpr int kMaxCap = 16384;   // shared-memory candidate capacity limit

int rescore_cap(int k_eff) {
  int cap = 2048;
  while (cap < k_eff) cap <<= 1;
  return cap;
}

// Workspace regions for a route call.
struct RouteLayout {
  size_t q_route, k_route, cb_norm, cb_image, q_codes, k_codes, counts, partials, bucket_ptr,
      bucket_keys, bucket_codes, ovf, ovf2, ovf3, flags;
  // bucket-major re-score (rescore_bucket.cu), when `bucket`
  bool bucket;
  size_t qbar, q_ptr, q_rows, q_counts, q_partials, part, seg_off, cursor, cand;
  int64_t cand_capacity;
  size_t total;
  int tiles;
  int64_t chunks;
};

// The bucket-major re-score runs where it applies (16-bit q/k, d 64 or 128,
// b = 4, a <= 32, min(top_k, n) <= 512) unless SSA_RESCORE=walk selects the
// walking kernel for every unit (both give the same indices).
bool bucket_rescore(const SsaRouteArgs& a) {
  const char* env = std::getenv("SSA_RESCORE");
  if (env && std::strcmp(env, "walk") == 0) return false;
  return static_cast<int64_t>(a.n_q) * a.a < (1ll << 31) &&
         ssa::rescore_bucket_supported(a.d, a.a, a.b, std::min(a.top_k, a.n), true, static_cast<ssa_dtype>(a.dtype));
}

// Candidate-buffer entries a unit is given: twice the larger of k and the
// candidates expected with uniformly used codes (a * b / n_codes of the keys
// a query sees; under the causal mask a query sees its prefix, taken at the
// middle of the call's rows or of the sequence, whichever is later).  A unit
// that finds the buffer full is re-scored by the walking kernel instead.
// SSA_RESCORE_UNIT_ROOM=<entries> overrides the figure (tests use a small
// value to send units down the walking kernel).
int64_t cand_per_unit(const SsaRouteArgs& a) {
  if (const char* env = std::getenv("SSA_RESCORE_UNIT_ROOM")) {
    const long long v = std::atoll(env);
    if (v >= 0) return v;
  }
  const double visible = a.causal ? std::min<double>(a.n, std::max(a.q_offset + a.n_q / 2.0, a.n / 2.0)) : a.n;
  const double expect = static_cast<double>(a.a) * a.b * visible / a.n_codes;
  const double per = 2.0 * std::max<double>(std::min(a.top_k, a.n), expect);
  return std::min<int64_t>(static_cast<int64_t>(std::ceil(per)), static_cast<int64_t>(a.n) * a.b);
}

// `bucket_ok`: false for the decode entry points, which always take the
// walking re-score (their index has free room after each bucket), so their
// workspace never holds the bucket path's regions.
RouteLayout route_layout(const SsaRouteArgs& a, bool bucket_ok = true) {
  RouteLayout L{};
  const int64_t B = a.batch, hk = a.h_kv;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t at = off; off += round_up(bytes); return at; };
  L.q_route = take(static_cast<size_t>(B * hk * a.n_q * a.d_s) * 4);
  L.k_route = take(static_cast<size_t>(B * hk * a.n * a.d_s) * 4);
  L.cb_norm = take(static_cast<size_t>(a.codebook_heads) * a.n_codes * a.d_s * 4);
  L.cb_image = take(ssa::code_score_tc_supported(a.d_s, a.n_codes)
                        ? ssa::codebook_image_bytes(a.codebook_heads, a.n_codes, a.d_s)
                        : 0);
  L.q_codes = take(static_cast<size_t>(B * a.n_q * hk * a.a) * 4);
  L.k_codes = take(static_cast<size_t>(B * a.n * hk * a.b) * 4);
  const int tile_keys = a.b > 0 ? ssa::index_tile_keys(a.b) : 1;
  L.tiles = static_cast<int>(ssa::cdiv(a.n, tile_keys));
  L.chunks = ssa::cdiv(static_cast<int64_t>(a.n_codes) * L.tiles, ssa::kScanChunk);
  L.counts = take(static_cast<size_t>(B * hk) * a.n_codes * L.tiles * 4);
  L.partials = take(static_cast<size_t>(B * hk * L.chunks) * 4);
  L.bucket_ptr = take(static_cast<size_t>(B * hk) * (a.n_codes + 1) * 4);
  L.bucket_keys = take(static_cast<size_t>(B * hk) * a.n * a.b * 4);
  L.bucket_codes = take(a.b == 4 ? static_cast<size_t>(B * hk) * a.n * 4 * 16 : 0);   // int4 per entry
  L.ovf = take((2 + static_cast<size_t>(B * hk) * a.n_q) * 4);   // overflow count, claim counter, unit list
  L.ovf2 = take((2 + static_cast<size_t>(B * hk) * a.n_q) * 4);  // second-tier count, claim counter, list
  L.ovf3 = take((2 + static_cast<size_t>(B * hk) * a.n_q) * 4);  // third tier, the same
  L.flags = take(4);                                               // index-validation flag
  L.bucket = bucket_ok && a.a >= 1 && bucket_rescore(a);
  if (L.bucket) {
    const int64_t units = B * hk * a.n_q;
    const int qtiles = static_cast<int>(ssa::cdiv(a.n_q, ssa::index_tile_keys(a.a)));
    const int64_t qchunks = ssa::cdiv(static_cast<int64_t>(a.n_codes) * qtiles, ssa::kScanChunk);
    L.qbar = take(static_cast<size_t>(units) * 2 * a.d * 2);
    L.q_ptr = take(static_cast<size_t>(B * hk) * (a.n_codes + 1) * 4);
    L.q_rows = take(static_cast<size_t>(B * hk) * a.n_q * a.a * 4);
    L.q_counts = take(static_cast<size_t>(B * hk) * a.n_codes * qtiles * 4);
    L.q_partials = take(static_cast<size_t>(B * hk * qchunks) * 4);
    L.part = take(static_cast<size_t>(units) * (a.a + 1) * 4);
    L.seg_off = take(static_cast<size_t>(units) * 8);
    L.cursor = take(8);
    L.cand_capacity = units * cand_per_unit(a);
    L.cand = take(static_cast<size_t>(L.cand_capacity) * 8);
  }
  L.total = off;
  return L;
}

// Validation shared by the router entry points.  `need_q` is false for
// get_code_assignment, which reads only k.
ssa_status check_route(const SsaRouteArgs* a, bool need_q, bool need_stage2) {
  if (!a) return fail(SSA_ERR_INVALID_ARG, "args is NULL");
  if (a->batch < 0 || a->n < 1 || a->n_q < 0 || a->q_offset < 0)
    return fail(SSA_ERR_INVALID_ARG, "bad sizes batch=%d n=%d n_q=%d q_offset=%d", a->batch, a->n,
                a->n_q, a->q_offset);
  if (a->h_kv < 1 || a->h_q < 1 || a->h_q % a->h_kv != 0)
    return fail(SSA_ERR_INVALID_ARG, "num_q_heads (%d) must be a multiple of num_kv_heads (%d)",
                a->h_q, a->h_kv);
  if (a->d < 8 || a->d > 256 || a->d % 8 != 0)
    return fail(SSA_ERR_UNSUPPORTED, "head_dim %d: need a multiple of 8 in [8, 256]", a->d);
  if (!(a->d_s == 4 || a->d_s == 8 || a->d_s == 16 || a->d_s == 32 || a->d_s == 64))
    return fail(SSA_ERR_UNSUPPORTED, "route_dim %d: need 4, 8, 16, 32 or 64", a->d_s);
  if (a->n_codes < 1 || a->n_codes > 32767)
    return fail(SSA_ERR_UNSUPPORTED, "num_codebook %d: need 1..32767", a->n_codes);
  if (a->b < 1 || a->b > 32 || a->b > a->n_codes)
    return fail(SSA_ERR_UNSUPPORTED, "codes_per_key %d: need 1..min(32, num_codebook)", a->b);
  if (need_q && (a->a < 1 || a->a > 32 || a->a > a->n_codes))
    return fail(SSA_ERR_UNSUPPORTED, "codes_per_query %d: need 1..min(32, num_codebook)", a->a);
  if (need_stage2) {
    if (a->top_k < 1) return fail(SSA_ERR_INVALID_ARG, "top_k %d < 1", a->top_k);
    if (std::min(a->top_k, a->n) > kMaxCap)
      return fail(SSA_ERR_UNSUPPORTED, "min(top_k, n) = %d exceeds %d", std::min(a->top_k, a->n), kMaxCap);
    if (!a->indices) return fail(SSA_ERR_INVALID_ARG, "indices is NULL");
    if (a->index_dtype != SSA_I32 && a->index_dtype != SSA_I64)
      return fail(SSA_ERR_INVALID_ARG, "bad index dtype");
    if (static_cast<int64_t>(a->q_offset) + a->n_q > a->n)
      return fail(SSA_ERR_INVALID_ARG, "q_offset + n_q (%d + %d) exceeds n (%d)", a->q_offset, a->n_q, a->n);
  }
  if (static_cast<int64_t>(a->n) * a->b >= (1ll << 31))
    return fail(SSA_ERR_UNSUPPORTED, "n * codes_per_key must be < 2^31");
  // the re-score numbers its (sequence, KV head, query) units with 32-bit ints
  if (static_cast<int64_t>(a->batch) * a->h_kv * std::max(a->n_q, a->n) >= (1ll << 31))
    return fail(SSA_ERR_UNSUPPORTED, "batch * num_kv_heads * seq_len must be < 2^31");
  if (!(a->temperature > 0.f)) return fail(SSA_ERR_INVALID_ARG, "temperature must be > 0");
  if (!valid_dtype(a->dtype) || !valid_dtype(a->w_dtype))
    return fail(SSA_ERR_INVALID_ARG, "bad dtype");
  if (a->codebook_heads != 1 && a->codebook_heads != a->h_kv)
    return fail(SSA_ERR_INVALID_ARG, "codebook_heads %d must be 1 or num_kv_heads", a->codebook_heads);
  if (!a->k || !a->w_kr || !a->codebook) return fail(SSA_ERR_INVALID_ARG, "k / w_kr / codebook is NULL");
  if (need_q && (!a->q || !a->w_qr)) return fail(SSA_ERR_INVALID_ARG, "q / w_qr is NULL");
  // the re-score reads the b = 4 codes of a key as one 16-byte vector
  if (a->k_codes && !aligned16(a->k_codes))
    return fail(SSA_ERR_ALIGNMENT, "k_codes must be 16-byte aligned");
  if (!aligned16(a->k) || !stride16(a->k_stride_n, a->dtype) || !stride16(a->k_stride_h, a->dtype) ||
      !stride16(a->k_stride_b, a->dtype))
    return fail(SSA_ERR_ALIGNMENT, "k must be 16-byte aligned with 16-byte strides");
  if (need_q && (!aligned16(a->q) || !stride16(a->q_stride_n, a->dtype) ||
                 !stride16(a->q_stride_h, a->dtype) || !stride16(a->q_stride_b, a->dtype)))
    return fail(SSA_ERR_ALIGNMENT, "q must be 16-byte aligned with 16-byte strides");
  return SSA_OK;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

// Codebook scoring + top-kk of `rows` routed vectors: the tcgen05 kernel when
// the shape allows it (d_s 16/32, N_c a multiple of 256), else the CUDA-core one.
cudaError_t score_and_select(const SsaRouteArgs& a, const RouteLayout& L, void* ws, const float* route,
                             int64_t n_rows, int kk, int32_t* codes, cudaStream_t st) {
  using namespace ssa;
  const int64_t bhs = static_cast<int64_t>(a.batch) * a.h_kv;
  if (code_score_tc_supported(a.d_s, a.n_codes)) {
    CodeScoreTcParams tp{};
    tp.route = route;
    tp.image = at<unsigned char>(ws, L.cb_image);
    tp.codes = codes;
    tp.error = a.status;
    tp.batch_heads = bhs;
    tp.n_rows = n_rows;
    tp.tiles_per_head = cdiv(n_rows, 128);
    tp.h_kv = a.h_kv;
    tp.codebook_heads = a.codebook_heads;
    tp.n_codes = a.n_codes;
    tp.kk = kk;
    tp.temperature = a.temperature;
    return launch_code_score_tc(tp, a.d_s, st);
  }
  CodeSelectParams sp{route, at<float>(ws, L.cb_norm), codes, bhs, n_rows, a.h_kv, a.codebook_heads,
                      a.n_codes, a.d_s, kk, a.temperature};
  return launch_code_select(sp, st);
}

// `rope` (optional): rotate q and k on load and write the rotated rows to its
// q_out / k_out (ssa_route_rope).
ssa_status run_stage1(const SsaRouteArgs& a, const RouteLayout& L, void* ws, cudaStream_t st,
                      bool keys, bool queries, int32_t* q_codes, int32_t* k_codes,
                      const SsaRopeArgs* rope = nullptr) {
  using namespace ssa;
  cudaError_t e = launch_codebook_normalize(a.codebook, a.w_dtype, at<float>(ws, L.cb_norm),
                                            static_cast<int64_t>(a.codebook_heads) * a.n_codes, a.d_s, st);
  if (e != cudaSuccess) return cuda_status(e, "codebook_normalize");
  if (code_score_tc_supported(a.d_s, a.n_codes)) {
    e = launch_codebook_image(at<float>(ws, L.cb_norm), at<void>(ws, L.cb_image), a.codebook_heads,
                              a.n_codes, a.d_s, st);
    if (e != cudaSuccess) return cuda_status(e, "codebook_image");
  }
  if (keys) {
    RouteProjectParams kp{a.k, a.k_stride_b, a.k_stride_n, a.k_stride_h, a.w_kr,
                          at<float>(ws, L.k_route), static_cast<int64_t>(a.batch) * a.h_kv * a.n, a.n,
                          a.h_kv, 1, a.d, a.d_s};
    kp.status = a.status;
    if (rope) {
      kp.rope_cos = rope->cos; kp.rope_sin = rope->sin;
      kp.rope_sb = rope->table_stride_b; kp.rope_sn = rope->table_stride_n; kp.pos_offset = 0;
      kp.x_out = rope->k_out;
      kp.out_sb = rope->k_out_stride_b; kp.out_sn = rope->k_out_stride_n; kp.out_sh = rope->k_out_stride_h;
    }
    e = launch_route_project(kp, a.dtype, a.w_dtype, st);
    if (e != cudaSuccess) return cuda_status(e, "route_project(k)");
    e = score_and_select(a, L, ws, at<float>(ws, L.k_route), a.n, a.b, k_codes, st);
    if (e != cudaSuccess) return cuda_status(e, "code_select(k)");
  }
  if (queries && a.n_q > 0) {
    RouteProjectParams qp{a.q, a.q_stride_b, a.q_stride_n, a.q_stride_h, a.w_qr,
                          at<float>(ws, L.q_route), static_cast<int64_t>(a.batch) * a.h_kv * a.n_q,
                          a.n_q, a.h_kv, a.h_q / a.h_kv, a.d, a.d_s};
    qp.status = a.status;
    if (rope) {
      qp.rope_cos = rope->cos; qp.rope_sin = rope->sin;
      qp.rope_sb = rope->table_stride_b; qp.rope_sn = rope->table_stride_n; qp.pos_offset = a.q_offset;
      qp.x_out = rope->q_out;
      qp.out_sb = rope->q_out_stride_b; qp.out_sn = rope->q_out_stride_n; qp.out_sh = rope->q_out_stride_h;
    }
    e = launch_route_project(qp, a.dtype, a.w_dtype, st);
    if (e != cudaSuccess) return cuda_status(e, "route_project(q)");
    e = score_and_select(a, L, ws, at<float>(ws, L.q_route), a.n_q, a.a, q_codes, st);
    if (e != cudaSuccess) return cuda_status(e, "code_select(q)");
  }
  return SSA_OK;
}

ssa::IndexParams index_params(const SsaRouteArgs& a, const RouteLayout& L, void* ws,
                              const int32_t* k_codes, int32_t* bucket_ptr, int32_t* bucket_keys) {
  ssa::IndexParams ip{};
  ip.k_codes = k_codes;
  ip.bucket_ptr = bucket_ptr;
  ip.bucket_keys = bucket_keys;
  ip.counts = at<uint32_t>(ws, L.counts);
  ip.partials = at<uint32_t>(ws, L.partials);
  ip.status = a.status;
  ip.k_codes_sb = static_cast<int64_t>(a.n) * a.h_kv * a.b;
  ip.batch = a.batch;
  ip.n = a.n;
  ip.h_kv = a.h_kv;
  ip.b = a.b;
  ip.n_codes = a.n_codes;
  ip.tile_keys = ssa::index_tile_keys(a.b);
  ip.tiles = L.tiles;
  ip.chunks = L.chunks;
  return ip;
}

// Candidate union, re-score and top-k over a built code->key index.
// `dix` (decode): the index is the slotted one of ssa_decode_index_build,
// bucket_ptr / bucket_keys are ignored and its entry codes are read as stored.
ssa_status run_rescore(const SsaRouteArgs& a, const RouteLayout& L, void* ws, cudaStream_t st,
                       const int32_t* q_codes, const int32_t* k_codes, const int32_t* bucket_ptr,
                       const int32_t* bucket_keys, const int32_t* index_bad,
                       const SsaDecodeIndex* dix = nullptr, const ssa::QuerySegs* segs = nullptr) {
  using namespace ssa;
  RescoreParams rp{};
  rp.q = a.q; rp.q_sb = a.q_stride_b; rp.q_sn = a.q_stride_n; rp.q_sh = a.q_stride_h;
  rp.k = a.k; rp.k_sb = a.k_stride_b; rp.k_sn = a.k_stride_n; rp.k_sh = a.k_stride_h;
  rp.q_codes = q_codes;
  rp.k_codes = k_codes;
  rp.k_codes_sb = static_cast<int64_t>(a.n) * a.h_kv * a.b;
  rp.bucket_ptr = bucket_ptr;
  rp.bucket_keys = bucket_keys;
  rp.bucket_end = nullptr;                            // packed index
  rp.ptr_stride = static_cast<int64_t>(a.n_codes) + 1;
  rp.entry_stride = static_cast<int64_t>(a.n) * a.b;
  rp.index_bad = index_bad;
  if (dix) {
    rp.bucket_ptr = dix->bucket_start;
    rp.bucket_end = dix->bucket_end;
    rp.bucket_keys = dix->bucket_keys;
    rp.entry_stride = dix->entry_capacity;
    rp.bucket_codes = reinterpret_cast<const int4*>(dix->bucket_codes);
    if (dix->k_codes_stride_b) rp.k_codes_sb = dix->k_codes_stride_b;
  } else if (a.b == 4) {
    int4* bc = at<int4>(ws, L.bucket_codes);
    const cudaError_t ec = launch_index_codes(bucket_keys, k_codes, bc, static_cast<int64_t>(a.batch) * a.h_kv, a.n,
                                              a.h_kv, st);
    if (ec != cudaSuccess) return cuda_status(ec, "index_codes");
    rp.bucket_codes = bc;
  }
  rp.out = a.indices;
  rp.index_i64 = a.index_dtype == SSA_I64;
  rp.cand_counts = a.cand_counts;
  rp.status = a.status;
  rp.batch = a.batch; rp.n = a.n; rp.n_q = a.n_q; rp.q_offset = a.q_offset;
  rp.seg = segs ? *segs : ssa::contiguous_segs(a.q_offset, a.n_q);
  rp.h_kv = a.h_kv; rp.group = a.h_q / a.h_kv; rp.d = a.d; rp.a = a.a; rp.b = a.b;
  rp.n_codes = a.n_codes; rp.top_k = a.top_k; rp.causal = a.causal ? 1 : 0;
  rp.cap = rescore_cap(std::min(a.top_k, a.n));
  rp.ovf_count = at<int32_t>(ws, L.ovf);
  rp.ovf_next = at<int32_t>(ws, L.ovf) + 1;
  rp.ovf_list = at<int32_t>(ws, L.ovf) + 2;
  rp.ovf2_count = at<int32_t>(ws, L.ovf2);
  rp.ovf2_next = at<int32_t>(ws, L.ovf2) + 1;
  rp.ovf2_list = at<int32_t>(ws, L.ovf2) + 2;
  rp.ovf3_count = at<int32_t>(ws, L.ovf3);
  rp.ovf3_next = at<int32_t>(ws, L.ovf3) + 1;
  rp.ovf3_list = at<int32_t>(ws, L.ovf3) + 2;
  if (L.bucket && !dix) {
    rp.qbar = at<void>(ws, L.qbar);
    rp.q_ptr = at<int32_t>(ws, L.q_ptr);
    rp.q_rows = at<int32_t>(ws, L.q_rows);
    rp.q_counts = at<uint32_t>(ws, L.q_counts);
    rp.q_partials = at<uint32_t>(ws, L.q_partials);
    rp.part = at<int32_t>(ws, L.part);
    rp.seg_off = at<int64_t>(ws, L.seg_off);
    rp.cursor = at<unsigned long long>(ws, L.cursor);
    rp.cand = at<uint64_t>(ws, L.cand);
    rp.cand_capacity = L.cand_capacity;
  }
  return cuda_status(launch_rescore(rp, a.dtype, st), "rescore_topk");
}

ssa_status run_stage2(const SsaRouteArgs& a, const RouteLayout& L, void* ws, cudaStream_t st,
                      const int32_t* q_codes, const int32_t* k_codes) {
  ssa::IndexParams ip = index_params(a, L, ws, k_codes, at<int32_t>(ws, L.bucket_ptr),
                                     at<int32_t>(ws, L.bucket_keys));
  cudaError_t e = ssa::launch_build_index(ip, st);
  if (e != cudaSuccess) return cuda_status(e, "build_index");
  return run_rescore(a, L, ws, st, q_codes, k_codes, ip.bucket_ptr, ip.bucket_keys, nullptr);
}

// ---------------------------------------------------------------------------
// Allocation-free index build (ssa_build_index_noalloc)
//
// For callers that cannot allocate device memory: code running inside a CUDA
// stream capture (where cudaMalloc is not allowed), under a runtime that owns
// all device memory, or in a loop that must never allocate.  Its scratch -- the per-tile code counts and the scan partials that
// ssa_build_index takes from the caller's workspace -- lives in this
// file-scope device array instead.  Every GPU that loads the library holds the
// array until the process exits.  Host code cannot use the symbol itself as a
// device address, so the address is looked up once per device (with that
// device current) by cudaGetSymbolAddress and cached.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;   // 16 MiB
__device__ __align__(256) unsigned char g_index_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

ssa_status noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SSA_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_index_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(index scratch)");
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SSA_OK;
}

// Query segments of a caller (ssa_*_segments): 1..kMaxSeg runs covering the
// n_q rows in order, positions ascending and inside [0, n).
ssa_status check_segments(const SsaQuerySegments* s, int n_q, int n, ssa::QuerySegs& out) {
  if (!s) return fail(SSA_ERR_INVALID_ARG, "segments is NULL");
  if (s->count < 1 || s->count > SSA_MAX_SEGMENTS)
    return fail(SSA_ERR_INVALID_ARG, "segment count %d outside 1..%d", s->count, SSA_MAX_SEGMENTS);
  out = ssa::QuerySegs{};
  out.count = s->count;
  int64_t rows = 0, next_pos = 0;
  for (int i = 0; i < s->count; ++i) {
    if (s->rows[i] < 0 || s->positions[i] < next_pos)
      return fail(SSA_ERR_INVALID_ARG, "segment %d: rows %d at position %d (positions must ascend, segments not overlap)",
                  i, s->rows[i], s->positions[i]);
    out.row[i] = static_cast<int>(rows);
    out.pos[i] = s->positions[i];
    rows += s->rows[i];
    next_pos = static_cast<int64_t>(s->positions[i]) + s->rows[i];
    if (next_pos > n) return fail(SSA_ERR_INVALID_ARG, "segment %d ends at position %lld > n = %d", i,
                                  static_cast<long long>(next_pos), n);
  }
  if (rows != n_q) return fail(SSA_ERR_INVALID_ARG, "segments cover %lld rows, n_q = %d", static_cast<long long>(rows), n_q);
  out.row[s->count] = n_q;
  return SSA_OK;
}

// Validation of a caller's decode index (ssa_decode_*).
ssa_status check_decode_index(const SsaRouteArgs& a, const SsaDecodeIndex* ix) {
  if (!ix) return fail(SSA_ERR_INVALID_ARG, "index is NULL");
  if (!ix->bucket_start || !ix->bucket_end || !ix->bucket_keys || !ix->min_free)
    return fail(SSA_ERR_INVALID_ARG, "bucket_start / bucket_end / bucket_keys / min_free is NULL");
  if (ix->slack < 1) return fail(SSA_ERR_INVALID_ARG, "slack %d < 1", ix->slack);
  if (ix->entry_capacity < 1 || ix->entry_capacity >= (1ll << 31))
    return fail(SSA_ERR_UNSUPPORTED, "entry_capacity must be in [1, 2^31)");
  if (a.b == 4 && !ix->bucket_codes)
    return fail(SSA_ERR_INVALID_ARG, "bucket_codes is required when codes_per_key == 4");
  if (a.b != 4 && ix->bucket_codes)
    return fail(SSA_ERR_INVALID_ARG, "bucket_codes is for codes_per_key == 4 only");
  if (ix->bucket_codes && !aligned16(ix->bucket_codes))
    return fail(SSA_ERR_ALIGNMENT, "bucket_codes must be 16-byte aligned");
  if (!a.k_codes || !aligned16(a.k_codes)) return fail(SSA_ERR_ALIGNMENT, "k_codes must be set and 16-byte aligned");
  return SSA_OK;
}

ssa::DecodeIndexParams decode_params(const SsaRouteArgs& a, const SsaDecodeIndex* ix) {
  ssa::DecodeIndexParams p{};
  p.start = ix->bucket_start;
  p.end = ix->bucket_end;
  p.keys = ix->bucket_keys;
  p.codes = reinterpret_cast<int4*>(ix->bucket_codes);
  p.min_free = ix->min_free;
  p.k_codes = a.k_codes;
  p.k_codes_sb = ix->k_codes_stride_b ? ix->k_codes_stride_b : static_cast<int64_t>(a.n) * a.h_kv * a.b;
  p.status = a.status;
  p.entry_capacity = ix->entry_capacity;
  p.batch = a.batch; p.n = a.n; p.h_kv = a.h_kv; p.b = a.b; p.n_codes = a.n_codes; p.slack = ix->slack;
  return p;
}

// Validation shared by the attention entry points; fills the kernel params.
ssa_status attn_params(const SsaAttnArgs* a, ssa::AttnParams& p) {
  if (!a) return fail(SSA_ERR_INVALID_ARG, "args is NULL");
  if (a->batch < 0 || a->n_q < 0 || a->n < 1 || a->q_offset < 0 || a->top_k < 1)
    return fail(SSA_ERR_INVALID_ARG, "bad sizes");
  if (a->h_kv < 1 || a->h_q % a->h_kv != 0)
    return fail(SSA_ERR_INVALID_ARG, "num_q_heads (%d) must be a multiple of num_kv_heads (%d)", a->h_q, a->h_kv);
  if (a->h_q / a->h_kv > 16) return fail(SSA_ERR_UNSUPPORTED, "GQA group size %d > 16", a->h_q / a->h_kv);
  if (static_cast<int64_t>(a->batch) * a->h_kv * a->n_q >= (1ll << 31))
    return fail(SSA_ERR_UNSUPPORTED, "batch * num_kv_heads * query rows must be < 2^31");
  if (a->d < 8 || a->d > 256 || a->d % 8 != 0)
    return fail(SSA_ERR_UNSUPPORTED, "head_dim %d: need a multiple of 8 in [8, 256]", a->d);
  if (!valid_dtype(a->dtype)) return fail(SSA_ERR_INVALID_ARG, "bad dtype");
  if (a->index_dtype != SSA_I32 && a->index_dtype != SSA_I64) return fail(SSA_ERR_INVALID_ARG, "bad index dtype");
  if (!a->q || !a->k || !a->v || !a->indices || !a->out) return fail(SSA_ERR_INVALID_ARG, "NULL pointer");
  if (!(a->scale != 0.f)) return fail(SSA_ERR_INVALID_ARG, "scale must be non-zero");
  if (!aligned16(a->k) || !stride16(a->k_stride_n, a->dtype) || !stride16(a->k_stride_h, a->dtype) ||
      !stride16(a->k_stride_b, a->dtype))
    return fail(SSA_ERR_ALIGNMENT, "k must be 16-byte aligned with 16-byte strides");
  p.q = a->q; p.q_sb = a->q_stride_b; p.q_sn = a->q_stride_n; p.q_sh = a->q_stride_h;
  p.k = a->k; p.k_sb = a->k_stride_b; p.k_sn = a->k_stride_n; p.k_sh = a->k_stride_h;
  p.v = a->v; p.v_sb = a->v_stride_b; p.v_sn = a->v_stride_n; p.v_sh = a->v_stride_h;
  p.idx = a->indices; p.i_sb = a->idx_stride_b; p.i_sn = a->idx_stride_n; p.i_sh = a->idx_stride_h;
  p.index_i64 = a->index_dtype == SSA_I64;
  p.out = a->out; p.o_sb = a->out_stride_b; p.o_sn = a->out_stride_n; p.o_sh = a->out_stride_h;
  p.status = a->status;
  p.batch = a->batch; p.n_q = a->n_q; p.n = a->n; p.q_offset = a->q_offset;
  p.seg = ssa::contiguous_segs(a->q_offset, a->n_q);
  p.h_kv = a->h_kv; p.group = a->h_q / a->h_kv; p.d = a->d; p.top_k = a->top_k;
  p.causal = a->causal ? 1 : 0;
  p.inv_scale = 1.0f / a->scale;
  return SSA_OK;
}

}  // namespace

extern "C" {

const char* ssa_status_str(ssa_status s) {
  switch (s) {
    case SSA_OK: return "ok";
    case SSA_ERR_INVALID_ARG: return "invalid argument";
    case SSA_ERR_UNSUPPORTED: return "unsupported size";
    case SSA_ERR_WORKSPACE: return "workspace missing or too small";
    case SSA_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case SSA_ERR_CUDA: return "CUDA error";
    case SSA_ERR_DEVICE: return "device-side error";
  }
  return "unknown status";
}

const char* ssa_last_error(void) { return g_last_error.c_str(); }

size_t ssa_route_workspace_size(const SsaRouteArgs* args) {
  if (!args) return 0;
  return route_layout(*args).total;
}

ssa_status ssa_route(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  int32_t* kc = args->k_codes ? args->k_codes : at<int32_t>(workspace, L.k_codes);
  s = run_stage1(*args, L, workspace, st, true, true, qc, kc);
  if (s != SSA_OK) return s;
  return run_stage2(*args, L, workspace, st, qc, kc);
}

ssa_status ssa_route_rope(const SsaRouteArgs* args, const SsaRopeArgs* rope, void* workspace,
                          size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  if (!rope) return fail(SSA_ERR_INVALID_ARG, "rope is NULL");
  if (!ssa::route_project_rope_supported(args->d, args->d_s, args->dtype))
    return fail(SSA_ERR_UNSUPPORTED, "route_rope needs 16-bit q/k, head_dim 64 or 128 and route_dim 8/16/32/64");
  if (!rope->cos || !rope->sin || !rope->q_out || !rope->k_out)
    return fail(SSA_ERR_INVALID_ARG, "cos / sin / q_out / k_out is NULL");
  if (rope->table_stride_b < 0 || rope->table_stride_n < args->d)
    return fail(SSA_ERR_INVALID_ARG, "bad RoPE table strides");
  if (!aligned16(rope->cos) || !aligned16(rope->sin) || !stride16(rope->table_stride_b, args->dtype) ||
      !stride16(rope->table_stride_n, args->dtype))
    return fail(SSA_ERR_ALIGNMENT, "RoPE tables must be 16-byte aligned with 16-byte strides");
  if (!aligned16(rope->q_out) || !aligned16(rope->k_out) || !stride16(rope->q_out_stride_b, args->dtype) ||
      !stride16(rope->q_out_stride_n, args->dtype) || !stride16(rope->q_out_stride_h, args->dtype) ||
      !stride16(rope->k_out_stride_b, args->dtype) || !stride16(rope->k_out_stride_n, args->dtype) ||
      !stride16(rope->k_out_stride_h, args->dtype))
    return fail(SSA_ERR_ALIGNMENT, "q_out / k_out must be 16-byte aligned with 16-byte strides");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  int32_t* kc = args->k_codes ? args->k_codes : at<int32_t>(workspace, L.k_codes);
  s = run_stage1(*args, L, workspace, st, true, true, qc, kc, rope);
  if (s != SSA_OK) return s;
  // stage 2 re-scores with the rotated rows
  SsaRouteArgs r = *args;
  r.q = rope->q_out;
  r.q_stride_b = rope->q_out_stride_b; r.q_stride_n = rope->q_out_stride_n; r.q_stride_h = rope->q_out_stride_h;
  r.k = rope->k_out;
  r.k_stride_b = rope->k_out_stride_b; r.k_stride_n = rope->k_out_stride_n; r.k_stride_h = rope->k_out_stride_h;
  return run_stage2(r, L, workspace, st, qc, kc);
}

ssa_status ssa_route_with_key_codes(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  if (!args->k_codes) return fail(SSA_ERR_INVALID_ARG, "k_codes is NULL (it is the input here)");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  s = run_stage1(*args, L, workspace, st, false, true, qc, nullptr);
  if (s != SSA_OK) return s;
  return run_stage2(*args, L, workspace, st, qc, args->k_codes);
}

ssa_status ssa_route_with_index(const SsaRouteArgs* args, const int32_t* bucket_ptr, const int32_t* bucket_keys,
                                void* workspace, size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  if (!args->k_codes || !bucket_ptr || !bucket_keys)
    return fail(SSA_ERR_INVALID_ARG, "k_codes, bucket_ptr and bucket_keys are inputs here and must be set");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  // the index comes from the caller: check it once, before any kernel trusts it
  int32_t* bad = at<int32_t>(workspace, L.flags);
  cudaError_t e = ssa::launch_validate_index(bucket_ptr, bucket_keys, static_cast<int64_t>(args->batch) * args->h_kv,
                                             args->n_codes, args->n, args->b, bad, args->status, st);
  if (e != cudaSuccess) return cuda_status(e, "validate_index");
  s = run_stage1(*args, L, workspace, st, false, true, qc, nullptr);
  if (s != SSA_OK) return s;
  return run_rescore(*args, L, workspace, st, qc, args->k_codes, bucket_ptr, bucket_keys, bad);
}

ssa_status ssa_code_assign(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes,
                           void* stream) {
  ssa_status s = check_route(args, false, false);
  if (s != SSA_OK) return s;
  if (!args->k_codes) return fail(SSA_ERR_INVALID_ARG, "k_codes is NULL");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0) return SSA_OK;
  return run_stage1(*args, L, workspace, static_cast<cudaStream_t>(stream), true, false, nullptr,
                    args->k_codes);
}

ssa_status ssa_select_from_scores(const float* scores, int64_t rows, int32_t n_cols, int32_t kk,
                                  int32_t* out_idx, void* stream) {
  if (!scores || !out_idx) return fail(SSA_ERR_INVALID_ARG, "NULL pointer");
  if (rows < 0 || n_cols < 1 || kk < 1 || kk > 32 || kk > n_cols)
    return fail(SSA_ERR_UNSUPPORTED, "need rows >= 0, 1 <= kk <= min(32, n_cols)");
  cudaError_t e = ssa::launch_select_from_scores(scores, rows, n_cols, kk, out_idx,
                                                 static_cast<cudaStream_t>(stream));
  return cuda_status(e, "select_from_scores");
}

ssa_status ssa_build_index(const SsaRouteArgs* args, const int32_t* k_codes, int32_t* bucket_ptr,
                           int32_t* bucket_keys, void* workspace, size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, false, false);
  if (s != SSA_OK) return s;
  if (!k_codes || !bucket_ptr || !bucket_keys) return fail(SSA_ERR_INVALID_ARG, "NULL pointer");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0) return SSA_OK;
  ssa::IndexParams ip = index_params(*args, L, workspace, k_codes, bucket_ptr, bucket_keys);
  return cuda_status(ssa::launch_build_index(ip, static_cast<cudaStream_t>(stream)), "build_index");
}

int64_t ssa_decode_index_capacity(int32_t max_keys, int32_t b, int32_t n_codes, int32_t slack) {
  if (max_keys < 0 || b < 1 || n_codes < 1 || slack < 1) return 0;
  return 2 * static_cast<int64_t>(max_keys) * b + static_cast<int64_t>(n_codes) * slack;
}

ssa_status ssa_decode_index_build(const SsaRouteArgs* args, const SsaDecodeIndex* index, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, false, false);
  if (s != SSA_OK) return s;
  s = check_decode_index(*args, index);
  if (s != SSA_OK) return s;
  if (!args->k_codes) return fail(SSA_ERR_INVALID_ARG, "k_codes (the cached keys' codes) is NULL");
  const int64_t need = ssa_decode_index_capacity(args->n, args->b, args->n_codes, index->slack);
  if (index->entry_capacity < need)
    return fail(SSA_ERR_WORKSPACE, "decode index holds %lld slots per (sequence, head); %d keys need %lld",
                static_cast<long long>(index->entry_capacity), args->n, static_cast<long long>(need));
  const RouteLayout L = route_layout(*args, false);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(index->min_free, 0x7f, sizeof(int32_t), st);
  if (e != cudaSuccess) return cuda_status(e, "reset min_free");
  if (args->batch == 0) return SSA_OK;
  // the packed index in the workspace, then laid out with free slots
  ssa::IndexParams ip = index_params(*args, L, workspace, args->k_codes, at<int32_t>(workspace, L.bucket_ptr),
                                     at<int32_t>(workspace, L.bucket_keys));
  if (index->k_codes_stride_b) ip.k_codes_sb = index->k_codes_stride_b;
  e = ssa::launch_build_index(ip, st);
  if (e != cudaSuccess) return cuda_status(e, "build_index");
  return cuda_status(ssa::launch_decode_index_layout(decode_params(*args, index), ip.bucket_ptr, ip.bucket_keys, st),
                     "decode_index_layout");
}

ssa_status ssa_decode_index_append(const SsaRouteArgs* args, const SsaDecodeIndex* index, int32_t first,
                                   int32_t count, void* stream) {
  ssa_status s = check_route(args, false, false);
  if (s != SSA_OK) return s;
  s = check_decode_index(*args, index);
  if (s != SSA_OK) return s;
  if (!args->k_codes) return fail(SSA_ERR_INVALID_ARG, "k_codes (the cached keys' codes) is NULL");
  if (first < 0 || count < 0 || static_cast<int64_t>(first) + count > args->n)
    return fail(SSA_ERR_INVALID_ARG, "keys %d .. %d + %d are not all among the %d cached keys", first, first, count,
                args->n);
  if (args->batch == 0 || count == 0) return SSA_OK;
  return cuda_status(ssa::launch_decode_index_append(decode_params(*args, index), first, count,
                                                     static_cast<cudaStream_t>(stream)),
                     "decode_index_append");
}

ssa_status ssa_decode_route(const SsaRouteArgs* args, const SsaDecodeIndex* index, void* workspace,
                            size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  s = check_decode_index(*args, index);
  if (s != SSA_OK) return s;
  if (!args->k_codes) return fail(SSA_ERR_INVALID_ARG, "k_codes (the cached keys' codes) is NULL");
  const RouteLayout L = route_layout(*args, false);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  s = run_stage1(*args, L, workspace, st, false, true, qc, nullptr);
  if (s != SSA_OK) return s;
  return run_rescore(*args, L, workspace, st, qc, args->k_codes, nullptr, nullptr, nullptr, index);
}

ssa_status ssa_build_index_noalloc(const SsaRouteArgs* args, const int32_t* k_codes, int32_t* bucket_ptr,
                                   int32_t* bucket_keys, void* stream) {
  ssa_status s = check_route(args, false, false);
  if (s != SSA_OK) return s;
  if (!k_codes || !bucket_ptr || !bucket_keys) return fail(SSA_ERR_INVALID_ARG, "NULL pointer");
  // the index build reads only the counts and partials regions of the layout
  const RouteLayout L = route_layout(*args);
  const size_t counts_bytes = round_up(static_cast<size_t>(args->batch) * args->h_kv * args->n_codes * L.tiles * 4);
  const size_t partial_bytes = static_cast<size_t>(args->batch) * args->h_kv * L.chunks * 4;
  if (counts_bytes + partial_bytes > kNoAllocScratchBytes)
    return fail(SSA_ERR_UNSUPPORTED,
                "index build needs %zu bytes of scratch; the allocation-free entry point holds %zu "
                "(use ssa_build_index with a workspace)",
                counts_bytes + partial_bytes, kNoAllocScratchBytes);
  void* scratch = nullptr;
  s = noalloc_scratch(&scratch);
  if (s != SSA_OK) return s;
  if (args->batch == 0) return SSA_OK;
  RouteLayout S{};
  S.counts = 0;
  S.partials = counts_bytes;
  S.tiles = L.tiles;
  S.chunks = L.chunks;
  ssa::IndexParams ip = index_params(*args, S, scratch, k_codes, bucket_ptr, bucket_keys);
  return cuda_status(ssa::launch_build_index(ip, static_cast<cudaStream_t>(stream)), "build_index_noalloc");
}

ssa_status ssa_select_candidates(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  if (!args->q_codes || !args->k_codes) return fail(SSA_ERR_INVALID_ARG, "q_codes / k_codes is NULL");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  return run_stage2(*args, L, workspace, static_cast<cudaStream_t>(stream), args->q_codes,
                    args->k_codes);
}

ssa_status ssa_route_with_index_segments(const SsaRouteArgs* args, const SsaQuerySegments* segments,
                                         const int32_t* bucket_ptr, const int32_t* bucket_keys, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  ssa::QuerySegs segs;
  s = check_segments(segments, args->n_q, args->n, segs);
  if (s != SSA_OK) return s;
  if (!args->k_codes || !bucket_ptr || !bucket_keys)
    return fail(SSA_ERR_INVALID_ARG, "k_codes, bucket_ptr and bucket_keys are inputs here and must be set");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* qc = args->q_codes ? args->q_codes : at<int32_t>(workspace, L.q_codes);
  int32_t* bad = at<int32_t>(workspace, L.flags);
  cudaError_t e = ssa::launch_validate_index(bucket_ptr, bucket_keys, static_cast<int64_t>(args->batch) * args->h_kv,
                                             args->n_codes, args->n, args->b, bad, args->status, st);
  if (e != cudaSuccess) return cuda_status(e, "validate_index");
  s = run_stage1(*args, L, workspace, st, false, true, qc, nullptr);
  if (s != SSA_OK) return s;
  return run_rescore(*args, L, workspace, st, qc, args->k_codes, bucket_ptr, bucket_keys, bad, nullptr, &segs);
}

ssa_status ssa_query_codes(const SsaRouteArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, false);
  if (s != SSA_OK) return s;
  if (!args->q_codes) return fail(SSA_ERR_INVALID_ARG, "q_codes is NULL (it is the output here)");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  return run_stage1(*args, L, workspace, static_cast<cudaStream_t>(stream), false, true, args->q_codes, nullptr);
}

ssa_status ssa_select_candidates_segments(const SsaRouteArgs* args, const SsaQuerySegments* segments,
                                          const int32_t* bucket_ptr, const int32_t* bucket_keys,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  ssa_status s = check_route(args, true, true);
  if (s != SSA_OK) return s;
  ssa::QuerySegs segs;
  s = check_segments(segments, args->n_q, args->n, segs);
  if (s != SSA_OK) return s;
  if (!args->q_codes || !args->k_codes || !bucket_ptr || !bucket_keys)
    return fail(SSA_ERR_INVALID_ARG, "q_codes, k_codes, bucket_ptr and bucket_keys are inputs here and must be set");
  const RouteLayout L = route_layout(*args);
  if (!workspace || workspace_bytes < L.total)
    return fail(SSA_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", L.total, workspace_bytes);
  if (args->batch == 0 || args->n_q == 0) return SSA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* bad = at<int32_t>(workspace, L.flags);
  cudaError_t e = ssa::launch_validate_index(bucket_ptr, bucket_keys, static_cast<int64_t>(args->batch) * args->h_kv,
                                             args->n_codes, args->n, args->b, bad, args->status, st);
  if (e != cudaSuccess) return cuda_status(e, "validate_index");
  return run_rescore(*args, L, workspace, st, args->q_codes, args->k_codes, bucket_ptr, bucket_keys, bad, nullptr,
                     &segs);
}

ssa_status ssa_sparse_attn_segments(const SsaAttnArgs* a, const SsaQuerySegments* segments, void* stream) {
  ssa::AttnParams p{};
  ssa_status s = attn_params(a, p);
  if (s != SSA_OK) return s;
  s = check_segments(segments, a->n_q, a->n, p.seg);
  if (s != SSA_OK || a->batch == 0 || a->n_q == 0) return s;
  return cuda_status(ssa::launch_sparse_attn(p, a->dtype, static_cast<cudaStream_t>(stream)), "sparse_attn");
}

ssa_status ssa_l2_read_probe(const void* buf, size_t bytes, int32_t reps, unsigned long long* sink, void* stream) {
  if (!buf || !sink) return fail(SSA_ERR_INVALID_ARG, "NULL pointer");
  if (!aligned16(buf) || bytes < 16 || reps < 1) return fail(SSA_ERR_INVALID_ARG, "need a 16-byte aligned buffer and reps >= 1");
  return cuda_status(ssa::launch_l2_read_probe(buf, bytes, reps, sink, static_cast<cudaStream_t>(stream)),
                     "l2_read_probe");
}

ssa_status ssa_sparse_attn(const SsaAttnArgs* a, void* stream) {
  ssa::AttnParams p{};
  const ssa_status s = attn_params(a, p);
  if (s != SSA_OK || a->batch == 0 || a->n_q == 0) return s;
  return cuda_status(ssa::launch_sparse_attn(p, a->dtype, static_cast<cudaStream_t>(stream)), "sparse_attn");
}

ssa_status ssa_sparse_attn_backward(const SsaAttnArgs* a, const void* d_out, void* d_q, float* d_k, float* d_v,
                                    void* stream) {
  ssa::AttnBwdParams bp{};
  const ssa_status s = attn_params(a, bp.fwd);
  if (s != SSA_OK) return s;
  if (!d_out || !d_q || !d_k || !d_v) return fail(SSA_ERR_INVALID_ARG, "NULL gradient pointer");
  if (a->d > 256) return fail(SSA_ERR_UNSUPPORTED, "head_dim %d > 256", a->d);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t acc = static_cast<size_t>(a->batch) * a->n * a->h_kv * a->d * sizeof(float);
  cudaError_t e = cudaMemsetAsync(d_k, 0, acc, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_v, 0, acc, st);
  if (e != cudaSuccess) return cuda_status(e, "zero dK / dV");
  if (a->batch == 0 || a->n_q == 0) return SSA_OK;
  bp.d_out = d_out;
  bp.d_q = d_q;
  bp.d_k = d_k;
  bp.d_v = d_v;
  bp.acc_sn = static_cast<int64_t>(a->h_kv) * a->d;
  return cuda_status(ssa::launch_sparse_attn_bwd(bp, a->dtype, st), "sparse_attn_backward");
}

}  // extern "C"
