// K2: the code -> key inverted index (per batch element and KV head).
//
// The reference evaluates "key j shares a code with query i" as a dense
// [n, h_kv, n] boolean mask (_build_candidate_mask, ssa/router.py:216-259).
// Here the same relation is stored in linear memory, as the design document
// describes (ssa_design.md:103-112): bucket c of head h holds every key j
// with c among its top-b codes, keys ascending.
//
// Three phases, all deterministic:
//   1. index_count_kernel  -- per key tile, a shared-memory histogram of
//      codes (warp-aggregated shared atomics), written to counts[bh][c][t].
//   2. scan (reduce / partials / apply) -- exclusive prefix over (c, t) per
//      (bat, h): counts become write offsets, bucket_ptr[c] = offset[c][0].
//   3. index_scatter_kernel -- each tile sorts its (code, entry) pairs in
//      shared memory (two stable radix passes of 8 bits on the code; pairs
//      are unique, so the order is fixed), then writes key j at
//      offset[c][t] + rank within its code run.
//      Keys are therefore ascending within every bucket.
#include "common.cuh"
#include "kernels.cuh"

namespace ssa {

constexpr int kIndexThreads = 512;

__global__ void __launch_bounds__(kIndexThreads) index_count_kernel(IndexParams p) {
  extern __shared__ uint32_t hist[];          // [n_codes]
  const int t = blockIdx.x;
  const int bh = blockIdx.y;                  // bat * h_kv + h
  const int h = bh % p.h_kv, bat = bh / p.h_kv;
  for (int c = threadIdx.x; c < p.n_codes; c += blockDim.x) hist[c] = 0;
  __syncthreads();
  const int j0 = t * p.tile_keys;
  const int nk = min(p.tile_keys, p.n - j0);
  const int entries = nk * p.b;
  for (int e = threadIdx.x; e < entries; e += blockDim.x) {
    const int jl = e / p.b, s = e % p.b;
    const int c = checked_code(p.k_codes[bat * p.k_codes_sb + (static_cast<int64_t>(j0 + jl) * p.h_kv + h) * p.b + s],
                               p.n_codes, p.status);
    // warp-aggregated: one shared atomic per distinct code in the warp
    const unsigned active = __activemask();
    const unsigned peers = __match_any_sync(active, c);
    const int leader = __ffs(peers) - 1;
    if ((threadIdx.x % kWarp) == leader) atomicAdd(&hist[c], __popc(peers));
  }
  __syncthreads();
  uint32_t* out = p.counts + static_cast<int64_t>(bh) * p.n_codes * p.tiles;
  for (int c = threadIdx.x; c < p.n_codes; c += blockDim.x)
    out[static_cast<int64_t>(c) * p.tiles + t] = hist[c];
}

// --- exclusive scan over counts[bh][0 .. n_codes*tiles) ----------------------
template <int THREADS>
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums,
                                                         uint32_t* total) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == kWarp - 1) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    constexpr int W = THREADS / kWarp;
    uint32_t s = lane < W ? warp_sums[lane] : 0u;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < W) warp_sums[lane] = s;      // inclusive
    if (lane == W - 1) *total = s;
  }
  __syncthreads();
  const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
  const uint32_t r = before + x - v;
  __syncthreads();
  return r;
}

constexpr int kScanThreads = 1024;
constexpr int kScanPerThread = kScanChunk / kScanThreads;

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(IndexParams p) {
  __shared__ uint32_t red[kScanThreads / kWarp];
  const int64_t len = static_cast<int64_t>(p.n_codes) * p.tiles;
  const int bh = blockIdx.y;
  const int64_t chunk = blockIdx.x;
  const uint32_t* src = p.counts + bh * len + chunk * kScanChunk;
  const int64_t rest = len - chunk * kScanChunk;
  const int64_t m = rest < kScanChunk ? rest : kScanChunk;
  uint32_t s = 0;
  for (int64_t e = threadIdx.x; e < m; e += kScanThreads) s += src[e];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = s;
  __syncthreads();
  if (threadIdx.x < kWarp) {
    s = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) p.partials[bh * p.chunks + chunk] = s;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_partials_kernel(IndexParams p) {
  __shared__ uint32_t ws[kScanThreads / kWarp];
  __shared__ uint32_t tot;
  const int bh = blockIdx.x;
  uint32_t carry = 0;
  uint32_t* part = p.partials + bh * p.chunks;
  for (int64_t base = 0; base < p.chunks; base += kScanThreads) {
    const int64_t e = base + threadIdx.x;
    const uint32_t v = e < p.chunks ? part[e] : 0u;
    const uint32_t ex = block_exclusive_scan<kScanThreads>(v, ws, &tot);
    if (e < p.chunks) part[e] = carry + ex;
    carry += tot;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(IndexParams p) {
  __shared__ uint32_t ws[kScanThreads / kWarp];
  __shared__ uint32_t tot;
  const int64_t len = static_cast<int64_t>(p.n_codes) * p.tiles;
  const int bh = blockIdx.y;
  const int64_t chunk = blockIdx.x;
  uint32_t* src = p.counts + bh * len + chunk * kScanChunk;
  const int64_t rest = len - chunk * kScanChunk;
  const int64_t m = rest < kScanChunk ? rest : kScanChunk;
  uint32_t v[kScanPerThread];
  uint32_t local = 0;
#pragma unroll
  for (int r = 0; r < kScanPerThread; ++r) {
    const int64_t e = static_cast<int64_t>(threadIdx.x) * kScanPerThread + r;
    v[r] = e < m ? src[e] : 0u;
    local += v[r];
  }
  uint32_t run = block_exclusive_scan<kScanThreads>(local, ws, &tot) + p.partials[bh * p.chunks + chunk];
  int32_t* ptr = p.bucket_ptr + static_cast<int64_t>(bh) * (p.n_codes + 1);
#pragma unroll
  for (int r = 0; r < kScanPerThread; ++r) {
    const int64_t e = static_cast<int64_t>(threadIdx.x) * kScanPerThread + r;
    if (e < m) {
      src[e] = run;
      const int64_t flat = chunk * kScanChunk + e;
      if (flat % p.tiles == 0) ptr[flat / p.tiles] = static_cast<int32_t>(run);
    }
    run += v[r];
  }
  if (chunk == 0 && threadIdx.x == 0) ptr[p.n_codes] = p.n * p.b;
}

// --- stable scatter -------------------------------------------------------
// Each tile sorts its composite keys (code << 16 | entry) in shared memory by
// a two-pass LSD radix sort on the code (8 bits a pass).  A pass is stable:
// warp w ranks its 256 consecutive keys step by step (__match_any_sync on the
// digit, per-warp digit counters), a block scan over (digit, warp) turns the
// counters into offsets, and every key moves to offset + rank.  Entries enter
// in entry order, so after both passes the keys of a code ascend.  Padding
// keys (0xffffffff) sort last.
constexpr int kRadixBins = 256;
constexpr int kScatterWarps = kIndexThreads / kWarp;                  // 16
constexpr int kPerThread = kIndexSortEntries / kIndexThreads;        // 8 keys a thread
static_assert(kPerThread * kIndexThreads == kIndexSortEntries, "tile = threads x keys a thread");

struct ScatterSmem {
  uint32_t keys[2][kIndexSortEntries];
  uint32_t cnt[kRadixBins * kScatterWarps];   // [digit][warp]
  uint32_t part[kIndexThreads];
};

__device__ __forceinline__ void radix_pass(ScatterSmem& s, const uint32_t* src, uint32_t* dst, int shift) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  for (int i = threadIdx.x; i < kRadixBins * kScatterWarps; i += blockDim.x) s.cnt[i] = 0;
  __syncthreads();
  // warp w owns keys [w * 256, w * 256 + 256): 8 steps of 32, in order
  uint32_t key[kPerThread], rank[kPerThread];
#pragma unroll
  for (int st = 0; st < kPerThread; ++st) {
    const int e = warp * (kWarp * kPerThread) + st * kWarp + lane;
    key[st] = src[e];
    const uint32_t d = (key[st] >> shift) & (kRadixBins - 1);
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    uint32_t* c = &s.cnt[d * kScatterWarps + warp];
    const uint32_t base = *c;
    rank[st] = base + __popc(peers & ((1u << lane) - 1u));
    __syncwarp();
    if (lane == __ffs(peers) - 1) *c = base + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // exclusive scan of cnt in (digit, warp) order: each thread 8 consecutive counters
  uint32_t local[kPerThread], sum = 0;
#pragma unroll
  for (int t = 0; t < kPerThread; ++t) {
    local[t] = s.cnt[threadIdx.x * kPerThread + t];
    sum += local[t];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == kWarp - 1) s.part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < kScatterWarps ? s.part[lane] : 0u, w = v;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kScatterWarps) s.part[lane] = w - v;                  // exclusive over warps
  }
  __syncthreads();
  uint32_t run = s.part[warp] + incl - sum;
#pragma unroll
  for (int t = 0; t < kPerThread; ++t) {
    s.cnt[threadIdx.x * kPerThread + t] = run;
    run += local[t];
  }
  __syncthreads();
#pragma unroll
  for (int st = 0; st < kPerThread; ++st) {
    const uint32_t d = (key[st] >> shift) & (kRadixBins - 1);
    dst[s.cnt[d * kScatterWarps + warp] + rank[st]] = key[st];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kIndexThreads) index_scatter_kernel(IndexParams p) {
  extern __shared__ __align__(16) unsigned char scatter_smem[];
  ScatterSmem& s = *reinterpret_cast<ScatterSmem*>(scatter_smem);
  const int t = blockIdx.x;
  const int bh = blockIdx.y;
  const int h = bh % p.h_kv, bat = bh / p.h_kv;
  const int j0 = t * p.tile_keys;
  const int nk = min(p.tile_keys, p.n - j0);
  const int entries = nk * p.b;
  // composite key (code << 16 | entry): unique within the tile; padding last
  for (int e = threadIdx.x; e < kIndexSortEntries; e += blockDim.x) {
    uint32_t kv = 0xffffffffu;
    if (e < entries) {
      const int jl = e / p.b, sl = e % p.b;
      const uint32_t c = static_cast<uint32_t>(checked_code(
          p.k_codes[bat * p.k_codes_sb + (static_cast<int64_t>(j0 + jl) * p.h_kv + h) * p.b + sl], p.n_codes, nullptr));
      kv = (c << 16) | static_cast<uint32_t>(e);
    }
    s.keys[0][e] = kv;
  }
  __syncthreads();
  radix_pass(s, s.keys[0], s.keys[1], 16);      // low 8 bits of the code
  radix_pass(s, s.keys[1], s.keys[0], 24);      // high 8 bits
  const uint32_t* keys = s.keys[0];
  const uint32_t* off = p.counts + static_cast<int64_t>(bh) * p.n_codes * p.tiles;
  int32_t* dst = p.bucket_keys + static_cast<int64_t>(bh) * p.n * p.b;
  for (int e = threadIdx.x; e < entries; e += blockDim.x) {
    const uint32_t kv = keys[e];
    const uint32_t c = kv >> 16;
    // first position of this code's run: lower bound of (c << 16)
    int lo = 0, hi = e;
    const uint32_t target = c << 16;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (keys[mid] < target) lo = mid + 1; else hi = mid;
    }
    const uint32_t pos = off[static_cast<int64_t>(c) * p.tiles + t] + static_cast<uint32_t>(e - lo);
    const int32_t e_tile = static_cast<int32_t>(kv & 0xffffu);
    dst[pos] = p.store_entry ? j0 * p.b + e_tile : j0 + e_tile / p.b;
  }
}

__global__ void validate_index_kernel(const int32_t* ptr, const int32_t* keys, int64_t batch_heads, int n_codes,
                                      int n, int b, int32_t* bad, int32_t* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int entries = n * b;
  bool ok = true;
  for (int64_t t = t0; t < batch_heads * (n_codes + 1); t += stride) {
    const int c = static_cast<int>(t % (n_codes + 1));
    const int v = ptr[t];
    ok &= v >= 0 && v <= entries;
    if (c > 0) ok &= ptr[t - 1] <= v;
  }
  for (int64_t t = t0; t < batch_heads * entries; t += stride) ok &= static_cast<unsigned>(keys[t]) < static_cast<unsigned>(n);
  if (!ok) {
    atomicOr(bad, 1);
    set_status(status, SSA_DEVICE_BAD_INDEX);
  }
}

__global__ void index_codes_kernel(const int32_t* keys, const int32_t* k_codes, int4* out, int64_t batch_heads,
                                   int n, int h_kv) {
  const int64_t total = batch_heads * n * 4;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t bh = e / (static_cast<int64_t>(n) * 4);
    const int64_t bat = bh / h_kv;
    const int h = static_cast<int>(bh % h_kv);
    const int j = keys[e];
    out[e] = static_cast<unsigned>(j) < static_cast<unsigned>(n)
                 ? *reinterpret_cast<const int4*>(k_codes + ((bat * n + j) * h_kv + h) * 4)
                 : make_int4(-1, -1, -1, -1);
  }
}

cudaError_t launch_index_codes(const int32_t* bucket_keys, const int32_t* k_codes, int4* bucket_codes,
                               int64_t batch_heads, int n, int h_kv, cudaStream_t st) {
  const int64_t total = batch_heads * n * 4;
  if (total == 0) return cudaSuccess;
  const int64_t blocks = cdiv(total, 256) < 148 * 8 ? cdiv(total, 256) : 148 * 8;
  index_codes_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(bucket_keys, k_codes, bucket_codes,
                                                                  batch_heads, n, h_kv);
  return cudaGetLastError();
}

cudaError_t launch_validate_index(const int32_t* bucket_ptr, const int32_t* bucket_keys, int64_t batch_heads,
                                  int n_codes, int n, int b, int32_t* bad, int32_t* status, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  validate_index_kernel<<<592, 256, 0, st>>>(bucket_ptr, bucket_keys, batch_heads, n_codes, n, b, bad, status);
  return cudaGetLastError();
}

cudaError_t launch_build_index(const IndexParams& p, cudaStream_t st) {
  const int bhs = p.batch * p.h_kv;
  if (bhs == 0 || p.n == 0) return cudaSuccess;
  const size_t hist_smem = static_cast<size_t>(p.n_codes) * sizeof(uint32_t);
  cudaFuncSetAttribute(index_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(hist_smem));
  dim3 g1(p.tiles, bhs);
  index_count_kernel<<<g1, kIndexThreads, hist_smem, st>>>(p);
  dim3 g2(static_cast<unsigned>(p.chunks), bhs);
  scan_reduce_kernel<<<g2, kScanThreads, 0, st>>>(p);
  scan_partials_kernel<<<bhs, kScanThreads, 0, st>>>(p);
  scan_apply_kernel<<<g2, kScanThreads, 0, st>>>(p);
  cudaFuncSetAttribute(index_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(sizeof(ScatterSmem)));
  index_scatter_kernel<<<g1, kIndexThreads, sizeof(ScatterSmem), st>>>(p);
  return cudaGetLastError();
}

}  // namespace ssa
